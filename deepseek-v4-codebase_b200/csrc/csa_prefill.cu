// Chunked-prefill CSA indexer on the 5th-generation tensor cores (sm_100a):
// tcgen05.mma with operands in shared memory and accumulators in TMEM.
//
// Semantics (reference itz-sayak/deepseek-v4-codebase, aether_2b/modeling.py
// :591-615): for every query token t of a prefill chunk
//   score[s] = sum_h softplus(w_h) * relu(q_h . k_s)   over the causally
//   visible compressed blocks s < t // compression (modeling.py:612-614),
// and the exact top-k (score desc, block index asc) of those blocks.  Keys
// come from the paged TurboQuant cache (codes c, per-entry scale); queries
// are rotated once (q . decode(c) = scale * (WHT(diag * q) . c)).
//
// Numerics.  The rotated query of head h is put in 22-bit fixed point,
// q_int = rint(q_rot / s_h) with s_h = max|q_rot| / 2^21, and split into two
// limbs q_int = 2048 a + b with |a|, |b| <= 1024, both exact in fp16.  Codes
// are exact in fp16 (|c| <= 127).  Each limb's 64-term dot product is an
// integer below 2^24, so the fp32 tensor-core accumulation is exact; the
// epilogue forms dot = 2048 D_a + D_b (one rounding), then
// score = (sum_h alpha_h relu(dot_h)) * scale with alpha_h = softplus(w_h) s_h.
//
// Tiling.  One CTA serves 32 query tokens of one request.  The MMA is
//   D[128 keys x 256] = A[128 keys x 64 dims] * B[256 x 64 dims]^T
// with B's 256 rows = 32 queries x 4 heads x 2 limbs, so the head sum is
// within one TMEM lane (no shuffles).  Two 256-column accumulators in TMEM
// (512 columns) let the epilogue of tile j overlap the MMAs of tile j + 1.
//
// Warp roles (512 threads):
//   warp 0       bulk (TMA) copies of the two index pages of each key tile
//   warp 1       MMA issue (one thread) and tcgen05.commit
//   warps 4-7    codes -> fp16 in the canonical no-swizzle K-major layout
//   warps 8-15   epilogue: TMEM -> registers, scores, streaming top-k
// Streaming top-k: per query a candidate buffer (key, block) with a running
// threshold T, owned by one warp; a key enters if key > T.  When a tile's
// keys would overflow the buffer (512 entries, 448 at 8-bit), the owner radix-selects
// the k-th largest (ties to the lower block index), keeps exactly k entries
// and raises T to that key; later keys equal to T lose the tie (they have
// higher block indices).  At the end the exact top-k of the buffer is
// written in ascending block order.
#include <cuda_fp8.h>

#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"

namespace aether {
namespace prefill {


// packed fp32x2 helpers (sm_100 fma.rn.f32x2: per-lane IEEE fma)
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pack_u2(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

constexpr int kThreads = 512;
constexpr int kQ = 32;                  // query tokens per CTA
constexpr int kTileKeys = 128;          // keys per MMA tile (M)
constexpr int kN = kQ * kIdxHeads * 2;  // 256 accumulator columns per tile
constexpr int kMaxK = 256;
constexpr uint32_t kLBO = 128, kSBO = 1024;  // canonical layout strides (bytes)

template <int BITS>
struct Cfg {
  static constexpr int RB = kIdxDim * BITS / 8;
  static constexpr int PB = page_bytes(RB);
  static constexpr int RAW_SLOTS = BITS == 4 ? 3 : 2;
  static constexpr int CAP = BITS == 4 ? 512 : 448;  // candidate entries per query
  static constexpr int RAW_BYTES = 2 * PB;  // two pages per 128-key tile
  static constexpr int OFF_B = 0;                               // fp16 [256][64] canonical
  static constexpr int OFF_A = OFF_B + kN * kIdxDim * 2;        // fp16 [2][128][64] canonical
  static constexpr int OFF_RAW = OFF_A + 2 * kTileKeys * kIdxDim * 2;
  static constexpr int OFF_SCL = OFF_RAW + RAW_SLOTS * ((RAW_BYTES + 127) & ~127);  // fp32 [4][128]
  static constexpr int OFF_BUF = OFF_SCL + 4 * kTileKeys * 4;   // uint2 [32][CAP]
  static constexpr int OFF_X = OFF_BUF + kQ * CAP * 8;         // u32 [32][128] score exchange
  static constexpr int OFF_MISC = OFF_X + kQ * kTileKeys * 4;
  static constexpr int SMEM = OFF_MISC + 2048;
  static_assert(SMEM <= 232448, "shared memory");
  static_assert(OFF_MISC % 16 == 0 && OFF_BUF % 16 == 0 && OFF_SCL % 16 == 0, "alignment");
};

struct alignas(16) Misc {
  float alpha[kQ][kIdxHeads];  // first: read as float4
  uint64_t raw_full[3], raw_empty[3], a_full[2], a_empty[2], acc_full[2], acc_empty[2];
  uint32_t tmem;
  int abort_flag;
  int ntiles;
  int vis[kQ];
  uint32_t thr[kQ];  // per-query threshold and buffer count (owned by one warp)
  uint32_t cnt[kQ];
  uint32_t lut8[16];
};
static_assert(sizeof(Misc) <= 2048, "misc area");

struct Params {
  const float* index_q;    // [Qtot][4][64]
  const float* index_w;    // [Qtot][4]
  const uint8_t* idx_pages;
  const int32_t* page_table;
  const int32_t* req_info;  // [R][4]: first query row, query count, position of query 0, blocks in cache
  const int32_t* tiles;     // [ntiles][2]: request, first query within the request
  const float* diag_idx;
  uint32_t* cand_keys;      // [Qtot][top_k]
  int32_t* cand_ids;        // [Qtot][top_k]
  int* err;
  long long* dbg;  // per-CTA phase clocks [grid][16] (profiling aid), or null
  int table_stride, num_pages, compression, top_k;
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((kLBO >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((kSBO >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // sm100 descriptor version; no swizzle, base offset 0
  return d;
}
// kind::f16 instruction descriptor: D f32, A and B f16, both K-major, N x M
__host__ __device__ constexpr uint32_t umma_idesc(int n, int m) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
// byte offset of element (row r, k) in the canonical no-swizzle K-major layout
__device__ __forceinline__ uint32_t canon(int r, int k) {
  return (r >> 3) * kSBO + (k >> 3) * kLBO + (r & 7) * 16 + (k & 7) * 2;
}
// The e4m3 indexer (F8): 64-dim rows of 8-bit elements are 4 core matrices
// of 16 elements, so the 8-row group stride is 512 bytes
constexpr uint32_t kSBO8 = 512;
constexpr int kN8 = kQ * kIdxHeads;  // 128 accumulator columns per tile: (query, head)
__device__ __forceinline__ uint32_t canon8(int r, int k) {
  return (r >> 3) * kSBO8 + (k >> 4) * kLBO + (r & 7) * 16 + (k & 15);
}
__device__ __forceinline__ uint64_t umma_desc8(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((kLBO >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((kSBO8 >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}
// e4m3 bytes of two floats (saturating, round to nearest even)
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ void mbar_arrive_cta(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait; a timeout sets the CTA's abort flag so every role winds down.
// `backoff` roles (producer, MMA issue, conversion) sleep between polls so
// their waiting leaves the issue slots to the epilogue warps.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Misc* m, int* err,
                                              bool backoff = false) {
  if (*reinterpret_cast<volatile int*>(&m->abort_flag)) return false;
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int it = 0; it < 16; ++it) {
      if (mbar_try_wait(addr, parity)) return true;
      if (backoff) __nanosleep(64);
    }
    if (*reinterpret_cast<volatile int*>(&m->abort_flag)) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  report_error(err, kErrWaitTimeout);
  *reinterpret_cast<volatile int*>(&m->abort_flag) = 1;
  return false;
}
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// nibble pair of one byte -> half2(lo, hi), exact signed values
__device__ __forceinline__ uint32_t nib2h2(uint32_t byte) {
  uint32_t y = (byte & 0xFu) | ((byte & 0xF0u) << 12);
  y = (y ^ 0x00080008u) | 0x64006400u;  // 1024 + (v + 8)
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));  // - 1032
  return *reinterpret_cast<uint32_t*>(&h);
}
// two int8 codes (low 16 bits of w) -> half2
__device__ __forceinline__ uint32_t s8x2h2(uint32_t w) {
  uint32_t y = __byte_perm(w ^ 0x8080u, 0x64646464u, 0x5140);  // 1024 + (v + 128)
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));  // - 1152
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------- selection
// One warp: the K-th largest key of n <= CAP entries (key desc, block asc),
// keeping exactly min(K, n) of them at the front of buf (order not kept).
// Returns the threshold key.  With slack > 0 (streaming prunes) the radix
// walk stops as soon as the keys at or above the current prefix number at
// most K + slack: those are all kept, the returned threshold is that prefix
// and *kept their count.  Every key of the exact top-K is among them, and a
// later key equal to the threshold cannot enter the top-K (at least K kept
// keys are >= it with lower block indices), so insertion stays "key > thr".  The keys sit in registers (16 per lane) and
// an MSB-first bitwise radix select counts matches with warp reductions:
// no shared-memory atomics, which serialise when keys share their top bits.
template <int CAP>
__device__ __forceinline__ uint32_t warp_prune(uint2* buf, int n, int K, int lane, int slack = 0,
                                               int* kept = nullptr) {
  constexpr int PER = CAP / 32;
  uint32_t kk[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int idx = i * 32 + lane;
    kk[i] = idx < n ? buf[idx].x : 0u;  // 0 never matches: real keys are >= 1
  }
  // bits shared by every real key need no radix step: start below the
  // highest bit where two keys differ
  uint32_t kor = 0, kand = 0xFFFFFFFFu;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    if (i * 32 + lane < n) {
      kor |= kk[i];
      kand &= kk[i];
    }
  }
  kor = __reduce_or_sync(0xffffffffu, kor);
  kand = __reduce_and_sync(0xffffffffu, kand);
  const uint32_t diff = kor ^ kand;
  const int top = diff ? 31 - __clz(diff) : -1;
  uint32_t prefix = top >= 31 ? 0u : (kand & ~((2u << top) - 1u)), R = static_cast<uint32_t>(K);
  if (top < 0) prefix = kand;  // all keys equal
  uint32_t inrange = static_cast<uint32_t>(n);  // keys matching prefix on the bits walked so far
  bool early = false;
#pragma unroll 1
  for (int bit = top; bit >= 0; --bit) {
    const uint32_t want = prefix | (1u << bit), hm = ~((1u << bit) - 1u);
    uint32_t c = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) c += (kk[i] & hm) == want;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= R) {
      prefix = want;
      inrange = c;
    } else {
      R -= c;
      inrange -= c;
    }
    // keys >= prefix (lower bits zero): the K - R above the range and the range itself
    if (slack > 0 && static_cast<uint32_t>(K) - R + inrange <= static_cast<uint32_t>(K + slack)) {
      early = true;
      break;
    }
  }
  if (early) {  // keep every key >= prefix
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (i * 32 >= n) break;
      const bool keep = i * 32 + lane < n && kk[i] >= prefix;
      const uint2 e = keep ? buf[i * 32 + lane] : make_uint2(0, 0);
      const uint32_t bal = __ballot_sync(0xffffffffu, keep);
      __syncwarp();
      if (keep) buf[out + __popc(bal & ((1u << lane) - 1u))] = e;
      out += __popc(bal);
      __syncwarp();
    }
    if (kept) *kept = static_cast<int>(out);
    return prefix;
  }
  if (kept) *kept = min(K, n);
  const uint32_t thr = prefix, take_eq = R;
  uint32_t eq = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) eq += kk[i] == thr;
  eq = __reduce_add_sync(0xffffffffu, eq);
  // keep flags first, then an in-order compaction whose writes never pass
  // the reads of the same round
  uint32_t keepm = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    bool keep = kk[i] > thr;
    if (kk[i] == thr) {
      if (eq <= take_eq) {
        keep = true;
      } else {  // equal keys beyond take_eq: keep the lowest block indices
        const uint32_t my = buf[i * 32 + lane].y;
        uint32_t before = 0;
        for (int j = 0; j < n; ++j) {
          const uint2 o = buf[j];
          before += o.x == thr && o.y < my;
        }
        keep = before < take_eq;
      }
    }
    keepm |= static_cast<uint32_t>(keep) << i;
  }
  __syncwarp();
  uint32_t out = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    if (i * 32 >= n) break;
    const bool keep = (keepm >> i) & 1u;
    const uint2 e = keep ? buf[i * 32 + lane] : make_uint2(0, 0);
    const uint32_t bal = __ballot_sync(0xffffffffu, keep);
    __syncwarp();
    if (keep) buf[out + __popc(bal & ((1u << lane) - 1u))] = e;
    out += __popc(bal);
    __syncwarp();
  }
  return thr;
}

template <int CAP>
__device__ __noinline__ uint32_t warp_prune_call(uint2* buf, int n, int K, int lane) {
  return warp_prune<CAP>(buf, n, K, lane);
}

template <int BITS, bool F8 = false>
__global__ void __launch_bounds__(kThreads, 1) csa_prefill_index_kernel(Params p) {
  using C = Cfg<BITS>;
  extern __shared__ __align__(1024) uint8_t smem[];
  Misc* m = reinterpret_cast<Misc*>(smem + C::OFF_MISC);
  uint2* cbuf = reinterpret_cast<uint2*>(smem + C::OFF_BUF);
  float* sscl = reinterpret_cast<float*>(smem + C::OFF_SCL);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto stamp = [&](int slot) {
    if (p.dbg) p.dbg[blockIdx.x * 16 + slot] = clock64();
  };
  if (tid == 0) stamp(0);
  const int req = p.tiles[blockIdx.x * 2], q0 = p.tiles[blockIdx.x * 2 + 1];
  const int row0 = p.req_info[req * 4], nq = p.req_info[req * 4 + 1];
  const int pos0 = p.req_info[req * 4 + 2], nblk = p.req_info[req * 4 + 3];
  const int32_t* ptab = p.page_table + static_cast<long long>(req) * p.table_stride;

  if (tid == 0) {
    for (int i = 0; i < C::RAW_SLOTS; ++i) {
      mbar_init(&m->raw_full[i], 1);
      mbar_init(&m->raw_empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&m->a_full[i], 128);
      mbar_init(&m->a_empty[i], 1);
      mbar_init(&m->acc_full[i], 1);
      mbar_init(&m->acc_empty[i], 8);
    }
    m->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&m->tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  uint32_t* lut8 = m->lut8;  // F8: signed 4-bit code -> e4m3 byte
  if (F8 && tid < 16) lut8[tid] = e4m3x2(static_cast<float>(static_cast<int>(tid ^ 8u) - 8), 0.f) & 0xFFu;
  // ---- prologue: rotated fixed-point query limbs (B operand), head weights
  // and causal limits; one warp per (query, head)
  for (int v = warp; v < kQ * kIdxHeads; v += kThreads / 32) {
    const int qi = v >> 2, h = v & 3;
    const int q = q0 + qi;
    const bool valid = q < nq;
    float x0 = 0.f, x1 = 0.f, w = 0.f;
    if (valid) {
      const float* src = p.index_q + (static_cast<long long>(row0 + q) * kIdxHeads + h) * kIdxDim;
      x0 = src[2 * lane] * p.diag_idx[2 * lane];
      x1 = src[2 * lane + 1] * p.diag_idx[2 * lane + 1];
      w = p.index_w[static_cast<long long>(row0 + q) * kIdxHeads + h];
    }
    {  // normalised 64-point WHT, 2 values per lane
      const float a = x0, b = x1;
      x0 = a + b;
      x1 = a - b;
    }
#pragma unroll
    for (int ld = 1; ld < 32; ld <<= 1) {
      const bool up = (lane & ld) != 0;
      const float o0 = __shfl_xor_sync(0xffffffffu, x0, ld), o1 = __shfl_xor_sync(0xffffffffu, x1, ld);
      x0 = up ? o0 - x0 : x0 + o0;
      x1 = up ? o1 - x1 : x1 + o1;
    }
    x0 *= 0.125f;
    x1 *= 0.125f;
    const float am = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
    if constexpr (F8) {
      // e4m3 query, one scale per (query, head): the largest element maps to
      // 448, the largest finite e4m3 value; B row (query, head)
      const float s8 = am > 0.f ? am / 448.0f : 1.0f;
      const uint32_t b2 = valid ? e4m3x2(x0 / s8, x1 / s8) : 0u;
      *reinterpret_cast<uint16_t*>(smem + C::OFF_B + canon8(qi * kIdxHeads + h, 2 * lane)) =
          static_cast<uint16_t>(b2);
      if (lane == 0) m->alpha[qi][h] = valid ? softplus_f(w) * s8 : 0.f;
      continue;
    }
    const float s = am > 0.f ? am / 2097152.0f : 1.0f;  // 2^21
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int qint = valid ? __float2int_rn(__fdiv_rn(k ? x1 : x0, s)) : 0;
      const int a = (qint + 1024) >> 11, b = qint - a * 2048;
      const int d = 2 * lane + k;
      // B row (query pair, head, limb, query & 1): the two queries of a pair
      // sit in adjacent accumulator columns, so the epilogue pairs them in
      // packed fp32 FMAs
      const int n0 = ((qi >> 1) * kIdxHeads + h) * 4 + (qi & 1), nb = n0 + 2;
      *reinterpret_cast<__half*>(smem + C::OFF_B + canon(n0, d)) = __int2half_rn(a);
      *reinterpret_cast<__half*>(smem + C::OFF_B + canon(nb, d)) = __int2half_rn(b);
    }
    if (lane == 0) m->alpha[qi][h] = valid ? softplus_f(w) * s : 0.f;
  }
  if (tid < kQ) {
    const int q = q0 + tid;
    m->vis[tid] = q < nq ? min(nblk, (pos0 + q) / p.compression) : 0;
    m->thr[tid] = 0;
    m->cnt[tid] = 0;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B operand -> tensor core
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (tid == 0) {
    int mv = 0;
    for (int i = 0; i < kQ; ++i) mv = max(mv, m->vis[i]);
    m->ntiles = (mv + kTileKeys - 1) / kTileKeys;
  }
  __syncthreads();
  const int ntiles = m->ntiles;
  const uint32_t tmem = m->tmem;
  if (tid == 0) stamp(1);

  if (warp == 0) {
    // ------------------------------------------------ page producer
    if (lane == 0) {
      const int npages = min((nblk + kPage - 1) / kPage, p.table_stride);
      for (int j = 0; j < ntiles; ++j) {
        const int slot = j % C::RAW_SLOTS, use = j / C::RAW_SLOTS;
        if (use > 0 && !wait_or_abort(&m->raw_empty[slot], (use - 1) & 1, m, p.err, true)) break;
        uint8_t* dst = smem + C::OFF_RAW + slot * ((C::RAW_BYTES + 127) & ~127);
        const int np = min(2, npages - 2 * j);
        mbar_expect_tx(&m->raw_full[slot], static_cast<uint32_t>(max(np, 0) * C::PB));
        for (int k = 0; k < np; ++k) {
          int phys = ptab[2 * j + k];
          if (phys < 0 || phys >= p.num_pages) {
            report_error(p.err, kErrBadPage);
            phys = 0;
          }
          bulk_g2s(dst + k * C::PB, p.idx_pages + static_cast<long long>(phys) * C::PB, C::PB, &m->raw_full[slot]);
        }
      }
      stamp(2);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(F8 ? kN8 : kN, kTileKeys);
      const uint32_t sB = smem_u32(smem + C::OFF_B);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1, use = j >> 1;
        if (!wait_or_abort(&m->a_full[st], use & 1, m, p.err, true)) break;
        if (use > 0 && !wait_or_abort(&m->acc_empty[st], (use - 1) & 1, m, p.err, true)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sA = smem_u32(smem + C::OFF_A + st * kTileKeys * kIdxDim * 2);
        const uint32_t dt = tmem + st * kN;
        if constexpr (F8) {
#pragma unroll
          for (int kk = 0; kk < kIdxDim / 32; ++kk) {  // 32 e4m3 elements = 2 core matrices per step
            const uint64_t da = umma_desc8(sA + kk * 2 * kLBO), db = umma_desc8(sB + kk * 2 * kLBO);
            asm volatile(
                "{ .reg .pred p; setp.ne.u32 p, %4, 0;\n"
                "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }" ::"r"(dt),
                "l"(da), "l"(db), "r"(idesc), "r"(static_cast<uint32_t>(kk)));
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < kIdxDim / 16; ++kk) {
            const uint64_t da = umma_desc(sA + kk * 2 * kLBO), db = umma_desc(sB + kk * 2 * kLBO);
            asm volatile(
                "{ .reg .pred p; setp.ne.u32 p, %4, 0;\n"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(dt),
                "l"(da), "l"(db), "r"(idesc), "r"(static_cast<uint32_t>(kk)));
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&m->a_empty[st]))
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&m->acc_full[st]))
                     : "memory");
      }
      stamp(3);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------ code conversion
    const int r = tid - 128;  // key row of the tile
    for (int j = 0; j < ntiles; ++j) {
      const int slot = j % C::RAW_SLOTS, ruse = j / C::RAW_SLOTS, st = j & 1, ause = j >> 1;
      if (!wait_or_abort(&m->raw_full[slot], ruse & 1, m, p.err, true)) break;
      if (ause > 0 && !wait_or_abort(&m->a_empty[st], (ause - 1) & 1, m, p.err, true)) break;
      const uint8_t* page = smem + C::OFF_RAW + slot * ((C::RAW_BYTES + 127) & ~127) + (r >> 6) * C::PB;
      const uint8_t* row = page + (r & 63) * C::RB;
      uint8_t* A = smem + C::OFF_A + st * kTileKeys * kIdxDim * 2;
      if constexpr (F8) {
        // codes -> e4m3: exact for the 4-bit range [-8, 7], rounded for 8-bit
#pragma unroll
        for (int c = 0; c < kIdxDim / 16; ++c) {  // 16 dims per 16-byte chunk
          uint32_t o[4];
          if (BITS == 4) {
            const uint2 w = *reinterpret_cast<const uint2*>(row + 8 * c);
            const uint32_t wb[2] = {w.x, w.y};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t b0 = (wb[i >> 1] >> (16 * (i & 1))) & 0xFFu, b1 = (wb[i >> 1] >> (16 * (i & 1) + 8)) & 0xFFu;
              o[i] = lut8[b0 & 15u] | (lut8[b0 >> 4] << 8) | (lut8[b1 & 15u] << 16) | (lut8[b1 >> 4] << 24);
            }
          } else {
            const uint4 w = *reinterpret_cast<const uint4*>(row + 16 * c);
            const uint32_t wb[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int8_t* c8 = reinterpret_cast<const int8_t*>(&wb[i]);
              o[i] = e4m3x2(c8[0], c8[1]) | (e4m3x2(c8[2], c8[3]) << 16);
            }
          }
          *reinterpret_cast<uint4*>(A + canon8(r, 16 * c)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      } else if (BITS == 4) {
        const uint4 v0 = *reinterpret_cast<const uint4*>(row), v1 = *reinterpret_cast<const uint4*>(row + 16);
        const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int g = 0; g < 8; ++g)  // 8 dims = 4 bytes per core-matrix row
          *reinterpret_cast<uint4*>(A + canon(r, 8 * g)) =
              make_uint4(nib2h2(wv[g] & 0xFFu), nib2h2((wv[g] >> 8) & 0xFFu), nib2h2((wv[g] >> 16) & 0xFFu),
                         nib2h2(wv[g] >> 24));
      } else {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint4 v = *reinterpret_cast<const uint4*>(row + 16 * g);
          *reinterpret_cast<uint4*>(A + canon(r, 16 * g)) =
              make_uint4(s8x2h2(v.x & 0xFFFFu), s8x2h2(v.x >> 16), s8x2h2(v.y & 0xFFFFu), s8x2h2(v.y >> 16));
          *reinterpret_cast<uint4*>(A + canon(r, 16 * g + 8)) =
              make_uint4(s8x2h2(v.z & 0xFFFFu), s8x2h2(v.z >> 16), s8x2h2(v.w & 0xFFFFu), s8x2h2(v.w >> 16));
        }
      }
      sscl[(j & 3) * kTileKeys + r] = *reinterpret_cast<const float*>(page + kPage * C::RB + (r & 63) * 4);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_cta(&m->a_full[st]);
      mbar_arrive_cta(&m->raw_empty[slot]);
    }
    if (tid == 128) stamp(4);
  } else if (warp >= 8) {
    // ------------------------------------------------ epilogue + top-k
    // Each quad-warp turns its 32 keys x 16 queries of TMEM into score keys
    // and writes them to the exchange area; after one barrier warp e owns
    // queries 4e .. 4e + 3 for all 128 keys of the tile: it appends the keys
    // above each query's threshold to that query's buffer and prunes it,
    // with the threshold and count in registers.  Two barriers per tile
    // order the exchange area's writes and reads.
    const int e = warp - 8;                    // 0..7
    const int quad = warp & 3, half = e >> 2;  // TMEM lanes 32 quad.., queries 16 half..
    const int r = 32 * quad + lane;            // key row of the tile
    uint32_t* xbuf = reinterpret_cast<uint32_t*>(smem + C::OFF_X);
    long long t_wait = 0, t_ld = 0, t_ins = 0, t_prune = 0;
    int nprune = 0;
    // threshold, buffer count and causal limit of this warp's four queries
    // (owner phase), kept in registers for the whole stream
    uint32_t thr_r[4] = {0u, 0u, 0u, 0u}, cnt_r[4] = {0u, 0u, 0u, 0u};
    int vis_r[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) vis_r[qq] = m->vis[4 * e + qq];
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1, use = j >> 1;
      long long c0 = clock64();
      // a timed-out wait sets the abort flag; all epilogue warps leave
      // together after the next named barrier
      const bool got = wait_or_abort(&m->acc_full[st], use & 1, m, p.err);
      if (!got) {
        named_sync(1, 256);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      long long c1 = clock64();
      t_wait += c1 - c0;
      const float kscale = sscl[(j & 3) * kTileKeys + r];
      uint32_t* xo = xbuf;
      if constexpr (F8) {  // 64 columns: (query, head) of this half's 16 queries
        uint32_t v[64];
        const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) + st * kN + half * 64;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,"
            "%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, "
            "[%64];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]),
              "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]),
              "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]), "=r"(v[49]),
              "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]),
              "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
            : "r"(ta));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int qq = 0; qq < 16; ++qq) {
          const int qa = half * 16 + qq;
          const float4 a = *reinterpret_cast<const float4*>(m->alpha[qa]);
          float sc = a.x * fmaxf(__uint_as_float(v[4 * qq]), 0.f);
          sc = fmaf(a.y, fmaxf(__uint_as_float(v[4 * qq + 1]), 0.f), sc);
          sc = fmaf(a.z, fmaxf(__uint_as_float(v[4 * qq + 2]), 0.f), sc);
          sc = fmaf(a.w, fmaxf(__uint_as_float(v[4 * qq + 3]), 0.f), sc);
          xo[qa * kTileKeys + r] = __float_as_uint(__fmul_rn(sc, kscale)) + 1u;
        }
      }
#pragma unroll
      for (int c2 = 0; c2 < (F8 ? 0 : 2); ++c2) {  // 2 x 64 columns = 8 queries each
        uint32_t v[64];
        const uint32_t ta = tmem + (static_cast<uint32_t>(32 * quad) << 16) + st * kN + half * 128 + c2 * 64;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,"
            "%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, "
            "[%64];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]),
              "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]),
              "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]), "=r"(v[49]),
              "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]),
              "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
            : "r"(ta));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        // two queries per packed fp32 FMA (fma.rn.f32x2): each lane rounds
        // exactly as the scalar fmaf(2048, D_a, D_b), fmaf(alpha, relu, acc)
        // sequence, so the keys are bit-identical to the oracle's
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          const int qa = half * 16 + c2 * 8 + 2 * pp;
          const float4 a0 = *reinterpret_cast<const float4*>(m->alpha[qa]);
          const float4 a1 = *reinterpret_cast<const float4*>(m->alpha[qa + 1]);
          const float al0[4] = {a0.x, a0.y, a0.z, a0.w}, al1[4] = {a1.x, a1.y, a1.z, a1.w};
          uint64_t sc2 = pack_f2(0.f, 0.f);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint32_t* vv = v + pp * 16 + h * 4;
            const uint64_t dot2 = fma_f2(pack_f2(2048.f, 2048.f), pack_u2(vv[0], vv[1]), pack_u2(vv[2], vv[3]));
            float d0, d1;
            unpack_f2(dot2, d0, d1);
            sc2 = fma_f2(pack_f2(al0[h], al1[h]), pack_f2(fmaxf(d0, 0.f), fmaxf(d1, 0.f)), sc2);
          }
          float s0, s1;
          unpack_f2(sc2, s0, s1);
          xo[qa * kTileKeys + r] = __float_as_uint(__fmul_rn(s0, kscale)) + 1u;
          xo[(qa + 1) * kTileKeys + r] = __float_as_uint(__fmul_rn(s1, kscale)) + 1u;
        }
      }
      // this warp's TMEM reads are done: the accumulator may be overwritten
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(&m->acc_empty[st]);
      named_sync(1, 256);
      long long c2 = clock64();
      t_ld += c2 - c1;
      if (*reinterpret_cast<volatile int*>(&m->abort_flag)) break;
      // owner phase: queries 4e .. 4e + 3, all 128 keys of the tile; the
      // four queries are processed side by side (independent latency chains)
      {
        uint32_t kv[4][4], pm[4], npass[4];
        uint32_t (&thrq)[4] = thr_r, (&cntq)[4] = cnt_r;
        const int(&visq)[4] = vis_r;
        const int b0 = j * kTileKeys + 4 * lane;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int qi = 4 * e + qq;
          const uint4 v4 = *reinterpret_cast<const uint4*>(xo + qi * kTileKeys + 4 * lane);
          kv[qq][0] = v4.x; kv[qq][1] = v4.y; kv[qq][2] = v4.z; kv[qq][3] = v4.w;
        }
        uint32_t bal[4][4];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          pm[qq] = 0;
          npass[qq] = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool ps = b0 + i < visq[qq] && kv[qq][i] > thrq[qq];
            pm[qq] |= static_cast<uint32_t>(ps) << i;
            bal[qq][i] = __ballot_sync(0xffffffffu, ps);
            npass[qq] += __popc(bal[qq][i]);
          }
        }
        // rare: a buffer would overflow -> prune it (one inlined call site),
        // then re-evaluate all four queries against the new thresholds
        uint32_t need = 0;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) need |= static_cast<uint32_t>(cntq[qq] + npass[qq] > C::CAP) << qq;
        if (need) {
          const long long cp0 = clock64();
          for (uint32_t mk = need; mk; mk &= mk - 1u) {
            const int qq = __ffs(mk) - 1, qi = 4 * e + qq;
            // register arrays indexed without local memory
            const int n = static_cast<int>(qq == 0 ? cntq[0] : qq == 1 ? cntq[1] : qq == 2 ? cntq[2] : cntq[3]);
            // a tile adds at most kTileKeys keys: the slack keeps that much room
            const int slack = max(0, min(32, C::CAP - p.top_k - kTileKeys));
            int kept = 0;
            const uint32_t t = warp_prune<C::CAP>(cbuf + qi * C::CAP, n, p.top_k, lane, slack, &kept);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (k == qq) {
                thrq[k] = t;
                cntq[k] = static_cast<uint32_t>(kept);
              }
            ++nprune;
            __syncwarp();
          }
          t_prune += clock64() - cp0;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            pm[qq] = 0;
            npass[qq] = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const bool ps = b0 + i < visq[qq] && kv[qq][i] > thrq[qq];
              pm[qq] |= static_cast<uint32_t>(ps) << i;
              bal[qq][i] = __ballot_sync(0xffffffffu, ps);
              npass[qq] += __popc(bal[qq][i]);
            }
          }
        }
        // append in block order (lane-major, then the lane's 4 keys)
        const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          if (npass[qq] == 0) continue;  // warp-uniform: nothing passes (the common case late on)
          uint2* qb = cbuf + (4 * e + qq) * C::CAP;
          uint32_t pos = cntq[qq] + __popc(bal[qq][0] & lt) + __popc(bal[qq][1] & lt) + __popc(bal[qq][2] & lt) +
                         __popc(bal[qq][3] & lt);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if ((pm[qq] >> i) & 1u) qb[pos++] = make_uint2(kv[qq][i], static_cast<uint32_t>(b0 + i));
          cntq[qq] += npass[qq];
        }
        __syncwarp();  // appends land before the next tile's prunes read them
      }
      t_ins += clock64() - c2;
      named_sync(1, 256);  // the exchange area is rewritten by the next tile
    }
    if (lane < 4) {
      m->thr[4 * e + lane] = lane == 0 ? thr_r[0] : lane == 1 ? thr_r[1] : lane == 2 ? thr_r[2] : thr_r[3];
      m->cnt[4 * e + lane] = lane == 0 ? cnt_r[0] : lane == 1 ? cnt_r[1] : lane == 2 ? cnt_r[2] : cnt_r[3];
    }
    __syncwarp();
    if (tid == 256 && p.dbg) {
      p.dbg[blockIdx.x * 16 + 8] = t_wait;
      p.dbg[blockIdx.x * 16 + 9] = t_ld;
      p.dbg[blockIdx.x * 16 + 10] = t_ins;
      p.dbg[blockIdx.x * 16 + 12] = nprune;
      p.dbg[blockIdx.x * 16 + 11] = t_prune;
      p.dbg[blockIdx.x * 16 + 5] = clock64();
    }
    // ---- final exact top-k per query, written in ascending block order
    const bool ok = !*reinterpret_cast<volatile int*>(&m->abort_flag);
#pragma unroll 1
    for (int qq = 0; qq < 4; ++qq) {
      const int qi = 4 * e + qq, q = q0 + qi;
      if (q >= nq) continue;
      uint2* b = cbuf + qi * C::CAP;
      int n = ok ? min(static_cast<int>(m->cnt[qi]), C::CAP) : 0;
      const int K = min(p.top_k, m->vis[qi]);
      if (n > K) {
        warp_prune_call<C::CAP>(b, n, K, lane);
        n = K;
      }
      __syncwarp();
      uint32_t* ok_keys = p.cand_keys + static_cast<long long>(row0 + q) * p.top_k;
      int32_t* ok_ids = p.cand_ids + static_cast<long long>(row0 + q) * p.top_k;
      for (int i = lane; i < n; i += 32) {  // rank by block index (distinct)
        const uint2 me = b[i];
        int rank = 0;
        for (int k2 = 0; k2 < n; ++k2) rank += b[k2].y < me.y;
        ok_keys[rank] = me.x;
        ok_ids[rank] = static_cast<int32_t>(me.y);
      }
      for (int i = n + lane; i < p.top_k; i += 32) {
        ok_keys[i] = 0u;
        ok_ids[i] = -1;
      }
    }
  }
  // ---- teardown: every role is done with TMEM
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0) stamp(6);
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

static long long* g_debug = nullptr;

template <int BITS, bool F8>
static int launch(const Params& p, int ntiles, cudaStream_t st) {
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(csa_prefill_index_kernel<BITS, F8>), Cfg<BITS>::SMEM,
                                "csa_prefill"))
    return rc;
  csa_prefill_index_kernel<BITS, F8><<<ntiles, kThreads, Cfg<BITS>::SMEM, st>>>(p);
  return check_launch(F8 ? "csa_prefill_topk_fp8" : "csa_prefill_topk");
}

}  // namespace prefill
}  // namespace aether

using namespace aether;

extern "C" int aether_csa_prefill_topk(const float* index_q, const float* index_w, const uint8_t* idx_pages,
                                       const int32_t* page_table, int table_stride, int num_pages,
                                       const int32_t* req_info, const int32_t* tiles, int ntiles, int compression,
                                       const float* diag_idx, int bits, int top_k, uint32_t* cand_keys,
                                       int32_t* cand_ids, int* err, void* stream) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(top_k >= 1 && top_k <= prefill::kMaxK, "top_k must be in [1, %d], got %d", prefill::kMaxK, top_k);
  AETHER_REQUIRE(compression >= 1, "compression must be positive");
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  AETHER_REQUIRE(ntiles >= 0, "negative tile count");
  if (ntiles == 0) return 0;
  prefill::Params p{index_q, index_w, idx_pages, page_table, req_info, tiles, diag_idx, cand_keys, cand_ids, err,
                    prefill::g_debug, table_stride, num_pages, compression, top_k};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return bits == 4 ? prefill::launch<4, false>(p, ntiles, st) : prefill::launch<8, false>(p, ntiles, st);
}

// As aether_csa_prefill_topk, with the scores computed on e4m3 operands
// (tcgen05 kind::f8f6f4): the rotated index query is quantised to e4m3 per
// (query, head), 4-bit codes are exact in e4m3 and 8-bit codes are rounded to
// it.  The selection is the exact top-k of these approximate scores, so it
// agrees with the exact indexer only up to a recall below 1.
extern "C" int aether_csa_prefill_topk_fp8(const float* index_q, const float* index_w, const uint8_t* idx_pages,
                                           const int32_t* page_table, int table_stride, int num_pages,
                                           const int32_t* req_info, const int32_t* tiles, int ntiles,
                                           int compression, const float* diag_idx, int bits, int top_k,
                                           uint32_t* cand_keys, int32_t* cand_ids, int* err, void* stream) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(top_k >= 1 && top_k <= prefill::kMaxK, "top_k must be in [1, %d], got %d", prefill::kMaxK, top_k);
  AETHER_REQUIRE(compression >= 1, "compression must be positive");
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  AETHER_REQUIRE(ntiles >= 0, "negative tile count");
  if (ntiles == 0) return 0;
  prefill::Params p{index_q, index_w, idx_pages, page_table, req_info, tiles, diag_idx, cand_keys, cand_ids, err,
                    prefill::g_debug, table_stride, num_pages, compression, top_k};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return bits == 4 ? prefill::launch<4, true>(p, ntiles, st) : prefill::launch<8, true>(p, ntiles, st);
}

// Profiling aid: when buf is non-null, later prefill launches record per-CTA
// SM-clock phase stamps and per-phase cycle totals into buf[cta * 16 + i].
extern "C" void aether_csa_prefill_set_debug(long long* buf) { aether::prefill::g_debug = buf; }
