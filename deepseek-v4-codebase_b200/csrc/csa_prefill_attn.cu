// Chunked-prefill sparse sink attention on the 5th-generation tensor cores
// (sm_100a): tcgen05.mma with operands in shared memory, accumulators in TMEM.
//
// Semantics (aether_2b/modeling.py:616-642, the per-query-row part of the
// CSA forward): every query token t attends, with the per-head sink, to its
// selected compressed blocks (the top-k list of csa_prefill_topk) and to its
// causal window of raw rows; the output is returned before the inverse
// output RoPE.  Compressed entries stay in TurboQuant form: with the rotated
// query q_rot = WHT(diag * q) / sqrt(128),
//   score(block) = scale * (q_rot . c),   O = diag * WHT(sum_b p_b scale_b c_b) / sqrt(128)
// so codes enter the tensor cores as exact fp16 integers and the per-entry
// scale rides on the softmax weight.
//
// One token per pipeline step.  Its 256 candidate code rows and 128 window
// rows are expanded to fp16 tiles in shared memory, in the canonical
// no-swizzle layout: element (row, dim) at
//   (row / 8) * 2048 + (dim / 8) * 128 + (row % 8) * 16 + (dim % 8) * 2.
// K and V are the same rows (one shared compressed K/V per block), and that
// one tile is both operands:
//   S  = K q^T : A = tile read K-major  (M = rows, K = dims), B = q [16 x 128]
//   O^T = V^T P : A = tile read MN-major (M = dims, K = rows), B = P [16 x rows]
// with M = 128, N = 16 (heads padded to 16).  S and O live in TMEM.
//
// Persistent: grid = one CTA per SM, token i of a CTA is row
// blockIdx.x + i * gridDim.x.  Two pipeline slots; warps:
//   0-3, 4-7   gather groups, one per slot: candidate ids, page table, code
//              rows and scales (loaded before the slot frees), window rows,
//              the rotated / plain fp16 queries, the attended-id output
//   8-23       epilogue, four head groups of 4 warps (4 heads each): S from
//              TMEM, masked softmax with the sink (heads reduced across the
//              128 TMEM lanes), P to shared memory; then O from TMEM, inverse
//              WHT across lanes, bf16 output
//   24         TMEM allocation and MMA issue (one thread)
// Every wait is bounded (kWaitLimitNs); a timeout sets the error word and an
// abort flag, and every role leaves its loop at its next check.
#include "aether_b200.h"
#include "capi_util.cuh"
#include <algorithm>
#include <cstddef>

#include "common.cuh"
#include "decode_common.cuh"

namespace aether {
namespace pattn {

constexpr int kThreads = 800;
constexpr int kEpiWarp0 = 8;
constexpr int kHeadGroups = 4;  // epilogue warp groups, 4 heads each
constexpr int kMmaWarp = kEpiWarp0 + 4 * kHeadGroups;
constexpr int kKeys = 256;  // candidate list capacity (top_k <= 256)
constexpr int kWin = 128;
constexpr int kNH = 16;  // padded heads (MMA N)
constexpr uint32_t kGrp = 2048;  // bytes per 8-row group of a [rows][128] fp16 tile
constexpr uint32_t kCM = 128;    // bytes per core matrix
constexpr int kNoPage = -2147483647 - 1;  // candidate slot not attended

// smem map (bytes).  The window tiles come first and the code tiles last so
// that every operand window lies inside the allocation.
constexpr int OFF_TW = 0;                           // [2][128 rows] fp16, 32 KB each
constexpr int OFF_TC = OFF_TW + 2 * kWin * 256;     // [2][256 rows] fp16, 64 KB each
constexpr int OFF_Q = OFF_TC + 2 * kKeys * 256;     // [2][Qr 4 KB | Qw 4 KB]
constexpr int OFF_PC = OFF_Q + 2 * 8192;            // P of the codes [16][256] fp16 (8 KB)
constexpr int OFF_PW = OFF_PC + 8192;               // P of the window [16][128] fp16 (4 KB)
constexpr int OFF_SCL = OFF_PW + 4096;              // [2][256] fp32 entry scale, -1 = not attended
constexpr int OFF_MISC = OFF_SCL + 2 * kKeys * 4;
constexpr int OFF_XB = OFF_MISC + 1024;            // [4 head groups][2][128] fp32 WHT exchange
constexpr int SMEM = OFF_XB + kHeadGroups * 1024;
static_assert(SMEM <= 232448, "shared memory");

struct alignas(16) Misc {
  uint64_t tile_full[2], tile_empty[2], s_full[2], o_full[2], o_empty[2], p_full, p_empty, fin;
  uint32_t tmem;
  int abort_flag;
  int wl[2];
  alignas(16) float redm[kHeadGroups][4][4];  // [head group][warp quarter][head] (float4 stores)
  alignas(16) float reds[kHeadGroups][4][4];
  float sink[kNH];
  uint32_t cnt[2][2][2][4];  // [group][token parity][list half][warp]: valid entries (attended-id compaction)
};
static_assert(sizeof(Misc) <= 1024, "misc");
static_assert(offsetof(Misc, redm) % 16 == 0 && offsetof(Misc, reds) % 16 == 0, "float4 rows");

struct Params {
  const __nv_bfloat16* q;       // [B][H][128]
  const float* sink;            // [H]
  const __nv_bfloat16* window;  // flat raw rows [*][128]
  const long long* win_row;     // [B] first window row
  const int32_t* window_len;    // [B]
  const uint8_t* kv_pages;
  const int32_t* page_table;
  const int32_t* q_row;         // [B] page-table row
  const int32_t* nblocks;       // [B] visible blocks
  const float* diag;            // [128] Rademacher diagonal
  const uint32_t* cand_keys;    // [B][cand_stride], 0 = empty slot
  const int32_t* cand_ids;
  __nv_bfloat16* out;           // [B][H][128]
  int32_t* sel_out;             // [B][top_k] attended ids, -1 padded (optional)
  int* err;
  long long* dbg;  // per-CTA wait / phase cycles [grid][16] (profiling aid), or null
  int table_stride, num_pages, cand_stride, B, H, top_k;
  float softmax_scale;
};

__device__ __forceinline__ uint32_t toff(int r, int d) {
  return (r >> 3) * kGrp + (d >> 3) * kCM + (r & 7) * 16 + (d & 7) * 2;
}
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // sm100 descriptor version; no swizzle
  return d;
}
// kind::f16 instruction descriptor: D f32, A and B f16, B K-major, M = 128,
// N = 16; A K-major or MN-major
constexpr uint32_t kIdescK = (1u << 4) | ((kNH >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescMN = kIdescK | (1u << 15);

__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.u32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(static_cast<uint32_t>(acc)));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t ta, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(ta));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// OR of `pred` over the `n` threads of named barrier `id` (also a barrier)
__device__ __forceinline__ bool named_any(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.or.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Bounded wait on an mbarrier phase; false (and the abort flag set) on a
// timeout or when another role has aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Misc* m, int* err) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int it = 0; it < 16; ++it)
      if (mbar_try_wait(addr, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&m->abort_flag)) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  report_error(err, kErrWaitTimeout);
  *reinterpret_cast<volatile int*>(&m->abort_flag) = 1;
  return false;
}
__device__ __forceinline__ bool aborted(Misc* m) { return *reinterpret_cast<volatile int*>(&m->abort_flag) != 0; }

// nibble pair of one byte -> half2(lo, hi), exact signed values in [-8, 7]
__device__ __forceinline__ uint32_t nib2h2(uint32_t byte) {
  uint32_t y = (byte & 0xFu) | ((byte & 0xF0u) << 12);
  y = (y ^ 0x00080008u) | 0x64006400u;  // 1024 + (v + 8)
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return *reinterpret_cast<uint32_t*>(&h);
}
// two int8 codes (low 16 bits of w) -> half2
__device__ __forceinline__ uint32_t s8x2h2(uint32_t w) {
  uint32_t y = __byte_perm(w ^ 0x8080u, 0x64646464u, 0x5140);  // 1024 + (v + 128)
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t bf2h2(uint32_t v) {
  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  const __half2 h = __floats2half2_rn(f.x, f.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <int BITS>
__global__ void __launch_bounds__(kThreads, 1) csa_prefill_attend_kernel(Params p) {
  constexpr int RB = kHeadDim * BITS / 8;  // code bytes per entry
  constexpr int PB = page_bytes(RB);
  constexpr int NV = RB / 16;              // 16-byte loads per code row
  constexpr int NK = BITS == 4 ? 2 : 1;    // code rows a thread holds at once
  extern __shared__ __align__(1024) uint8_t smem[];
  Misc* m = reinterpret_cast<Misc*>(smem + OFF_MISC);
  float* scl = reinterpret_cast<float*>(smem + OFF_SCL);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntok = p.B > static_cast<int>(blockIdx.x)
                       ? (p.B - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / gridDim.x
                       : 0;
  const int nact = min(kHeadGroups, (p.H + 3) / 4);  // epilogue head groups with real heads

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&m->tile_full[s], 128);
      mbar_init(&m->tile_empty[s], 1);
      mbar_init(&m->s_full[s], 1);
      mbar_init(&m->o_full[s], 1);
      mbar_init(&m->o_empty[s], nact * 128);
    }
    mbar_init(&m->p_full, nact * 128);
    mbar_init(&m->p_empty, 1);
    mbar_init(&m->fin, 1);
    m->abort_flag = 0;
    fence_mbar_init();
  }
  if (tid < kNH) m->sink[tid] = tid < p.H ? p.sink[tid] : 0.f;
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&m->tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = m->tmem;
  long long* dbg = p.dbg ? p.dbg + blockIdx.x * 16 : nullptr;
  long long wait_cycles = 0, wait2 = 0, wait3 = 0;
  const long long t_start = dbg ? clock64() : 0;

  if (warp < kEpiWarp0) {
    // ------------------------------------------------ gather groups
    const int g = warp >> 2, gw = warp & 3, lt = tid & 127;
    const int s = g;
    uint8_t* Tc = smem + OFF_TC + s * kKeys * 256;
    uint8_t* Tw = smem + OFF_TW + s * kWin * 256;
    uint8_t* Qr = smem + OFF_Q + s * 8192;
    uint8_t* Qw = Qr + 4096;
    float* sc = scl + s * kKeys;
    // The group's next token is resolved one token ahead: its candidate
    // entries lt and lt + 128 are loaded while the current token is being
    // expanded, and its metadata and page-table entries right after the
    // current token is handed over.  A token then starts with its code rows.
    struct Next {
      uint32_t key[2];
      int gid[2];
      int phys[2];
      int qr, nbv, wl;
      long long wr;
    } nx;
    auto fetch_list = [&](int tok) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int j = lt + 128 * h2;
        nx.key[h2] = j < p.top_k ? __ldg(p.cand_keys + static_cast<long long>(tok) * p.cand_stride + j) : 0u;
        nx.gid[h2] = j < p.top_k ? __ldg(p.cand_ids + static_cast<long long>(tok) * p.cand_stride + j) : -1;
      }
    };
    auto fetch_pages = [&](int tok) {
      nx.qr = __ldg(p.q_row + tok);
      nx.nbv = __ldg(p.nblocks + tok);
      nx.wl = max(0, min(__ldg(p.window_len + tok), kWin));
      nx.wr = __ldg(p.win_row + tok);
      const int32_t* ptab = p.page_table + static_cast<long long>(nx.qr) * p.table_stride;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int gd = nx.gid[h2];
        const bool att = nx.key[h2] != 0u && gd >= 0 && gd < nx.nbv && (gd >> 6) < p.table_stride;
        nx.phys[h2] = att ? __ldg(ptab + (gd >> 6)) : kNoPage;
      }
    };
    if (g < ntok) {
      fetch_list(blockIdx.x + g * gridDim.x);
      fetch_pages(blockIdx.x + g * gridDim.x);
    }
    for (int i = g; i < ntok; i += 2) {
      const int u = i >> 1;
      const int tok = blockIdx.x + i * gridDim.x;
      const uint32_t key[2] = {nx.key[0], nx.key[1]};
      const int gid[2] = {nx.gid[0], nx.gid[1]};
      const int wl = nx.wl;
      const long long wr = nx.wr;
      // code row and scale of each attended candidate
      bool valid[2], att[2];
      const uint8_t* rowp[2] = {nullptr, nullptr};
      float cs[2] = {-1.f, -1.f};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        valid[h2] = key[h2] != 0u;
        const int phys = nx.phys[h2];
        att[h2] = phys >= 0 && phys < p.num_pages;
        if (phys != kNoPage && !att[h2]) report_error(p.err, kErrBadPage);
        if (att[h2]) {
          const uint8_t* pg = p.kv_pages + static_cast<long long>(phys) * PB;
          rowp[h2] = pg + (gid[h2] & 63) * RB;
          cs[h2] = __ldg(reinterpret_cast<const float*>(pg + kPage * RB) + (gid[h2] & 63));
        }
      }
      if (i + 2 < ntok) fetch_list(tok + 2 * gridDim.x);
      uint4 code[NK][NV];
#pragma unroll
      for (int h2 = 0; h2 < NK; ++h2)
#pragma unroll
        for (int v = 0; v < NV; ++v)
          code[h2][v] = att[h2] ? __ldg(reinterpret_cast<const uint4*>(rowp[h2]) + v) : make_uint4(0, 0, 0, 0);
      if (NK == 1 && att[1])  // 8-bit: the second row is read after the first is expanded
        asm volatile("prefetch.global.L2 [%0];" ::"l"(rowp[1]));
      // the query rows of this warp's heads gw, gw + 4, gw + 8, gw + 12
      uint2 qraw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int h = gw + 4 * k;
        qraw[k] = h < p.H ? __ldg(reinterpret_cast<const uint2*>(p.q + (static_cast<long long>(tok) * p.H + h) *
                                                                        kHeadDim) + lane)
                          : make_uint2(0, 0);
      }
      long long t0 = dbg ? clock64() : 0;
      if (u > 0) {
        const bool ok = wait_bar(&m->tile_empty[s], (u - 1) & 1, m, p.err);
        if (named_any(1 + g, 128, !ok || aborted(m))) break;
      }
      if (dbg) wait_cycles += clock64() - t0;
      // window row lt streams into the tile as raw bf16 while the codes and
      // queries are expanded; it is converted in place afterwards
      {
        const __nv_bfloat16* src = p.window + (wr + lt) * kHeadDim;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          if (lt < wl)
            cp_async16(Tw + toff(lt, 8 * c), src + 8 * c);
          else
            *reinterpret_cast<uint4*>(Tw + toff(lt, 8 * c)) = make_uint4(0, 0, 0, 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      }
      // code rows -> exact fp16 rows of the tile (zeros where not attended)
      auto expand = [&](int j, const uint4 (&cr)[NV]) {
        if (BITS == 4) {
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const uint32_t w4[4] = {cr[v].x, cr[v].y, cr[v].z, cr[v].w};
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)  // 8 dims per 32-bit word
              *reinterpret_cast<uint4*>(Tc + toff(j, 32 * v + 8 * q4)) =
                  make_uint4(nib2h2(w4[q4] & 0xFFu), nib2h2((w4[q4] >> 8) & 0xFFu), nib2h2((w4[q4] >> 16) & 0xFFu),
                             nib2h2(w4[q4] >> 24));
          }
        } else {
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const uint4 w = cr[v];
            *reinterpret_cast<uint4*>(Tc + toff(j, 16 * v)) =
                make_uint4(s8x2h2(w.x & 0xFFFFu), s8x2h2(w.x >> 16), s8x2h2(w.y & 0xFFFFu), s8x2h2(w.y >> 16));
            *reinterpret_cast<uint4*>(Tc + toff(j, 16 * v + 8)) =
                make_uint4(s8x2h2(w.z & 0xFFFFu), s8x2h2(w.z >> 16), s8x2h2(w.w & 0xFFFFu), s8x2h2(w.w >> 16));
          }
        }
      };
      sc[lt] = att[0] ? cs[0] : -1.f;
      sc[lt + 128] = att[1] ? cs[1] : -1.f;
      expand(lt, code[0]);
      if (NK == 2) {
        expand(lt + 128, code[NK - 1]);
      } else {
#pragma unroll
        for (int v = 0; v < NV; ++v)
          code[0][v] = att[1] ? __ldg(reinterpret_cast<const uint4*>(rowp[1]) + v) : make_uint4(0, 0, 0, 0);
        expand(lt + 128, code[0]);
      }
      // queries: plain fp16 rows for the window, rotated fp16 rows for the codes
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int h = gw + 4 * k;
        const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qraw[k].x));
        const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qraw[k].y));
        float v[4] = {f0.x * p.diag[lane * 4], f0.y * p.diag[lane * 4 + 1], f1.x * p.diag[lane * 4 + 2],
                      f1.y * p.diag[lane * 4 + 3]};
        *reinterpret_cast<uint2*>(Qw + toff(h, lane * 4)) = make_uint2(bf2h2(qraw[k].x), bf2h2(qraw[k].y));
        warp_wht128(v, lane);
        const float cn = 0.0883883461356163f;
        *reinterpret_cast<uint2*>(Qr + toff(h, lane * 4)) =
            make_uint2(pack_half2(v[0] * cn, v[1] * cn), pack_half2(v[2] * cn, v[3] * cn));
      }
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      if (lt < wl) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4* t = reinterpret_cast<uint4*>(Tw + toff(lt, 8 * c));
          const uint4 x = *t;
          *t = make_uint4(bf2h2(x.x), bf2h2(x.y), bf2h2(x.z), bf2h2(x.w));
        }
      }
      if (lt == 0) m->wl[s] = wl;
      // attended ids in list order (the valid entries, compacted)
      if (p.sel_out) {
        uint32_t* cnt = &m->cnt[g][u & 1][0][0];
        const uint32_t b0 = __ballot_sync(0xffffffffu, valid[0]), b1 = __ballot_sync(0xffffffffu, valid[1]);
        if (lane == 0) {
          cnt[gw] = __popc(b0);
          cnt[4 + gw] = __popc(b1);
        }
        named_sync(1 + g, 128);
        uint32_t base0 = 0, base1 = 0, tot0 = 0, tot1 = 0;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          if (w < gw) {
            base0 += cnt[w];
            base1 += cnt[4 + w];
          }
          tot0 += cnt[w];
          tot1 += cnt[4 + w];
        }
        const uint32_t lm = (1u << lane) - 1u;
        int32_t* so = p.sel_out + static_cast<long long>(tok) * p.top_k;
        if (valid[0]) so[base0 + __popc(b0 & lm)] = gid[0];
        if (valid[1]) so[tot0 + base1 + __popc(b1 & lm)] = gid[1];
        for (int j = static_cast<int>(tot0 + tot1) + lt; j < p.top_k; j += 128) so[j] = -1;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      arrive(&m->tile_full[s]);
      if (i + 2 < ntok) fetch_pages(tok + 2 * gridDim.x);
    }
    if (dbg && lt == 0) dbg[g] = wait_cycles;
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------ epilogue
    // head group hg (4 warps) owns heads 4 hg .. 4 hg + 3; warp quarter e
    // reads TMEM lanes 32 e .. 32 e + 31 (rows of S, dims of O).  Iteration i
    // runs the softmax of token i, then the output of token i - 1, whose
    // P V ran meanwhile.
    const int hg = (warp - kEpiWarp0) >> 2, e = warp & 3, r = e * 32 + lane;
    const int bar = 3 + hg, h0 = 4 * hg;
    const uint32_t lanebase = static_cast<uint32_t>(e * 32) << 16;
    const float ss = p.softmax_scale;
    uint8_t* Pc = smem + OFF_PC;
    uint8_t* Pw = smem + OFF_PW;
    float* xb = reinterpret_cast<float*>(smem + OFF_XB) + hg * 256;  // [2 heads][128] exchange
    float inv_out[4] = {0.f, 0.f, 0.f, 0.f};  // 1 / denominator of the token awaiting output
    long long ph[7] = {0, 0, 0, 0, 0, 0, 0};   // phase cycles (profiling aid)
    for (int i = 0; hg < nact && i <= ntok; ++i) {
      float inv_new[4] = {0.f, 0.f, 0.f, 0.f};
      if (i < ntok) {
        // ---- softmax of token i: per-warp (max, sum) pairs, one exchange
        const int s = i & 1, u = i >> 1;
        long long t0 = dbg ? clock64() : 0;
        bool ok = wait_bar(&m->tile_full[s], u & 1, m, p.err);
        ok = ok && wait_bar(&m->s_full[s], u & 1, m, p.err);
        if (dbg) wait_cycles += clock64() - t0;
        float x0[4] = {0.f, 0.f, 0.f, 0.f}, x1[4] = {0.f, 0.f, 0.f, 0.f}, xw[4] = {0.f, 0.f, 0.f, 0.f};
        long long c0 = dbg ? clock64() : 0;
        if (ok) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t tS = tmem + lanebase + s * 128 + h0;
          tmem_ld4(tS, x0);
          tmem_ld4(tS + 16, x1);
          tmem_ld4(tS + 32, xw);
          tmem_wait_ld();
        }
        long long c1 = dbg ? clock64() : 0;
        if (dbg) ph[0] += c1 - c0;
        const float sc0 = scl[s * kKeys + r], sc1 = scl[s * kKeys + 128 + r];
        const bool wv = r < m->wl[s];
        float ml[4], ll[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          x0[k] = sc0 >= 0.f ? x0[k] * sc0 * ss : -INFINITY;
          x1[k] = sc1 >= 0.f ? x1[k] * sc1 * ss : -INFINITY;
          xw[k] = wv ? xw[k] * ss : -INFINITY;
          ml[k] = warp_max(fmaxf(fmaxf(x0[k], x1[k]), xw[k]));
          const float base = ml[k] == -INFINITY ? 0.f : ml[k];
          x0[k] = __expf(x0[k] - base);
          x1[k] = __expf(x1[k] - base);
          xw[k] = __expf(xw[k] - base);
          ll[k] = warp_sum(x0[k] + x1[k] + xw[k]);
        }
        if (lane == 0) {
          *reinterpret_cast<float4*>(m->redm[hg][e]) = make_float4(ml[0], ml[1], ml[2], ml[3]);
          *reinterpret_cast<float4*>(m->reds[hg][e]) = make_float4(ll[0], ll[1], ll[2], ll[3]);
        }
        // P may be written once the previous token's P V has read it
        t0 = dbg ? clock64() : 0;
        if (dbg) ph[1] += t0 - c1;
        const bool ok2 = i == 0 || wait_bar(&m->p_empty, (i - 1) & 1, m, p.err);
        if (dbg) wait2 += clock64() - t0;
        c0 = dbg ? clock64() : 0;
        if (named_any(bar, 128, !ok || !ok2 || aborted(m))) break;
        c1 = dbg ? clock64() : 0;
        if (dbg) ph[2] += c1 - c0;
        float corr[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float M = m->sink[h0 + k];
#pragma unroll
          for (int w = 0; w < 4; ++w) M = fmaxf(M, m->redm[hg][w][k]);
          float L = __expf(m->sink[h0 + k] - M);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float mw = m->redm[hg][w][k];
            L += mw == -INFINITY ? 0.f : m->reds[hg][w][k] * __expf(mw - M);
          }
          corr[k] = ml[k] == -INFINITY ? 0.f : __expf(ml[k] - M);
          inv_new[k] = 1.f / L;
        }
        // P: codes carry their entry scale; key pairs (r, r + 1) per store
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int h = h0 + k;
          const float a0 = x0[k] * corr[k] * fmaxf(sc0, 0.f), a1 = x1[k] * corr[k] * fmaxf(sc1, 0.f),
                      aw = xw[k] * corr[k];
          const float b0 = __shfl_xor_sync(0xffffffffu, a0, 1), b1 = __shfl_xor_sync(0xffffffffu, a1, 1),
                      bw = __shfl_xor_sync(0xffffffffu, aw, 1);
          if ((lane & 1) == 0) {
            const uint32_t hb = (h >> 3) * 4096 + (h & 7) * 16;
            *reinterpret_cast<uint32_t*>(Pc + hb + (r >> 3) * kCM + (r & 7) * 2) = pack_half2(a0, b0);
            *reinterpret_cast<uint32_t*>(Pc + hb + ((r + 128) >> 3) * kCM + (r & 7) * 2) = pack_half2(a1, b1);
            *reinterpret_cast<uint32_t*>(Pw + (h >> 3) * 2048 + (h & 7) * 16 + (r >> 3) * kCM + (r & 7) * 2) =
                pack_half2(aw, bw);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        arrive(&m->p_full);
        if (dbg) ph[3] += clock64() - c1;
      }
      if (i > 0) {
        // ---- output of token i - 1: thread r owns dim r of the group's heads
        const int j = i - 1, s = j & 1, u = j >> 1;
        const int tok = blockIdx.x + j * gridDim.x;
        long long t0 = dbg ? clock64() : 0;
        const bool ok = wait_bar(&m->o_full[s], u & 1, m, p.err);
        if (dbg) wait3 += clock64() - t0;
        float oc[4] = {0.f, 0.f, 0.f, 0.f}, ow[4] = {0.f, 0.f, 0.f, 0.f};
        long long c0 = dbg ? clock64() : 0;
        if (ok) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          tmem_ld4(tmem + lanebase + s * 128 + 64 + h0, oc);
          tmem_ld4(tmem + lanebase + s * 128 + 80 + h0, ow);
          tmem_wait_ld();
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          arrive(&m->o_empty[s]);
        }
        long long c1 = dbg ? clock64() : 0;
        if (dbg) ph[4] += c1 - c0;
        // inverse WHT over the 128 dims: bits 5 and 6 through the group's
        // exchange buffer (two heads at a time), bits 0-4 by shuffles
        const int b5 = r & 31, idx = r >> 5;
        bool stop = false;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (half) named_sync(bar, 128);  // the first pair's reads are done
          xb[r] = oc[2 * half];
          xb[128 + r] = oc[2 * half + 1];
          if (half == 0) {
            stop = named_any(bar, 128, !ok || aborted(m));
          } else {
            named_sync(bar, 128);
          }
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const float* xr = xb + kk * 128 + b5;
            const float a = xr[0], b = xr[32], c = xr[64], d = xr[96];
            const float s0 = (idx & 1) ? a - b : a + b, s1 = (idx & 1) ? c - d : c + d;
            oc[2 * half + kk] = (idx & 2) ? s0 - s1 : s0 + s1;
          }
        }
        if (stop) break;
        c0 = dbg ? clock64() : 0;
        if (dbg) ph[5] += c0 - c1;
#pragma unroll
        for (int ld = 1; ld < 32; ld <<= 1) {
          const bool up = (lane & ld) != 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float o = __shfl_xor_sync(0xffffffffu, oc[k], ld);
            oc[k] = up ? o - oc[k] : oc[k] + o;
          }
        }
        const float dg = p.diag[r] * 0.0883883461356163f;
        __nv_bfloat16* orow = p.out + static_cast<long long>(tok) * p.H * kHeadDim;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float v = (oc[k] * dg + ow[k]) * inv_out[k];
          const float w = __shfl_xor_sync(0xffffffffu, v, 1);
          if (h0 + k < p.H && (lane & 1) == 0)
            *reinterpret_cast<__nv_bfloat162*>(orow + (h0 + k) * kHeadDim + r) = __floats2bfloat162_rn(v, w);
        }
        if (dbg) ph[6] += clock64() - c0;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) inv_out[k] = inv_new[k];
    }
    if (dbg && hg == 0 && r == 0) {
      dbg[2] = wait_cycles;
      dbg[3] = wait2;
      dbg[4] = wait3;
      for (int k = 0; k < 7; ++k) dbg[8 + k] = ph[k];
    }
  } else {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      for (int i = 0; i < ntok; ++i) {
        const int s = i & 1, u = i >> 1;
        long long t0 = dbg ? clock64() : 0;
        if (!wait_bar(&m->tile_full[s], u & 1, m, p.err)) break;
        if (dbg) wait_cycles += clock64() - t0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sTc = smem_u32(smem + OFF_TC + s * kKeys * 256);
        const uint32_t sTw = smem_u32(smem + OFF_TW + s * kWin * 256);
        const uint32_t sQr = smem_u32(smem + OFF_Q + s * 8192), sQw = sQr + 4096;
        const uint32_t dS = tmem + s * 128;
        // S = K q^T: rows 0-127 and 128-255 of the codes, then the window
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t b = sdesc(sQr + ks * 256, kCM, kGrp);
          mma(dS, sdesc(sTc + ks * 256, kCM, kGrp), b, kIdescK, ks > 0);
          mma(dS + 16, sdesc(sTc + 16 * kGrp + ks * 256, kCM, kGrp), b, kIdescK, ks > 0);
          mma(dS + 32, sdesc(sTw + ks * 256, kCM, kGrp), sdesc(sQw + ks * 256, kCM, kGrp), kIdescK, ks > 0);
        }
        commit(&m->s_full[s]);
        t0 = dbg ? clock64() : 0;
        if (!wait_bar(&m->p_full, i & 1, m, p.err)) break;
        if (dbg) wait2 += clock64() - t0;
        if (u > 0 && !wait_bar(&m->o_empty[s], (u - 1) & 1, m, p.err)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // O^T = V^T P: the tiles read MN-major (K = rows in steps of 16)
        const uint32_t sPc = smem_u32(smem + OFF_PC), sPw = smem_u32(smem + OFF_PW);
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks)
          mma(dS + 64, sdesc(sTc + ks * 2 * kGrp, kGrp, kCM), sdesc(sPc + ks * 2 * kCM, kCM, 4096), kIdescMN,
              ks > 0);
#pragma unroll
        for (int ks = 0; ks < kWin / 16; ++ks)
          mma(dS + 80, sdesc(sTw + ks * 2 * kGrp, kGrp, kCM), sdesc(sPw + ks * 2 * kCM, kCM, 2048), kIdescMN,
              ks > 0);
        commit(&m->o_full[s]);
        commit(&m->tile_empty[s]);
        commit(&m->p_empty);
      }
      if (dbg) {
        dbg[5] = wait_cycles;
        dbg[6] = wait2;
      }
      // every MMA issued has completed before TMEM is released
      commit(&m->fin);
      const uint32_t fa = smem_u32(&m->fin);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(fa, 0) && global_ns() - t0 < kWaitLimitNs) {
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (dbg && tid == 0) dbg[7] = clock64() - t_start;
  if (warp == kMmaWarp) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

static long long* g_debug = nullptr;

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

template <int BITS>
static int launch(const Params& p, cudaStream_t st) {
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(csa_prefill_attend_kernel<BITS>), SMEM,
                                "csa_prefill_attend"))
    return rc;
  const int grid = std::min(p.B, sm_count());
  csa_prefill_attend_kernel<BITS><<<grid, kThreads, SMEM, st>>>(p);
  return check_launch("csa_prefill_attend");
}

}  // namespace pattn
}  // namespace aether

using namespace aether;

extern "C" int aether_csa_prefill_attend(const void* q, const float* sink, const void* window,
                                         const long long* win_row, const int32_t* window_len, const uint8_t* kv_pages,
                                         const int32_t* page_table, int table_stride, int num_pages,
                                         const int32_t* q_row, const int32_t* nblocks, int max_nblocks,
                                         const float* diag_kv, const uint32_t* cand_keys, const int32_t* cand_ids,
                                         int cand_stride, int B, int H, int bits, int top_k, float softmax_scale,
                                         void* out, int32_t* sel_out, int* err, void* stream) {
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(H >= 1 && H <= kMaxHeads, "num_heads must be in [1, %d], got %d", kMaxHeads, H);
  AETHER_REQUIRE(top_k >= 1 && top_k <= pattn::kKeys, "top_k must be in [1, %d], got %d", pattn::kKeys, top_k);
  AETHER_REQUIRE(table_stride >= 1 && num_pages >= 1, "page table / pool must be non-empty");
  AETHER_REQUIRE(max_nblocks >= 0, "negative block count");
  AETHER_REQUIRE(B >= 0, "negative batch");
  AETHER_REQUIRE(q && sink && window && win_row && window_len && kv_pages && page_table && q_row && nblocks &&
                     diag_kv && cand_keys && cand_ids && out,
                 "csa_prefill_attend: null argument");
  AETHER_REQUIRE(cand_stride >= top_k && (cand_stride & 3) == 0,
                 "csa_prefill_attend: cand_stride must be >= top_k and a multiple of 4");
  if (B == 0) return 0;
  pattn::Params p{static_cast<const __nv_bfloat16*>(q), sink, static_cast<const __nv_bfloat16*>(window), win_row,
                  window_len, kv_pages, page_table, q_row, nblocks, diag_kv, cand_keys, cand_ids,
                  static_cast<__nv_bfloat16*>(out), sel_out, err, pattn::g_debug, table_stride, num_pages, cand_stride,
                  B, H, top_k, softmax_scale};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return bits == 4 ? pattn::launch<4>(p, st) : pattn::launch<8>(p, st);
}

// Profiling aid: when buf is non-null, later prefill-attention launches
// record per CTA (8 entries each) the SM-clock cycles spent waiting: the two
// gather groups (slot free), the epilogue (scores ready, P free, O ready),
// the MMA issuer (tiles ready, P ready), and the CTA's total.
extern "C" void aether_csa_prefill_attend_set_debug(long long* buf) { aether::pattn::g_debug = buf; }
