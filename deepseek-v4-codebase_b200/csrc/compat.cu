// Drop-in replacements for the reference extension's four ops
// (aether_kernels/csrc/bindings.cpp:124-141 of the reference):
//
//   sparse_sink_attention   bindings.cpp:21-46, sparse_sink_attention_cuda.cu:118-177
//   tiled_prefill_attention bindings.cpp:58-77, tiled_prefill_cuda.cu
//   csa_indexer_topk        bindings.cpp:88-101, csa_indexer_cuda.cu
//   hca_compress            bindings.cpp:110-119, hca_compress_cuda.cu
//
// Semantics follow the reference's PyTorch math, which is what its tests hold
// the kernels to (aether_pipeline/serving.py:99-130 for attention,
// aether_2b/modeling.py:609-615 for the indexer, aether_2b/serving.py:495-498
// for HCA compression).  Two deliberate differences from the reference CUDA
// kernels: the prefill sink enters the softmax denominator once (the
// reference adds it once per source token), and the indexer uses the
// canonical softplus/ReLU score with an exact, (score desc, index asc)
// ordered top-k instead of a raw weighted dot with an unordered serial pick.
#include <type_traits>

#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"
#include "decode_common.cuh"

namespace aether {

enum DTypeCode : int { kCF32 = 0, kCF16 = 1, kCBF16 = 2 };

template <typename T>
__device__ __forceinline__ float tofl(T v);
template <>
__device__ __forceinline__ float tofl<float>(float v) { return v; }
template <>
__device__ __forceinline__ float tofl<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float tofl<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T fromfl(float v);
template <>
__device__ __forceinline__ float fromfl<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half fromfl<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 fromfl<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ---------------------------------------------------------------------------
// Sparse sink attention: one warp per (b, t, h), online softmax over the K
// gathered sources, fp32 accumulation.  Index < 0 or >= S is skipped.
// idx == nullptr means "all S sources in order" (tiled prefill).
template <typename T, typename I, int DPL>
__global__ void __launch_bounds__(256) sink_attn_kernel(const T* __restrict__ q, const T* __restrict__ kv,
                                                        const I* __restrict__ idx, const T* __restrict__ sink,
                                                        T* __restrict__ out, int B, int Tt, int H, int D, int S,
                                                        int K, float scale, int sink_scalar) {
  const int lane = threadIdx.x & 31;
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (w >= static_cast<long long>(B) * Tt * H) return;
  const int h = static_cast<int>(w % H);
  const long long bt = w / H;
  const int b = static_cast<int>(bt / Tt);
  float qv[DPL], acc[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) {
    const int d = lane + 32 * k;
    qv[k] = d < D ? tofl<T>(q[w * D + d]) : 0.f;
    acc[k] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const I* ip = idx ? idx + bt * K : nullptr;
  const T* kvb = kv + static_cast<long long>(b) * S * 2 * D;
  for (int j = 0; j < K; ++j) {
    const long long src = ip ? static_cast<long long>(ip[j]) : j;
    if (src < 0 || src >= S) continue;
    const T* kp = kvb + src * 2 * D;
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) dot += qv[k] * tofl<T>(kp[d]);
    }
    dot = warp_sum(dot) * scale;
    const float mn = fmaxf(m, dot);
    const float corr = __expf(m - mn);  // m = -inf on the first source -> 0
    const float e = __expf(dot - mn);
    l = l * corr + e;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      acc[k] = acc[k] * corr + (d < D ? e * tofl<T>(kp[D + d]) : 0.f);
    }
    m = mn;
  }
  const float sk = tofl<T>(sink[sink_scalar ? 0 : h]);
  const float M = fmaxf(m, sk);
  const float a = m == -INFINITY ? 0.f : __expf(m - M);
  const float den = l * a + __expf(sk - M);
#pragma unroll
  for (int k = 0; k < DPL; ++k) {
    const int d = lane + 32 * k;
    if (d < D) out[w * D + d] = fromfl<T>(acc[k] * a / den);
  }
}


// ---------------------------------------------------------------------------
// Tensor-core path for the common shape (16-bit inputs, D = 128, H <= 16):
// one CTA per target token serves all heads.  Gathered K / V rows arrive in
// 128-row tiles (cp.async, double-buffered); S = Q K^T on mma.sync (16 heads x
// 16 sources per warp), an online softmax per head across tiles, O += P V on
// mma.sync (16 output dims per warp, fp16 P, V converted to fp16 in
// registers for bf16 inputs); the sink enters the denominator once at the end.
constexpr int kTcRows = 128;  // sources per tile
constexpr int kTcRow = 136;   // padded smem row (elements)
constexpr int kTcSt = kTcRows + 4;  // logit row stride (floats)
constexpr int kTcPst = kTcRows + 8;  // P row stride (halves)
constexpr int kTcSmem = (16 * kTcRow + 4 * kTcRows * kTcRow) * 2 + 16 * kTcSt * 4 + 16 * kTcPst * 2 + 2 * kTcRows * 4 +
                        3 * 16 * 4;

template <typename T>
__device__ __forceinline__ void tc_mma_qk(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) mma_bf16(c, a, b0, b1);
  else mma_f16(c, a, b0, b1);
}

template <typename T, typename I>
__global__ void __launch_bounds__(256) sink_attn_tc_kernel(const T* __restrict__ q, const T* __restrict__ kv,
                                                           const I* __restrict__ idx, const T* __restrict__ sink,
                                                           T* __restrict__ out, int Tt, int H, int S, int K,
                                                           float scale, int sink_scalar) {
  constexpr int D = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  T* Qs = reinterpret_cast<T*>(smem);
  T* Ks = Qs + 16 * kTcRow;                 // [2][128][kTcRow]
  T* Vs = Ks + 2 * kTcRows * kTcRow;        // [2][128][kTcRow]
  float* Ls = reinterpret_cast<float*>(Vs + 2 * kTcRows * kTcRow);  // [16][kTcSt]
  __half* Ps = reinterpret_cast<__half*>(Ls + 16 * kTcSt);          // [16][kTcPst]
  int* valid = reinterpret_cast<int*>(Ps + 16 * kTcPst);            // [2][128]
  float* mh = reinterpret_cast<float*>(valid + 2 * kTcRows);        // [16] running max
  float* lh = mh + 16;                                              // [16] running sum
  float* sch = lh + 16;                                             // [16] this tile's rescale
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const long long bt = blockIdx.x;
  const int b = static_cast<int>(bt / Tt);
  const I* ip = idx ? idx + bt * K : nullptr;
  const T* kvb = kv + static_cast<long long>(b) * S * 2 * D;
  // queries: heads past H are zero rows
  for (int i = tid; i < 16 * 16; i += 256) {
    const int h = i >> 4, c = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < H) v = *reinterpret_cast<const uint4*>(q + (bt * H + h) * D + c * 8);
    *reinterpret_cast<uint4*>(Qs + h * kTcRow + c * 8) = v;
  }
  if (tid < 16) {
    mh[tid] = -INFINITY;
    lh[tid] = 0.f;
  }
  const int ntiles = (K + kTcRows - 1) / kTcRows;
  auto load_tile = [&](int j, int buf) {
    T* kd = Ks + buf * kTcRows * kTcRow;
    T* vd = Vs + buf * kTcRows * kTcRow;
    for (int i = tid; i < kTcRows * 16; i += 256) {
      const int r = i >> 4, c = i & 15, e = j * kTcRows + r;
      long long src = -1;
      if (e < K) src = ip ? static_cast<long long>(ip[e]) : e;
      const bool ok = src >= 0 && src < S;
      if (c == 0) valid[buf * kTcRows + r] = ok;
      if (ok) {
        cp_async16(kd + r * kTcRow + c * 8, kvb + src * 2 * D + c * 8);
        cp_async16(vd + r * kTcRow + c * 8, kvb + src * 2 * D + D + c * 8);
      } else {
        *reinterpret_cast<uint4*>(kd + r * kTcRow + c * 8) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vd + r * kTcRow + c * 8) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float oacc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  if (ntiles > 0) load_tile(0, 0);
  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      load_tile(j + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    // ---- S: warp w scores sources [16 w, 16 w + 16) for all 16 heads
    {
      const T* kt = Ks + buf * kTcRows * kTcRow + warp * 16 * kTcRow;
      float c[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4], b0, b1, b2, b3;
        ldsm_x4(a[0], a[1], a[2], a[3], Qs + (lane & 15) * kTcRow + kk * 16 + (lane >> 4) * 8);
        ldsm_x4(b0, b1, b2, b3, kt + ((lane & 7) + ((lane >> 4) << 3)) * kTcRow + kk * 16 + ((lane >> 3) & 1) * 8);
        tc_mma_qk<T>(c[0], a, b0, b1);
        tc_mma_qk<T>(c[1], a, b2, b3);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = g + (e >> 1) * 8, col = warp * 16 + nt * 8 + 2 * t + (e & 1);
          Ls[h * kTcSt + col] = valid[buf * kTcRows + col] ? c[nt][e] * scale : -INFINITY;
        }
    }
    __syncthreads();
    // ---- online softmax: warp w owns heads 2w, 2w + 1; 4 sources per lane
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int h = 2 * warp + hh;
      const float4 z = *reinterpret_cast<const float4*>(Ls + h * kTcSt + 4 * lane);
      const float mt = warp_max(fmaxf(fmaxf(z.x, z.y), fmaxf(z.z, z.w)));
      const float mo = mh[h], mn = fmaxf(mo, mt);
      const float base = mn == -INFINITY ? 0.f : mn;
      const float p0 = __expf(z.x - base), p1 = __expf(z.y - base), p2 = __expf(z.z - base), p3 = __expf(z.w - base);
      *reinterpret_cast<uint2*>(Ps + h * kTcPst + 4 * lane) = make_uint2(pack_half2(p0, p1), pack_half2(p2, p3));
      const float ps = warp_sum((p0 + p1) + (p2 + p3));
      const float sc = mo == -INFINITY ? 0.f : __expf(mo - base);
      if (lane == 0) {
        lh[h] = lh[h] * sc + ps;
        mh[h] = mn;
        sch[h] = sc;
      }
    }
    __syncthreads();
    // ---- O = O * rescale + P V: warp w owns output dims [16 w, 16 w + 16)
    {
      const float s_lo = sch[g], s_hi = sch[g + 8];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        oacc[nt][0] *= s_lo; oacc[nt][1] *= s_lo;
        oacc[nt][2] *= s_hi; oacc[nt][3] *= s_hi;
      }
      const T* vt = Vs + buf * kTcRows * kTcRow;
#pragma unroll 4
      for (int kt = 0; kt < kTcRows / 16; ++kt) {
        uint32_t a[4];
        ldsm_x4(a[0], a[1], a[2], a[3], Ps + (lane & 15) * kTcPst + kt * 16 + (lane >> 4) * 8);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          uint32_t b0, b1;
          asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                       : "=r"(b0), "=r"(b1)
                       : "r"(smem_u32(vt + (kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kTcRow + warp * 16 +
                                      nt * 8)));
          if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            b0 = bf2_to_h2(b0);
            b1 = bf2_to_h2(b1);
          }
          mma_f16(oacc[nt], a, b0, b1);
        }
      }
    }
    __syncthreads();  // this tile's buffers are reused by the load two tiles on
  }
  // ---- sink and output: rows g and g + 8 of each n-tile
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int h = g + hr * 8;
    if (h >= H) continue;
    const float sk = tofl<T>(sink[sink_scalar ? 0 : h]);
    const float m = mh[h], M = fmaxf(m, sk);
    const float a = m == -INFINITY ? 0.f : __expf(m - M);
    const float inv = a / (lh[h] * a + __expf(sk - M));
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int d = warp * 16 + nt * 8 + 2 * t;
      T* o = out + (bt * H + h) * D + d;
      o[0] = fromfl<T>(oacc[nt][2 * hr] * inv);
      o[1] = fromfl<T>(oacc[nt][2 * hr + 1] * inv);
    }
  }
}

template <typename T, typename I>
static void launch_sink_attn(const void* q, const void* kv, const void* idx, const void* sink, void* out, int B,
                             int Tt, int H, int D, int S, int K, float scale, int sink_scalar, cudaStream_t st) {
  const long long warps = static_cast<long long>(B) * Tt * H;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  auto args = [&](auto kern) {
    kern<<<blocks, threads, 0, st>>>(static_cast<const T*>(q), static_cast<const T*>(kv),
                                     static_cast<const I*>(idx), static_cast<const T*>(sink),
                                     static_cast<T*>(out), B, Tt, H, D, S, K, scale, sink_scalar);
  };
  if constexpr (!std::is_same<T, float>::value) {
    if (D == 128 && H <= 16) {  // the tensor-core path
      if (ensure_smem_attr(reinterpret_cast<const void*>(sink_attn_tc_kernel<T, I>), kTcSmem,
                           "sparse_sink_attention") == 0) {
        sink_attn_tc_kernel<T, I><<<static_cast<unsigned>(static_cast<long long>(B) * Tt), 256, kTcSmem, st>>>(
            static_cast<const T*>(q), static_cast<const T*>(kv), static_cast<const I*>(idx),
            static_cast<const T*>(sink), static_cast<T*>(out), Tt, H, S, K, scale, sink_scalar);
        return;
      }
    }
  }
  if (D <= 32) args(sink_attn_kernel<T, I, 1>);
  else if (D <= 64) args(sink_attn_kernel<T, I, 2>);
  else if (D <= 128) args(sink_attn_kernel<T, I, 4>);
  else args(sink_attn_kernel<T, I, 8>);
}

static int sink_attn_dispatch(const void* q, const void* kv, const void* idx, int idx_is_64, const void* sink,
                              int sink_numel, void* out, int dtype, int B, int Tt, int H, int D, int S, int K,
                              float scale, cudaStream_t st) {
  AETHER_REQUIRE(D >= 1 && D <= 256, "head_dim must be in [1, 256], got %d", D);
  AETHER_REQUIRE(sink_numel == 1 || sink_numel == H, "sink must be a scalar or a [num_heads] tensor");
  AETHER_REQUIRE(dtype >= 0 && dtype <= 2, "unsupported dtype code %d", dtype);
  if (static_cast<long long>(B) * Tt * H == 0) return 0;
  const int ss = sink_numel == 1;
#define AETHER_SA(T)                                                                                 \
  do {                                                                                               \
    if (idx_is_64) launch_sink_attn<T, int64_t>(q, kv, idx, sink, out, B, Tt, H, D, S, K, scale, ss, st); \
    else launch_sink_attn<T, int32_t>(q, kv, idx, sink, out, B, Tt, H, D, S, K, scale, ss, st);     \
  } while (0)
  if (dtype == kCF32) AETHER_SA(float);
  else if (dtype == kCF16) AETHER_SA(__half);
  else AETHER_SA(__nv_bfloat16);
#undef AETHER_SA
  return check_launch("sparse_sink_attention");
}

// ---------------------------------------------------------------------------
// Dense indexer scores: one warp per (b, s); lanes over the index dim.
// score = sum_h softplus(w_h) * relu(q_h . k_s) in fp32.
__global__ void __launch_bounds__(256) dense_index_score_kernel(const float* __restrict__ iq,
                                                                const float* __restrict__ ikv,
                                                                const float* __restrict__ iw,
                                                                float* __restrict__ scores, int B, int IH, int IC,
                                                                int S) {
  const int lane = threadIdx.x & 31;
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (w >= static_cast<long long>(B) * S) return;
  const int b = static_cast<int>(w / S);
  const float* kp = ikv + w * IC;
  float total = 0.f;
  for (int h = 0; h < IH; ++h) {
    const float* qp = iq + (static_cast<long long>(b) * IH + h) * IC;
    float dot = 0.f;
    for (int c = lane; c < IC; c += 32) dot += qp[c] * kp[c];
    dot = warp_sum(dot);
    total += softplus_f(iw[b * IH + h]) * fmaxf(dot, 0.f);
  }
  if (lane == 0) scores[w] = total + 0.0f;
}

// Order-preserving key of an fp32 score (descending order of floats =
// descending order of keys), -0 folded onto +0.
__device__ __forceinline__ uint32_t score_key(float s) {
  uint32_t u = __float_as_uint(s + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exact top-k of one row per CTA: 4 x 8-bit MSB-first radix passes find the
// k-th largest key; keys above it are taken, ties at it by lowest index; the
// k winners are then sorted by (score desc, index asc) with a bitonic sort.
constexpr int kTopkThreads = 512;
constexpr int kTopkMax = 2048;
__global__ void __launch_bounds__(kTopkThreads) row_topk_kernel(const float* __restrict__ scores, int S, int k,
                                                                int64_t* __restrict__ out) {
  __shared__ uint32_t hist[256];
  __shared__ unsigned long long cand[kTopkMax];
  __shared__ uint32_t sh_bin, sh_above, sh_cnt_eq;
  __shared__ uint32_t wsum[kTopkThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = scores + static_cast<long long>(blockIdx.x) * S;
  uint32_t prefix = 0, R = static_cast<uint32_t>(k);
  int nbits = 0;
  bool all_eq = false;
  for (int pass = 0; pass < 4; ++pass) {
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    const int shift = 24 - 8 * pass;
    for (int base = 0; base < S; base += kTopkThreads) {
      const int i = base + tid;
      bool m = false;
      uint32_t dig = 0xFFFFFFFFu;
      if (i < S) {
        const uint32_t key = score_key(row[i]);
        m = nbits == 0 || (key >> (32 - nbits)) == prefix;
        if (m) dig = (key >> shift) & 255u;
      }
      if (m) atomicAdd(&hist[dig], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t s8 = 0;
      for (int q = 0; q < 8; ++q) s8 += hist[255 - 8 * lane - q];
      uint32_t inc = s8;
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      const uint32_t exc = inc - s8;
      const bool hit = exc < R && inc >= R;
      const uint32_t hm = __ballot_sync(0xffffffffu, hit);
      if (hit && lane == __ffs(hm) - 1) {
        uint32_t cum = exc;
        for (int q = 0; q < 8; ++q) {
          const int bin = 255 - 8 * lane - q;
          if (cum + hist[bin] >= R) {
            sh_bin = bin;
            sh_above = cum;
            sh_cnt_eq = hist[bin];
            break;
          }
          cum += hist[bin];
        }
      }
    }
    __syncthreads();
    R -= sh_above;
    prefix = (prefix << 8) | sh_bin;
    nbits += 8;
    const bool done = sh_cnt_eq == R;
    __syncthreads();
    if (done) {
      all_eq = true;
      break;
    }
  }
  // ordered compaction: strict (> prefix) all taken, equal ones lowest-index first
  const int E = (S + kTopkThreads - 1) / kTopkThreads;
  const int i0 = min(tid * E, S), i1 = min(i0 + E, S);
  uint32_t cs = 0, ce = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t top = score_key(row[i]) >> (32 - nbits);
    if (top > prefix) ++cs;
    else if (top == prefix) ++ce;
  }
  const uint32_t packed = cs | (ce << 16);
  uint32_t inc = packed;
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  uint32_t wb = 0;
  for (int w = 0; w < warp; ++w) wb += wsum[w];
  uint32_t tot = 0;
  for (int w = 0; w < kTopkThreads / 32; ++w) tot += wsum[w];
  const uint32_t take = all_eq ? (tot >> 16) : R;
  const uint32_t nstrict = tot & 0xFFFFu;
  const uint32_t exc = wb + inc - packed;
  uint32_t sb = exc & 0xFFFFu, eb = exc >> 16;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = score_key(row[i]);
    const uint32_t top = key >> (32 - nbits);
    int pos = -1;
    if (top > prefix) {
      pos = static_cast<int>(sb++);
    } else if (top == prefix) {
      if (eb < take) pos = static_cast<int>(nstrict + eb);
      ++eb;
    }
    if (pos >= 0 && pos < k)
      cand[pos] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
  }
  int n2 = 1;
  while (n2 < k) n2 <<= 1;
  for (int i = k + tid; i < n2; i += kTopkThreads) cand[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n2; i += kTopkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = cand[i], c = cand[j];
          if ((a < c) == desc) {
            cand[i] = c;
            cand[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < k; i += kTopkThreads)
    out[static_cast<long long>(blockIdx.x) * k + i] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(cand[i]));
}

// ---------------------------------------------------------------------------
// HCA window compression: out[b, d] = sum_m softmax_m(z[b, :, d])[m] * c[b, m, d]
template <typename T>
__global__ void hca_compress_kernel(const T* __restrict__ c, const T* __restrict__ z, T* __restrict__ out, int B,
                                    int M, int D) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(B) * D) return;
  const int b = static_cast<int>(i / D), d = static_cast<int>(i % D);
  const long long base = static_cast<long long>(b) * M * D + d;
  float mx = -INFINITY;
  for (int m = 0; m < M; ++m) mx = fmaxf(mx, tofl<T>(z[base + static_cast<long long>(m) * D]));
  float den = 0.f, acc = 0.f;
  for (int m = 0; m < M; ++m) {
    const float e = __expf(tofl<T>(z[base + static_cast<long long>(m) * D]) - mx);
    den += e;
    acc += e * tofl<T>(c[base + static_cast<long long>(m) * D]);
  }
  out[i] = fromfl<T>(acc / den);
}

}  // namespace aether

using namespace aether;

extern "C" {

int aether_sparse_sink_attention(const void* q, const void* kv, const void* topk_indices, int idx_is_int64,
                                 const void* sink, int sink_numel, void* out, int dtype, int B, int T, int H, int D,
                                 int S, int K, float softmax_scale, void* stream) {
  AETHER_REQUIRE(topk_indices != nullptr, "topk_indices must not be null");
  return sink_attn_dispatch(q, kv, topk_indices, idx_is_int64, sink, sink_numel, out, dtype, B, T, H, D, S, K,
                            softmax_scale, static_cast<cudaStream_t>(stream));
}

int aether_tiled_prefill_attention(const void* q, const void* kv, const void* sink, int sink_numel, void* out,
                                   int dtype, int B, int T, int H, int D, int S, float softmax_scale, int tile_size,
                                   void* stream) {
  AETHER_REQUIRE(tile_size > 0, "tile_size must be positive");
  return sink_attn_dispatch(q, kv, nullptr, 0, sink, sink_numel, out, dtype, B, T, H, D, S, S, softmax_scale,
                            static_cast<cudaStream_t>(stream));
}

size_t aether_csa_indexer_topk_scratch_bytes(int B, int S) {
  return static_cast<size_t>(B) * static_cast<size_t>(S) * sizeof(float);
}

int aether_csa_indexer_topk(const float* index_q, const float* index_kv, const float* index_weight, int B, int IH,
                            int IC, int S, int k, float* scratch, int64_t* out, void* stream) {
  AETHER_REQUIRE(k > 0, "k must be positive");
  AETHER_REQUIRE(k <= S, "k (%d) must not exceed the number of sources (%d)", k, S);
  AETHER_REQUIRE(k <= kTopkMax, "k must be <= %d, got %d", kTopkMax, k);
  AETHER_REQUIRE(S < 65536, "csa_indexer_topk: at most 65535 sources per row, got %d", S);
  AETHER_REQUIRE(B >= 0, "csa_indexer_topk: batch must be non-negative, got %d", B);
  AETHER_REQUIRE(scratch != nullptr, "csa_indexer_topk: scratch buffer is required");
  if (B == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long warps = static_cast<long long>(B) * S;
  dense_index_score_kernel<<<(warps * 32 + 255) / 256, 256, 0, st>>>(index_q, index_kv, index_weight, scratch, B,
                                                                     IH, IC, S);
  row_topk_kernel<<<B, kTopkThreads, 0, st>>>(scratch, S, k, out);
  return check_launch("csa_indexer_topk");
}

int aether_hca_compress(const void* buffer_c, const void* buffer_z, void* out, int dtype, int B, int M, int D,
                        void* stream) {
  AETHER_REQUIRE(dtype >= 0 && dtype <= 2, "unsupported dtype code %d", dtype);
  AETHER_REQUIRE(M >= 1, "hca_compress: window must be non-empty");
  if (static_cast<long long>(B) * D == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long n = static_cast<long long>(B) * D;
  const int threads = 128;
  const long long blocks = (n + threads - 1) / threads;
  if (dtype == kCF32)
    hca_compress_kernel<float><<<blocks, threads, 0, st>>>(static_cast<const float*>(buffer_c),
                                                          static_cast<const float*>(buffer_z),
                                                          static_cast<float*>(out), B, M, D);
  else if (dtype == kCF16)
    hca_compress_kernel<__half><<<blocks, threads, 0, st>>>(static_cast<const __half*>(buffer_c),
                                                           static_cast<const __half*>(buffer_z),
                                                           static_cast<__half*>(out), B, M, D);
  else
    hca_compress_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(static_cast<const __nv_bfloat16*>(buffer_c),
                                                                  static_cast<const __nv_bfloat16*>(buffer_z),
                                                                  static_cast<__nv_bfloat16*>(out), B, M, D);
  return check_launch("hca_compress");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// csa_indexer_topk without any allocation.
//
// Some callers cannot allocate device memory at the point where they need the
// indexer: code running inside a host callback or a custom allocator's hook,
// engines that must not call cudaMalloc while another stream is being
// captured, or plugins that only ever receive the caller's input and output
// buffers.  For them this variant keeps its score buffer in a fixed array of
// the library itself, so nothing is allocated per call.
//
// Limit: batch * sources <= kNoAllocScores (1 Mi fp32 scores, 4 MiB).  Every
// GPU that loads the library holds that array until the process exits.
// The first call on a device, with that device current, looks up the array's
// device address (cudaGetSymbolAddress) and caches it; make that first call
// before any stream capture.  The cached address belongs to the device's
// current context: after cudaDeviceReset on a device, unload and reload the
// library before calling this entry point there again.  All calls share the one array: every call
// overwrites the scores it reads, so nothing has to be cleared, but two calls
// whose kernels overlap on the GPU (different streams, no ordering) race on it.
#include <mutex>

namespace aether {

constexpr long long kNoAllocScores = 1ll << 20;
static __device__ __align__(256) float g_noalloc_scores[kNoAllocScores];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {};

static int noalloc_scratch(float** out) {
  int dev = 0;
  AETHER_CUDA_TRY(cudaGetDevice(&dev), "csa_indexer_topk_noalloc: cudaGetDevice");
  AETHER_REQUIRE(dev >= 0 && dev < 64, "csa_indexer_topk_noalloc: device ordinal %d not supported", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    AETHER_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scores), "csa_indexer_topk_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace aether

extern "C" {

long long aether_csa_indexer_topk_noalloc_max_scores(void) { return aether::kNoAllocScores; }

int aether_csa_indexer_topk_noalloc(const float* index_q, const float* index_kv, const float* index_weight, int B,
                                    int IH, int IC, int S, int k, int64_t* out, void* stream) {
  AETHER_REQUIRE(k > 0, "k must be positive");
  AETHER_REQUIRE(k <= S, "k (%d) must not exceed the number of sources (%d)", k, S);
  AETHER_REQUIRE(k <= kTopkMax, "k must be <= %d, got %d", kTopkMax, k);
  AETHER_REQUIRE(S < 65536, "csa_indexer_topk_noalloc: at most 65535 sources per row, got %d", S);
  AETHER_REQUIRE(B >= 0 && static_cast<long long>(B) * S <= aether::kNoAllocScores,
                 "csa_indexer_topk_noalloc: batch * sources = %lld exceeds the built-in scratch of %lld scores",
                 static_cast<long long>(B) * S, aether::kNoAllocScores);
  if (B == 0) return 0;
  float* scratch = nullptr;
  const int rc = aether::noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long warps = static_cast<long long>(B) * S;
  dense_index_score_kernel<<<(warps * 32 + 255) / 256, 256, 0, st>>>(index_q, index_kv, index_weight, scratch, B, IH,
                                                                     IC, S);
  row_topk_kernel<<<B, kTopkThreads, 0, st>>>(scratch, S, k, out);
  return check_launch("csa_indexer_topk_noalloc");
}

}  // extern "C"
