// TurboQuant (PolarQuant) encode / decode kernels.
//
// Reference semantics: aether_2b/turbo_quant.py
//   encode (:127-166): y = WHT(diag * x) in fp32, m = max|y| clamped to 1e-8,
//                      code = clamp(round_half_even(y / m * L), -L, L),
//                      scale = m / L with L = 127 (int8) or 7 (4-bit, packed
//                      two's complement nibbles, even element low nibble)
//   decode (:168-211): x = WHT(code * scale) * diag, cast to the output dtype
//   _wht   (:49-76)  : radix-2 butterfly, stages h = 1, 2, 4, ..., then * d^-0.5
//
// One warp per vector.  Each lane holds d/32 consecutive elements; butterfly
// stages below d/32 run in registers, larger ones via shuffles.  Every
// floating-point step uses the explicitly rounded intrinsics in the reference
// op order (no contraction, IEEE division), so codes and scales are
// bit-identical to the reference's fp32 torch path.
#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"

namespace aether {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

template <int D>
struct WhtConst;
template <>
struct WhtConst<128> {
  // float32(128 ** -0.5), the value torch uses when it multiplies an fp32
  // tensor by the Python double 128 ** -0.5.
  static __device__ __forceinline__ float c() { return 0.0883883461356163f; }
};
template <>
struct WhtConst<64> {
  static __device__ __forceinline__ float c() { return 0.125f; }
};

template <typename T>
__device__ __forceinline__ float ld_as_float(const T* p);
template <>
__device__ __forceinline__ float ld_as_float<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_as_float<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_as_float<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <typename T>
__device__ __forceinline__ void st_from_float(T* p, float v);
template <>
__device__ __forceinline__ void st_from_float<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st_from_float<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <>
__device__ __forceinline__ void st_from_float<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

// In-warp normalised WHT of a D-vector held as EPL=D/32 consecutive elements
// per lane (element index 32-lane-major: i = lane*EPL + k).
template <int D>
__device__ __forceinline__ void warp_wht(float (&v)[D / 32], int lane) {
  constexpr int EPL = D / 32;
#pragma unroll
  for (int h = 1; h < D; h <<= 1) {
    if (h < EPL) {
#pragma unroll
      for (int k = 0; k < EPL; ++k) {
        if ((k & h) == 0) {
          float a = v[k], b = v[k + h];
          v[k] = __fadd_rn(a, b);
          v[k + h] = __fsub_rn(a, b);
        }
      }
    } else {
      const int ld = h / EPL;
      const bool upper = (lane & ld) != 0;
#pragma unroll
      for (int k = 0; k < EPL; ++k) {
        float p = __shfl_xor_sync(0xffffffffu, v[k], ld);
        v[k] = upper ? __fsub_rn(p, v[k]) : __fadd_rn(v[k], p);
      }
    }
  }
  const float c = WhtConst<D>::c();
#pragma unroll
  for (int k = 0; k < EPL; ++k) v[k] = __fmul_rn(v[k], c);
}

// Destination address resolution: either dense rows, or paged slots
// (page_table[seq * stride + pos / 64], slot pos % 64) for cache appends.
struct RowDst {
  const int32_t* page_table;  // null => dense rows
  const int32_t* start_pos;   // [B] first block position written per sequence
  int table_stride;
  int rows_per_seq;
  int num_pages;
};

// Byte offsets of a row's codes and scale.  Dense: codes[row], scales[row].
// Paged: page = page_table[seq, pos / 64], slot = pos % 64 inside the
// [codes | scales] page layout (page_bytes).
__device__ __forceinline__ bool resolve_row(const RowDst& r, long long row, int rb, int* err, long long& code_off,
                                            long long& scale_off) {
  if (!r.page_table) {
    code_off = row * rb;
    scale_off = row * 4;
    return true;
  }
  const int seq = static_cast<int>(row / r.rows_per_seq);
  const int pos = r.start_pos[seq] + static_cast<int>(row % r.rows_per_seq);
  const int page = r.page_table[static_cast<long long>(seq) * r.table_stride + (pos >> 6)];
  if (page < 0 || page >= r.num_pages) {
    report_error(err, kErrBadPage);
    return false;
  }
  const long long base = static_cast<long long>(page) * page_bytes(rb);
  code_off = base + (pos & (kPage - 1)) * rb;
  scale_off = base + kPage * rb + (pos & (kPage - 1)) * 4;
  return true;
}

// Quantise a rotated vector (absmax m already clamped) and store one row:
// codes at row_codes (D or D/2 bytes), scale m / L at *scale.
template <int D, int BITS>
__device__ __forceinline__ void quantize_store(const float (&v)[D / 32], float m, int lane, uint8_t* row_codes,
                                               float* scale) {
  constexpr int EPL = D / 32;
  constexpr float L = BITS == 8 ? 127.f : 7.f;
  if (lane == 0) *scale = __fdiv_rn(m, L);
  int q[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    float t = rintf(__fmul_rn(__fdiv_rn(v[k], m), L));
    t = fminf(fmaxf(t, -L), L);
    q[k] = static_cast<int>(t);
  }
  if (BITS == 8) {
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < EPL; ++k) w |= (static_cast<uint32_t>(q[k]) & 0xFFu) << (8 * k);
    uint8_t* base = row_codes + lane * EPL;
    if (EPL == 4)
      *reinterpret_cast<uint32_t*>(base) = w;
    else
      *reinterpret_cast<uint16_t*>(base) = static_cast<uint16_t>(w);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < EPL; ++k) w |= (static_cast<uint32_t>(q[k]) & 0xFu) << (4 * k);
    uint8_t* base = row_codes + lane * (EPL / 2);
    if (EPL == 4)
      *reinterpret_cast<uint16_t*>(base) = static_cast<uint16_t>(w);
    else
      *base = static_cast<uint8_t>(w);
  }
}

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(256) tq_encode_kernel(const T* __restrict__ x, const float* __restrict__ diag,
                                                       uint8_t* __restrict__ codes, float* __restrict__ scales,
                                                       long long rows, RowDst dst, int* err) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  float v[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    const int i = lane * EPL + k;
    v[k] = __fmul_rn(ld_as_float(x + row * D + i), diag[i]);
  }
  warp_wht<D>(v, lane);
  float m = 0.f;
#pragma unroll
  for (int k = 0; k < EPL; ++k) m = fmaxf(m, fabsf(v[k]));
  m = warp_max(m);
  m = fmaxf(m, 9.99999993922529e-09f);  // float32(1e-8), torch clamp_(min=1e-8)
  constexpr int RB = BITS == 8 ? D : D / 2;
  long long coff, soff;
  if (!resolve_row(dst, row, RB, err, coff, soff)) return;
  uint8_t* scale_base = dst.page_table ? codes : reinterpret_cast<uint8_t*>(scales);
  quantize_store<D, BITS>(v, m, lane, codes + coff, reinterpret_cast<float*>(scale_base + soff));
}


// ------------------------------------------------------------ compress-on-emit
// One source segment of a compressed block: rows [B, rows, D] of values c and
// gate logits z, plus an optional per-row bias [rows, D] added to z.
struct EmitSeg {
  const void* c;
  const void* z;
  const float* bias;
  int rows;
};

struct EmitParams {
  EmitSeg s0, s1;            // s1.rows == 0: single segment (HCA)
  const int32_t* has_s1;     // [B] 0 => s1 skipped for that sequence (CSA first block); null => all use it
  int B;
  const int32_t* positions;  // [B] RoPE position of the emitted entry
  const float* inv_freq;     // [rope_dim / 2]
  int rope_dim;              // 0 => no RoPE
  const float* norm_w;       // [D]; null => no RMSNorm
  float norm_eps;
  const float* diag;         // [D] Rademacher diagonal
  uint8_t* pool;             // page pool; null => no cache write
  float* out;                // [B, D] fp32 compressed entry before quantisation; may be null
};

// Online softmax over the rows of one segment, per channel.
template <int D, typename T>
__device__ __forceinline__ void emit_accumulate(const EmitSeg& sg, int b, int lane, float (&mx)[D / 32],
                                                float (&den)[D / 32], float (&acc)[D / 32]) {
  constexpr int EPL = D / 32;
  const T* c = static_cast<const T*>(sg.c) + static_cast<long long>(b) * sg.rows * D;
  const T* z = static_cast<const T*>(sg.z) + static_cast<long long>(b) * sg.rows * D;
  for (int r = 0; r < sg.rows; ++r) {
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
      const int i = lane * EPL + k;
      float zz = ld_as_float(z + r * D + i);
      if (sg.bias) zz += sg.bias[r * D + i];
      const float cc = ld_as_float(c + r * D + i);
      if (zz > mx[k]) {
        const float f = expf(mx[k] - zz);  // mx = -inf => 0
        den[k] = den[k] * f + 1.f;
        acc[k] = acc[k] * f + cc;
        mx[k] = zz;
      } else {
        const float e = expf(zz - mx[k]);
        den[k] += e;
        acc[k] += e * cc;
      }
    }
  }
}

// One warp per emitting sequence: gated softmax pooling over the block's
// rows, RoPE of the last rope_dim channels (interleaved pairs), RMSNorm,
// TurboQuant encode and the write into the sequence's page slot.
template <int D, int BITS, typename T>
__global__ void __launch_bounds__(256) compress_emit_kernel(EmitParams p, RowDst dst, int* err) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (b >= p.B) return;
  float mx[EPL], den[EPL], acc[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    mx[k] = -INFINITY;
    den[k] = 0.f;
    acc[k] = 0.f;
  }
  emit_accumulate<D, T>(p.s0, b, lane, mx, den, acc);
  if (p.s1.rows > 0 && (p.has_s1 == nullptr || p.has_s1[b] != 0)) emit_accumulate<D, T>(p.s1, b, lane, mx, den, acc);
  float v[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) v[k] = den[k] > 0.f ? acc[k] / den[k] : 0.f;

  if (p.rope_dim > 0) {
    const float pos = static_cast<float>(p.positions[b]);
    const int first = D - p.rope_dim;
#pragma unroll
    for (int k = 0; k < EPL; k += 2) {
      const int i = lane * EPL + k;  // even channel of the pair (i, i + 1)
      if (i >= first) {
        const float ang = pos * p.inv_freq[(i - first) >> 1];
        const float cs = cosf(ang), sn = sinf(ang);
        const float x0 = v[k], x1 = v[k + 1];
        v[k] = x0 * cs - x1 * sn;
        v[k + 1] = x1 * cs + x0 * sn;
      }
    }
  }
  if (p.norm_w) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < EPL; ++k) ss += v[k] * v[k];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + p.norm_eps);
#pragma unroll
    for (int k = 0; k < EPL; ++k) v[k] = v[k] * r * p.norm_w[lane * EPL + k];
  }
  if (p.out) {
#pragma unroll
    for (int k = 0; k < EPL; ++k) p.out[static_cast<long long>(b) * D + lane * EPL + k] = v[k];
  }
  if (!p.pool) return;
#pragma unroll
  for (int k = 0; k < EPL; ++k) v[k] = __fmul_rn(v[k], p.diag[lane * EPL + k]);
  warp_wht<D>(v, lane);
  float m = 0.f;
#pragma unroll
  for (int k = 0; k < EPL; ++k) m = fmaxf(m, fabsf(v[k]));
  m = warp_max(m);
  m = fmaxf(m, 9.99999993922529e-09f);
  constexpr int RB = BITS == 8 ? D : D / 2;
  long long coff, soff;
  if (!resolve_row(dst, b, RB, err, coff, soff)) return;
  quantize_store<D, BITS>(v, m, lane, p.pool + coff, reinterpret_cast<float*>(p.pool + soff));
}

template <int D, int BITS>
static void launch_emit_t(int dtype, const EmitParams& p, const RowDst& dst, int* err, cudaStream_t st) {
  const int blocks = (p.B * 32 + 255) / 256;
  switch (dtype) {
    case kF32: compress_emit_kernel<D, BITS, float><<<blocks, 256, 0, st>>>(p, dst, err); break;
    case kF16: compress_emit_kernel<D, BITS, __half><<<blocks, 256, 0, st>>>(p, dst, err); break;
    default: compress_emit_kernel<D, BITS, __nv_bfloat16><<<blocks, 256, 0, st>>>(p, dst, err);
  }
}

// ------------------------------------------------- Lloyd-Max level format
// Alternative to the uniform levels: y = WHT(diag * x), scale = max|y| /
// c_max, and each element the index of the nearest of the 2^BITS levels
// (thr: the 2^BITS - 1 ascending fp32 midpoints; code = number of
// thresholds strictly below y / scale, i.e. the lower index on a midpoint).
// 8-bit: one index byte per element; 4-bit: index nibbles, even element low.
template <int D, int BITS, typename T>
__global__ void __launch_bounds__(256) tq_encode_lut_kernel(const T* __restrict__ x, const float* __restrict__ diag,
                                                           const float* __restrict__ thr, float cmax,
                                                           uint8_t* __restrict__ codes, float* __restrict__ scales,
                                                           long long rows) {
  constexpr int EPL = D / 32;
  constexpr int NT = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  float v[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    const int i = lane * EPL + k;
    v[k] = __fmul_rn(ld_as_float(x + row * D + i), diag[i]);
  }
  warp_wht<D>(v, lane);
  float m = 0.f;
#pragma unroll
  for (int k = 0; k < EPL; ++k) m = fmaxf(m, fabsf(v[k]));
  m = warp_max(m);
  m = fmaxf(m, 9.99999993922529e-09f);
  const float scale = __fdiv_rn(m, cmax);
  if (lane == 0) scales[row] = scale;
  int q[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    const float u = __fdiv_rn(v[k], scale);
    int lo = 0, hi = NT;  // first threshold >= u
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (thr[mid] < u)
        lo = mid + 1;
      else
        hi = mid;
    }
    q[k] = lo;
  }
  if (BITS == 8) {
    uint8_t* base = codes + row * D + lane * EPL;
#pragma unroll
    for (int k = 0; k < EPL; ++k) base[k] = static_cast<uint8_t>(q[k]);
  } else {
    uint8_t* base = codes + row * (D / 2) + lane * (EPL / 2);
#pragma unroll
    for (int k = 0; k < EPL / 2; ++k) base[k] = static_cast<uint8_t>(q[2 * k] | (q[2 * k + 1] << 4));
  }
}

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(256) tq_decode_lut_kernel(const uint8_t* __restrict__ codes,
                                                           const float* __restrict__ scales,
                                                           const float* __restrict__ diag,
                                                           const float* __restrict__ levels, T* __restrict__ out,
                                                           long long rows) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float s = scales[row];
  float v[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    const int i = lane * EPL + k;
    const int c = BITS == 8 ? codes[row * D + i] : (codes[row * (D / 2) + i / 2] >> (4 * (i & 1))) & 0xF;
    v[k] = __fmul_rn(levels[c], s);
  }
  warp_wht<D>(v, lane);
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    const int i = lane * EPL + k;
    st_from_float<T>(out + row * D + i, __fmul_rn(v[k], diag[i]));
  }
}

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(256) tq_decode_kernel(const uint8_t* __restrict__ codes,
                                                       const float* __restrict__ scales,
                                                       const float* __restrict__ diag, T* __restrict__ out,
                                                       long long rows) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const float s = scales[row];
  float v[EPL];
  if (BITS == 8) {
    const int8_t* c = reinterpret_cast<const int8_t*>(codes) + row * D + lane * EPL;
#pragma unroll
    for (int k = 0; k < EPL; ++k) v[k] = __fmul_rn(static_cast<float>(c[k]), s);
  } else {
    const uint8_t* c = codes + row * (D / 2) + lane * (EPL / 2);
#pragma unroll
    for (int k = 0; k < EPL / 2; ++k) {
      int b = c[k];
      int lo = b & 0xF, hi = (b >> 4) & 0xF;
      lo = lo >= 8 ? lo - 16 : lo;
      hi = hi >= 8 ? hi - 16 : hi;
      v[2 * k] = __fmul_rn(static_cast<float>(lo), s);
      v[2 * k + 1] = __fmul_rn(static_cast<float>(hi), s);
    }
  }
  warp_wht<D>(v, lane);
#pragma unroll
  for (int k = 0; k < EPL; ++k) {
    const int i = lane * EPL + k;
    st_from_float<T>(out + row * D + i, __fmul_rn(v[k], diag[i]));
  }
}

template <int D, int BITS>
static void launch_encode_t(int dtype, const void* x, const float* diag, uint8_t* codes, float* scales,
                            long long rows, RowDst dst, int* err, cudaStream_t st) {
  const int threads = 256;
  const long long blocks = (rows * 32 + threads - 1) / threads;
  switch (dtype) {
    case kF32:
      tq_encode_kernel<D, BITS, float><<<blocks, threads, 0, st>>>(static_cast<const float*>(x), diag, codes,
                                                                   scales, rows, dst, err);
      break;
    case kF16:
      tq_encode_kernel<D, BITS, __half><<<blocks, threads, 0, st>>>(static_cast<const __half*>(x), diag, codes,
                                                                    scales, rows, dst, err);
      break;
    default:
      tq_encode_kernel<D, BITS, __nv_bfloat16><<<blocks, threads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(x), diag, codes, scales, rows, dst, err);
  }
}

static int launch_encode(int dtype, const void* x, const float* diag, uint8_t* codes, float* scales,
                         long long rows, int d, int bits, RowDst dst, int* err, cudaStream_t st) {
  AETHER_REQUIRE(d == 64 || d == 128, "turbo_quant encode: last dim must be 64 or 128, got %d", d);
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(dtype >= 0 && dtype <= 2, "turbo_quant encode: unsupported dtype code %d", dtype);
  if (rows == 0) return 0;
  if (d == 128 && bits == 8) launch_encode_t<128, 8>(dtype, x, diag, codes, scales, rows, dst, err, st);
  if (d == 128 && bits == 4) launch_encode_t<128, 4>(dtype, x, diag, codes, scales, rows, dst, err, st);
  if (d == 64 && bits == 8) launch_encode_t<64, 8>(dtype, x, diag, codes, scales, rows, dst, err, st);
  if (d == 64 && bits == 4) launch_encode_t<64, 4>(dtype, x, diag, codes, scales, rows, dst, err, st);
  return check_launch("turbo_quant encode");
}

template <int D, int BITS>
static void launch_decode_t(int dtype, const uint8_t* codes, const float* scales, const float* diag, void* out,
                            long long rows, cudaStream_t st) {
  const int threads = 256;
  const long long blocks = (rows * 32 + threads - 1) / threads;
  switch (dtype) {
    case kF32:
      tq_decode_kernel<D, BITS, float><<<blocks, threads, 0, st>>>(codes, scales, diag, static_cast<float*>(out),
                                                                   rows);
      break;
    case kF16:
      tq_decode_kernel<D, BITS, __half><<<blocks, threads, 0, st>>>(codes, scales, diag,
                                                                    static_cast<__half*>(out), rows);
      break;
    default:
      tq_decode_kernel<D, BITS, __nv_bfloat16><<<blocks, threads, 0, st>>>(
          codes, scales, diag, static_cast<__nv_bfloat16*>(out), rows);
  }
}

}  // namespace aether

using namespace aether;

extern "C" {

int aether_tq_encode(const void* x, int dtype, long long rows, int d, int bits, const float* diag,
                     uint8_t* codes, float* scales, int* err, void* stream) {
  RowDst dst{nullptr, nullptr, 0, 1, 0};
  return launch_encode(dtype, x, diag, codes, scales, rows, d, bits, dst, err, static_cast<cudaStream_t>(stream));
}

int aether_tq_encode_into_pages(const void* x, int dtype, int batch, int rows_per_seq, int d, int bits,
                                const float* diag, const int32_t* page_table, int table_stride,
                                const int32_t* start_pos, int num_pages, uint8_t* page_pool, int* err,
                                void* stream) {
  AETHER_REQUIRE(page_table && start_pos, "encode_into_pages: page_table and start_pos are required");
  AETHER_REQUIRE(batch >= 0 && rows_per_seq >= 0, "encode_into_pages: negative size");
  RowDst dst{page_table, start_pos, table_stride, rows_per_seq > 0 ? rows_per_seq : 1, num_pages};
  return launch_encode(dtype, x, diag, page_pool, nullptr, static_cast<long long>(batch) * rows_per_seq, d, bits,
                       dst, err, static_cast<cudaStream_t>(stream));
}

int aether_compress_emit(const void* c0, const void* z0, const float* bias0, int rows0, const void* c1,
                         const void* z1, const float* bias1, int rows1, const int32_t* has_seg1, int dtype, int B,
                         int d, const int32_t* positions, const float* inv_freq, int rope_dim,
                         const float* norm_weight, float norm_eps, int bits, const float* diag,
                         const int32_t* page_table, int table_stride, const int32_t* slot_pos, int num_pages,
                         uint8_t* page_pool, float* out, int* err, void* stream) {
  AETHER_REQUIRE(d == 64 || d == 128, "compress_emit: dim must be 64 or 128, got %d", d);
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(dtype >= 0 && dtype <= 2, "compress_emit: unsupported dtype code %d", dtype);
  AETHER_REQUIRE(B >= 0 && rows0 > 0 && rows1 >= 0, "compress_emit: bad sizes B=%d rows0=%d rows1=%d", B, rows0,
                 rows1);
  AETHER_REQUIRE(c0 && z0 && (rows1 == 0 || (c1 && z1)), "compress_emit: missing segment tensors");
  AETHER_REQUIRE(rope_dim >= 0 && rope_dim <= d && rope_dim % 2 == 0, "compress_emit: rope_dim must be even and <= dim");
  AETHER_REQUIRE(rope_dim == 0 || (positions && inv_freq), "compress_emit: RoPE needs positions and inv_freq");
  AETHER_REQUIRE(page_pool == nullptr || (diag && page_table && slot_pos),
                 "compress_emit: a cache write needs diag, page_table and slot_pos");
  AETHER_REQUIRE(page_pool != nullptr || out != nullptr, "compress_emit: nothing to write (no page_pool, no out)");
  if (B == 0) return 0;
  EmitParams p{{c0, z0, bias0, rows0}, {c1, z1, bias1, rows1}, has_seg1, B, positions, inv_freq, rope_dim,
               norm_weight, norm_eps, diag, page_pool, out};
  RowDst dst{page_table, slot_pos, table_stride, 1, num_pages};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d == 128 && bits == 8) launch_emit_t<128, 8>(dtype, p, dst, err, st);
  if (d == 128 && bits == 4) launch_emit_t<128, 4>(dtype, p, dst, err, st);
  if (d == 64 && bits == 8) launch_emit_t<64, 8>(dtype, p, dst, err, st);
  if (d == 64 && bits == 4) launch_emit_t<64, 4>(dtype, p, dst, err, st);
  return check_launch("compress_emit");
}

int aether_tq_encode_lut(const void* x, int dtype, long long rows, int d, int bits, const float* diag,
                         const float* thresholds, float cmax, uint8_t* codes, float* scales, void* stream) {
  AETHER_REQUIRE(d == 64 || d == 128, "turbo_quant encode: last dim must be 64 or 128, got %d", d);
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(dtype >= 0 && dtype <= 2, "turbo_quant encode: unsupported dtype code %d", dtype);
  AETHER_REQUIRE(cmax > 0.f && thresholds, "turbo_quant encode: bad codebook");
  if (rows == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long blocks = (rows * 32 + 255) / 256;
#define AETHER_ENC_LUT(DD, BB)                                                                                   \
  if (d == DD && bits == BB) {                                                                                   \
    if (dtype == kF32)                                                                                           \
      tq_encode_lut_kernel<DD, BB, float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), diag,          \
                                                                  thresholds, cmax, codes, scales, rows);      \
    else if (dtype == kF16)                                                                                      \
      tq_encode_lut_kernel<DD, BB, __half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x), diag,        \
                                                                   thresholds, cmax, codes, scales, rows);     \
    else                                                                                                         \
      tq_encode_lut_kernel<DD, BB, __nv_bfloat16><<<blocks, 256, 0, st>>>(                                     \
          static_cast<const __nv_bfloat16*>(x), diag, thresholds, cmax, codes, scales, rows);                  \
  }
  AETHER_ENC_LUT(128, 8)
  AETHER_ENC_LUT(128, 4)
  AETHER_ENC_LUT(64, 8)
  AETHER_ENC_LUT(64, 4)
#undef AETHER_ENC_LUT
  return check_launch("turbo_quant encode (Lloyd-Max levels)");
}

int aether_tq_decode_lut(const uint8_t* codes, const float* scales, long long rows, int d, int bits,
                         const float* diag, const float* levels, void* out, int out_dtype, void* stream) {
  AETHER_REQUIRE(d == 64 || d == 128, "turbo_quant decode: last dim must be 64 or 128, got %d", d);
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(out_dtype >= 0 && out_dtype <= 2, "turbo_quant decode: unsupported dtype code %d", out_dtype);
  AETHER_REQUIRE(levels != nullptr, "turbo_quant decode: null codebook");
  if (rows == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long blocks = (rows * 32 + 255) / 256;
#define AETHER_DEC_LUT(DD, BB)                                                                                   \
  if (d == DD && bits == BB) {                                                                                   \
    if (out_dtype == kF32)                                                                                       \
      tq_decode_lut_kernel<DD, BB, float><<<blocks, 256, 0, st>>>(codes, scales, diag, levels,                 \
                                                                  static_cast<float*>(out), rows);             \
    else if (out_dtype == kF16)                                                                                  \
      tq_decode_lut_kernel<DD, BB, __half><<<blocks, 256, 0, st>>>(codes, scales, diag, levels,                \
                                                                   static_cast<__half*>(out), rows);           \
    else                                                                                                         \
      tq_decode_lut_kernel<DD, BB, __nv_bfloat16><<<blocks, 256, 0, st>>>(codes, scales, diag, levels,         \
                                                                          static_cast<__nv_bfloat16*>(out), rows); \
  }
  AETHER_DEC_LUT(128, 8)
  AETHER_DEC_LUT(128, 4)
  AETHER_DEC_LUT(64, 8)
  AETHER_DEC_LUT(64, 4)
#undef AETHER_DEC_LUT
  return check_launch("turbo_quant decode (Lloyd-Max levels)");
}

int aether_tq_decode(const uint8_t* codes, const float* scales, long long rows, int d, int bits,
                     const float* diag, void* out, int out_dtype, void* stream) {
  AETHER_REQUIRE(d == 64 || d == 128, "turbo_quant decode: last dim must be 64 or 128, got %d", d);
  AETHER_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8, got %d", bits);
  AETHER_REQUIRE(out_dtype >= 0 && out_dtype <= 2, "turbo_quant decode: unsupported dtype code %d", out_dtype);
  if (rows == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d == 128 && bits == 8) launch_decode_t<128, 8>(out_dtype, codes, scales, diag, out, rows, st);
  if (d == 128 && bits == 4) launch_decode_t<128, 4>(out_dtype, codes, scales, diag, out, rows, st);
  if (d == 64 && bits == 8) launch_decode_t<64, 8>(out_dtype, codes, scales, diag, out, rows, st);
  if (d == 64 && bits == 4) launch_decode_t<64, 4>(out_dtype, codes, scales, diag, out, rows, st);
  return check_launch("turbo_quant decode");
}

}  // extern "C"

namespace aether {
template <int D>
__global__ void __launch_bounds__(256) wht_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                  long long rows) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  float v[EPL];
#pragma unroll
  for (int k = 0; k < EPL; ++k) v[k] = x[row * D + lane * EPL + k];
  warp_wht<D>(v, lane);
#pragma unroll
  for (int k = 0; k < EPL; ++k) out[row * D + lane * EPL + k] = v[k];
}
}  // namespace aether

extern "C" int aether_wht(const float* x, float* out, long long rows, int d, void* stream) {
  AETHER_REQUIRE(d == 64 || d == 128, "wht kernel supports last dim 64 or 128, got %d", d);
  if (rows == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long blocks = (rows * 32 + 255) / 256;
  if (d == 128) aether::wht_kernel<128><<<blocks, 256, 0, st>>>(x, out, rows);
  else aether::wht_kernel<64><<<blocks, 256, 0, st>>>(x, out, rows);
  return aether::check_launch("wht");
}
