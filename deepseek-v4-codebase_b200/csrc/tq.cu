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

template <int D, int BITS, typename T>
__global__ void __launch_bounds__(256) tq_encode_kernel(const T* __restrict__ x, const float* __restrict__ diag,
                                                       uint8_t* __restrict__ codes, float* __restrict__ scales,
                                                       long long rows, RowDst dst, int* err) {
  constexpr int EPL = D / 32;
  constexpr float L = BITS == 8 ? 127.f : 7.f;
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
  if (lane == 0) *reinterpret_cast<float*>(scale_base + soff) = __fdiv_rn(m, L);
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
    uint8_t* base = codes + coff + lane * EPL;
    if (EPL == 4)
      *reinterpret_cast<uint32_t*>(base) = w;
    else
      *reinterpret_cast<uint16_t*>(base) = static_cast<uint16_t>(w);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < EPL; ++k) w |= (static_cast<uint32_t>(q[k]) & 0xFu) << (4 * k);
    uint8_t* base = codes + coff + lane * (EPL / 2);
    if (EPL == 4)
      *reinterpret_cast<uint16_t*>(base) = static_cast<uint16_t>(w);
    else
      *base = static_cast<uint8_t>(w);
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
