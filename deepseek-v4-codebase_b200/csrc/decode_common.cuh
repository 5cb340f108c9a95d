// Device helpers shared by the paged decode kernels (sm_100a): code-to-fp16
// conversion, bf16 mma, the in-warp 128-point WHT, programmatic-dependent-
// launch controls and the fixed-point limbs of the rotated index query.
#pragma once

#include "common.cuh"

namespace aether {

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// nibble pair of one byte -> half2(lo, hi), exact signed values
__device__ __forceinline__ uint32_t nib_byte_to_h2(uint32_t byte) {
  uint32_t y = (byte & 0xFu) | ((byte & 0xF0u) << 12);
  y = (y ^ 0x00080008u) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));  // 1032
  return *reinterpret_cast<uint32_t*>(&h);
}
// two int8 codes (low 16 bits of w) -> half2
__device__ __forceinline__ uint32_t s8pair_to_h2(uint32_t w) {
  uint32_t y = __byte_perm(w ^ 0x8080u, 0x64646464u, 0x5140);  // [b0^80, 0x64, b1^80, 0x64]
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));  // 1152
  return *reinterpret_cast<uint32_t*>(&h);
}
// selected nibble (shift sh) of two bytes -> half2
__device__ __forceinline__ uint32_t two_nib_to_h2(uint32_t b0, uint32_t b1, int sh) {
  uint32_t y = ((b0 >> sh) & 0xFu) | (((b1 >> sh) & 0xFu) << 16);
  y = (y ^ 0x00080008u) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&y);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t two_s8_to_h2(uint32_t b0, uint32_t b1) {
  return s8pair_to_h2((b0 & 0xFFu) | ((b1 & 0xFFu) << 8));
}
__device__ __forceinline__ uint32_t bf2_to_h2(uint32_t v) {
  const __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  const float2 f = __bfloat1622float2(b);
  return pack_half2(f.x, f.y);
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Entry `i` of the shared code LUT: uniform 4-bit codes map a byte to the
// half2 of its two signed nibbles; a level table (Lloyd-Max format) maps a
// 4-bit byte to half2(levels[lo], levels[hi]) and an 8-bit code to
// half(levels[i]) in the low half.  Uniform 8-bit codes convert
// arithmetically (s8pair_to_h2) and need no entry.
__device__ __forceinline__ uint32_t code_lut_entry(int bits, const float* levels, uint32_t i) {
  if (levels) return bits == 4 ? pack_half2(levels[i & 15u], levels[i >> 4]) : pack_half2(levels[i], 0.f);
  return nib_byte_to_h2(i);
}
// two 8-bit codes (low 16 bits of w) -> half2, uniform or through the LUT
__device__ __forceinline__ uint32_t code8_pair(uint32_t w, const uint32_t* lut, bool levels) {
  if (!levels) return s8pair_to_h2(w & 0xFFFFu);
  return (lut[w & 0xFFu] & 0xFFFFu) | (lut[(w >> 8) & 0xFFu] << 16);
}

// In-warp normalised 128-point WHT of 4 consecutive values per lane (unscaled).
__device__ __forceinline__ void warp_wht128(float (&v)[4], int lane) {
  {
    const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
    v[0] = a0 + a2;
    v[2] = a0 - a2;
    v[1] = a1 + a3;
    v[3] = a1 - a3;
  }
#pragma unroll
  for (int ld = 1; ld < 32; ld <<= 1) {
    const bool up = (lane & ld) != 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float o = __shfl_xor_sync(0xffffffffu, v[k], ld);
      v[k] = up ? o - v[k] : v[k] + o;
    }
  }
}


// Rotated index query of head `warp` (warps 0-3): 24-bit limbs into `limb`,
// their per-limb sums and alpha_h = softplus(w_h) * scale_h into misc.
// Rotated index query of head h, WHT(diag * q_h) with the normalised
// 64-point WHT: lane l holds dims 2l and 2l + 1 (in-warp butterfly).
__device__ __forceinline__ void rotate_index_query(const float* index_q, const float* diag_idx, int b, int h,
                                                   int lane, float& v0, float& v1) {
  const float* src = index_q + (static_cast<long long>(b) * kIdxHeads + h) * kIdxDim;
  v0 = src[lane * 2] * diag_idx[lane * 2];
  v1 = src[lane * 2 + 1] * diag_idx[lane * 2 + 1];
  {
    const float a = v0, c2 = v1;
    v0 = a + c2;
    v1 = a - c2;
  }
#pragma unroll
  for (int ld = 1; ld < 32; ld <<= 1) {
    const bool up = (lane & ld) != 0;
    const float o0 = __shfl_xor_sync(0xffffffffu, v0, ld);
    const float o1 = __shfl_xor_sync(0xffffffffu, v1, ld);
    v0 = up ? o0 - v0 : v0 + o0;
    v1 = up ? o1 - v1 : v1 + o1;
  }
  v0 *= 0.125f;
  v1 *= 0.125f;
}

__device__ __forceinline__ void index_query_limbs(const float* index_q, const float* index_w, const float* diag_idx,
                                                  int b, int warp, int lane, int8_t* limb, float* alpha,
                                                  int (*lsum)[3]) {
  const int h = warp;
  // the head weight is loaded with the query, not after the quantisation
  // (one global-load latency instead of two)
  const float wh = index_w[b * kIdxHeads + h];
  float v0, v1;
  rotate_index_query(index_q, diag_idx, b, h, lane, v0, v1);
  const float am = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
  const float s = am > 0.f ? am / 8355000.0f : 1.0f;
  int ls[3] = {0, 0, 0};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int v = __float2int_rn(__fdiv_rn(k ? v1 : v0, s));
    const int l0 = ((v + 128) & 255) - 128;
    const int w1 = (v - l0) >> 8;
    const int l1 = ((w1 + 128) & 255) - 128;
    const int l2 = (w1 - l1) >> 8;
    const int d = lane * 2 + k;
    limb[(h * 3 + 0) * kIdxDim + d] = static_cast<int8_t>(l0);
    limb[(h * 3 + 1) * kIdxDim + d] = static_cast<int8_t>(l1);
    limb[(h * 3 + 2) * kIdxDim + d] = static_cast<int8_t>(l2);
    ls[0] += l0;
    ls[1] += l1;
    ls[2] += l2;
  }
#pragma unroll
  for (int l = 0; l < 3; ++l) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls[l] += __shfl_xor_sync(0xffffffffu, ls[l], o);
  }
  if (lane == 0) {
    alpha[h] = softplus_f(wh) * s;
    lsum[h][0] = ls[0];
    lsum[h][1] = ls[1];
    lsum[h][2] = ls[2];
  }
}


// Per-lane B fragments of the s8 limb MMAs (m16n8k32, lane = 4 g + t):
// n-tile 0 column g is (head g/2, limb g%2), n-tile 1 column g is (head
// g/2, limb 2) for even g and zero for odd g; words [tile][k-half][reg].
// 4-bit codes enter the MMA as v + 8, so the accumulators start at
// -8 * (sum of the limb over the dims): c0i, c1i, c2i for lane t's head.
template <int BITS>
__device__ __forceinline__ void limb_fragments(const int8_t* limb, const int (*lsum)[3], int g, int t,
                                               uint32_t (&bq)[2][2][2], int& c0i, int& c1i, int& c2i) {
  const int hq = g >> 1;
  // eight consecutive limb bytes per (j, limb row) in one 8-byte load (limb
  // rows start 8-byte aligned); 8-bit codes take them in order, 4-bit codes
  // (dims interleaved by nibble) take the even bytes for hh = 0, odd for 1
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int d0 = 16 * t + 8 * j;
    const uint2 a8 = *reinterpret_cast<const uint2*>(limb + (hq * 3 + (g & 1)) * kIdxDim + d0);
    const uint2 b8 = (g & 1) ? make_uint2(0u, 0u) : *reinterpret_cast<const uint2*>(limb + (hq * 3 + 2) * kIdxDim + d0);
    if (BITS == 4) {
      bq[0][j][0] = __byte_perm(a8.x, a8.y, 0x6420);
      bq[0][j][1] = __byte_perm(a8.x, a8.y, 0x7531);
      bq[1][j][0] = __byte_perm(b8.x, b8.y, 0x6420);
      bq[1][j][1] = __byte_perm(b8.x, b8.y, 0x7531);
    } else {
      bq[0][j][0] = a8.x;
      bq[0][j][1] = a8.y;
      bq[1][j][0] = b8.x;
      bq[1][j][1] = b8.y;
    }
  }
  c0i = BITS == 4 ? -8 * lsum[t][0] : 0;
  c1i = BITS == 4 ? -8 * lsum[t][1] : 0;
  c2i = BITS == 4 ? -8 * lsum[t][2] : 0;
}

}  // namespace aether
