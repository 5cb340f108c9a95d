// Shared device helpers for the sm_100a kernels of the TurboQuant paged-KV
// decode path: error reporting, bounded mbarrier waits, bulk (TMA) copies,
// cp.async, ldmatrix and warp-level mma.sync wrappers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace aether {

// Problem-shape constants fixed by the model (Aether2BConfig).
constexpr int kHeadDim = 128;   // attention_head_dim
constexpr int kIdxDim = 64;     // indexer_head_dim
constexpr int kIdxHeads = 4;    // indexer heads on the decode path
constexpr int kPage = 64;       // compressed entries per cache page
constexpr int kMaxHeads = 16;   // query heads are padded to one 16-row MMA tile

// Cache page layout: one page holds 64 entries as [64 x code row][64 x fp32
// scale], so a page (codes and scales) moves with a single bulk copy.
__host__ __device__ constexpr int page_bytes(int row_bytes) { return kPage * row_bytes + kPage * 4; }

// Error bits written by kernels into the caller's status word.
enum : int {
  kErrWaitTimeout = 1,   // an mbarrier / copy wait ran past its bound
  kErrBadPage = 2,       // a page-table entry was outside the pool
  kErrBadShape = 4,      // a runtime size exceeded a compiled limit
};

__device__ __forceinline__ void report_error(int* err, int bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Nanoseconds of the GPU's global timer (%globaltimer): bounds waits by
// elapsed time rather than by a count of polls, whose duration varies.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Every bounded wait in these kernels gives up after this long.  A wait that
// runs out means a copy or a producer was lost; the status word then carries
// kErrWaitTimeout and that launch's outputs are undefined.
constexpr uint64_t kWaitLimitNs = 200ull * 1000 * 1000;  // 0.2 s

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on phase `parity` of an mbarrier.  Returns false (and sets
// kErrWaitTimeout) if the phase has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int it = 0; it < 64; ++it)
      if (mbar_try_wait(addr, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  report_error(err, kErrWaitTimeout);
  return false;
}

// Bounded wait until the sequence word *flag has reached `target` (u32
// sequence numbers compared with wrap-around).  The word is written by a
// stream memory operation on a copy stream after that stream's copy, so the
// wait never depends on another kernel making progress.  Returns false (and
// sets kErrWaitTimeout) after kWaitLimitNs.
__device__ __forceinline__ bool flag_wait(const uint32_t* flag, uint32_t target, int* err) {
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (static_cast<int32_t>(v - target) >= 0) return true;
    if (it == 0) {
      t0 = global_ns();
    } else if (global_ns() - t0 > kWaitLimitNs) {
      break;
    }
    __nanosleep(100);
  }
  report_error(err, kErrWaitTimeout);
  return false;
}

// Bulk global->shared copy (TMA engine, no tensor map, no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------- ldmatrix
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

// ---------------------------------------------------------------- mma.sync
// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// D(16x8,s32) += A(16x32,s8,row) * B(32x8,s8,col)   (exact integer arithmetic)
__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Signed 4-bit codes (two's complement nibbles, even element in the low
// nibble) to signed bytes.  `lo` receives the low nibbles of the 4 bytes of w,
// `hi` the high nibbles.  n ^ 8 = v + 8 in [0,15]; adding 0x78 and flipping
// the top bit yields v as a two's complement byte without inter-byte carries.
__device__ __forceinline__ void nib_to_s8(uint32_t w, uint32_t& lo, uint32_t& hi) {
  uint32_t l = (w & 0x0F0F0F0Fu) ^ 0x08080808u;
  uint32_t h = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
  lo = (l + 0x78787878u) ^ 0x80808080u;
  hi = (h + 0x78787878u) ^ 0x80808080u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// softplus as torch.nn.functional.softplus(beta=1, threshold=20).
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }

}  // namespace aether
