// Peer-memory exchange for context-parallel decode (one long sequence split
// by block range over G GPUs, one process per GPU).  It replaces the two
// all-gathers of a step (candidate lists, then partial attention results) by
// plain stores into the other GPUs' memory over NVLink:
//
//   * every rank owns one exchange buffer (cudaMalloc'd here) and shares its
//     CUDA IPC handle; the others open it, so each rank holds G base
//     pointers, its own among them;
//   * aether_peer_push copies a block of rows into this rank's slot of every
//     buffer, makes the stores visible system-wide, then writes this rank's
//     flag word in every buffer with a release store;
//   * aether_peer_wait returns once all G flag words of a kind have reached
//     the step's sequence number (acquire loads, bounded by kWaitLimitNs; a
//     timeout sets the error word and returns).
//
// Sequence numbers live in device memory (the control area's step word), so
// a captured CUDA graph replays correctly: the first push of a step bumps
// the word and every later push / wait of the step reads it.  No TMA, no
// multicast: plain 16-byte loads and stores.
//
// Control area (the first 256 bytes of every buffer): u32 flags[kinds][8] at
// byte 0, the step word at byte 128.
#include "aether_b200.h"
#include "capi_util.cuh"
#include "common.cuh"

namespace aether {
namespace cpx {

constexpr int kMaxRanks = 8;
constexpr int kMaxKinds = 4;
constexpr int kStepWordOffset = 128;
constexpr int kPushThreads = 1024;

struct PushArgs {
  const uint8_t* src;
  long long rows, row_bytes, src_stride;
  long long dst_offset, dst_stride, dst_col;  // bytes within each buffer
  uint8_t* dst[kMaxRanks];                    // every rank's buffer base (this rank's included)
  int G, rank, kind, bump;
  uint32_t* step_word;  // this rank's step word (local buffer)
};

__global__ void __launch_bounds__(kPushThreads) peer_push_kernel(PushArgs a) {
  __shared__ uint32_t seq;
  if (threadIdx.x == 0) {
    uint32_t s = *a.step_word;
    if (a.bump) {
      s += 1u;
      *a.step_word = s;
    }
    seq = s;
  }
  // rows of 16-byte words (row_bytes, strides and offsets are multiples of 16)
  const long long wpr = a.row_bytes / 16, total = a.rows * wpr;
  for (int g = 0; g < a.G; ++g) {
    uint8_t* base = a.dst[g] + a.dst_offset + a.dst_col;
    for (long long i = threadIdx.x; i < total; i += blockDim.x) {
      const long long r = i / wpr, w = i % wpr;
      const uint4 v = *reinterpret_cast<const uint4*>(a.src + r * a.src_stride + w * 16);
      *reinterpret_cast<uint4*>(base + r * a.dst_stride + w * 16) = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the rows above, on every GPU, before any flag
    for (int g = 0; g < a.G; ++g) {
      uint32_t* f = reinterpret_cast<uint32_t*>(a.dst[g]) + a.kind * kMaxRanks + a.rank;
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(seq) : "memory");
    }
  }
}

__global__ void peer_wait_kernel(const uint32_t* ctrl, int G, int kind, int* err) {
  if (threadIdx.x != 0) return;
  const uint32_t seq = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(ctrl) + kStepWordOffset);
  for (int g = 0; g < G; ++g) {
    if (!flag_wait(ctrl + kind * kMaxRanks + g, seq, err)) return;
  }
}

}  // namespace cpx
}  // namespace aether

using namespace aether;

extern "C" long long aether_cp_control_bytes(void) { return 256; }

extern "C" int aether_cp_buffer_create(long long bytes, void** ptr, void* ipc_handle) {
  AETHER_REQUIRE(bytes >= 256 && ptr && ipc_handle, "cp buffer: bad arguments");
  void* p = nullptr;
  AETHER_CUDA_TRY(cudaMalloc(&p, static_cast<size_t>(bytes)), "cp buffer: cudaMalloc");
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    set_last_error("cp buffer: %s", cudaGetErrorString(e));
    return 2;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return 0;
}

extern "C" int aether_cp_buffer_open(const void* ipc_handle, void** ptr) {
  AETHER_REQUIRE(ipc_handle && ptr, "cp buffer open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  AETHER_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cp buffer open");
  *ptr = p;
  return 0;
}

extern "C" int aether_cp_buffer_close(void* ptr) {
  AETHER_CUDA_TRY(cudaIpcCloseMemHandle(ptr), "cp buffer close");
  return 0;
}

extern "C" int aether_cp_buffer_destroy(void* ptr) {
  AETHER_CUDA_TRY(cudaFree(ptr), "cp buffer destroy");
  return 0;
}

extern "C" int aether_peer_push(const void* src, long long rows, long long row_bytes, long long src_stride,
                                void* const* bases, int G, int rank, long long dst_offset, long long dst_stride,
                                long long dst_col, int kind, int bump, void* stream) {
  AETHER_REQUIRE(G >= 1 && G <= cpx::kMaxRanks && rank >= 0 && rank < G, "peer push: bad rank / world size");
  AETHER_REQUIRE(kind >= 0 && kind < cpx::kMaxKinds, "peer push: bad kind");
  AETHER_REQUIRE(rows >= 0 && row_bytes >= 0 && row_bytes % 16 == 0 && src_stride % 16 == 0 && dst_stride % 16 == 0 &&
                     dst_offset % 16 == 0 && dst_col % 16 == 0 && dst_offset >= 256,
                 "peer push: sizes, strides and offsets must be multiples of 16 bytes, past the control area");
  AETHER_REQUIRE(src && bases, "peer push: null argument");
  AETHER_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0, "peer push: src must be 16-byte aligned");
  cpx::PushArgs a{};
  a.src = static_cast<const uint8_t*>(src);
  a.rows = rows;
  a.row_bytes = row_bytes;
  a.src_stride = src_stride;
  a.dst_offset = dst_offset;
  a.dst_stride = dst_stride;
  a.dst_col = dst_col;
  for (int g = 0; g < G; ++g) {
    AETHER_REQUIRE(bases[g] != nullptr, "peer push: missing buffer of rank %d", g);
    a.dst[g] = static_cast<uint8_t*>(bases[g]);
  }
  a.G = G;
  a.rank = rank;
  a.kind = kind;
  a.bump = bump;
  a.step_word = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(bases[rank]) + cpx::kStepWordOffset);
  cpx::peer_push_kernel<<<1, cpx::kPushThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("peer_push");
}

extern "C" int aether_peer_wait(const void* local_base, int G, int kind, int* err, void* stream) {
  AETHER_REQUIRE(local_base && G >= 1 && G <= cpx::kMaxRanks && kind >= 0 && kind < cpx::kMaxKinds,
                 "peer wait: bad arguments");
  cpx::peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint32_t*>(local_base),
                                                                         G, kind, err);
  return check_launch("peer_wait");
}
