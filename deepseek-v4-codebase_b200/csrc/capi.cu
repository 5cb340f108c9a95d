// Library-level C-ABI entry points: version, last error message, build info.
#include <string.h>

#include <map>
#include <mutex>
#include <utility>

#include "aether_b200.h"
#include "capi_util.cuh"

namespace aether {

static thread_local char g_last_error[1024] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return 2;
  }
  return 0;
}

int ensure_smem_attr(const void* fn, int bytes, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error("%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
    return 2;
  }
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes set
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(fn, dev);
  const auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return 0;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_last_error("%s: set shared memory size: %s", what, cudaGetErrorString(e));
    return 2;
  }
  done[key] = bytes;
  return 0;
}

}  // namespace aether

extern "C" {

const char* aether_last_error(void) { return aether::g_last_error; }

int aether_abi_version(void) { return 1; }

// Compute capability the kernels were compiled for (major*10+minor).
int aether_compiled_arch(void) { return 100; }

}
