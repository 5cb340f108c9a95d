// Host-side helpers shared by the C-ABI entry points: thread-local error
// message, argument checks and launch-error translation.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

namespace aether {

void set_last_error(const char* fmt, ...);

// Returns 0; used as `return ok();` at the end of an entry point after the
// launch, translating a pending launch error into status 2.
int check_launch(const char* what);

// Raises the dynamic shared-memory limit of kernel `fn` to `bytes` on the
// current device.  The attribute belongs to each device's context, so it is
// set once per (kernel, device) pair; the record is guarded by a mutex, so
// several host threads (or several devices driven by one process) are safe.
// Returns 0, or 2 with the last-error message set.
int ensure_smem_attr(const void* fn, int bytes, const char* what);

}  // namespace aether

#define AETHER_REQUIRE(cond, ...)          \
  do {                                     \
    if (!(cond)) {                         \
      ::aether::set_last_error(__VA_ARGS__); \
      return 1;                            \
    }                                      \
  } while (0)

#define AETHER_CUDA_TRY(expr, what)                                                    \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      ::aether::set_last_error("%s: %s", what, cudaGetErrorString(e_));                \
      return 2;                                                                        \
    }                                                                                  \
  } while (0)
