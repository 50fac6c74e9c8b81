// Shared host-side helpers: thread-local error reporting and status macros.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/woolly_cuda.h"

namespace wl {

void set_error(const std::string& msg);
// programmatic dependent launch for the kernels the calling thread enqueues
void set_pdl(bool on);
// true exactly once per (current device, key) across all host threads: guards
// per-device one-time set-up such as kernel attributes
bool first_use_on_device(const void* key);
inline int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

inline size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

}  // namespace wl

#define WL_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return wl::fail(e_ == cudaErrorMemoryAllocation ? WL_ERR_OUT_OF_MEMORY : WL_ERR_CUDA, \
                      std::string(#expr) + ": " + cudaGetErrorString(e_));             \
  } while (0)

#define WL_TRY(expr)       \
  do {                     \
    int s_ = (expr);       \
    if (s_ != WL_OK) return s_; \
  } while (0)

#define WL_CHECK_ARG(cond, msg) \
  do {                          \
    if (!(cond)) return wl::fail(WL_ERR_INVALID_ARGUMENT, msg); \
  } while (0)
