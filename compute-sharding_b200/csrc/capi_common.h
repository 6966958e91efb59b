// capi_common.h — error plumbing shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <string>

#include "../../include/stagefwd.h"

namespace sfc {

void set_error(const char *fmt, ...);
void clear_error();

// Record a CUDA failure and map it to SFC_E_CUDA.
inline int cuda_fail(cudaError_t e, const char *what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return SFC_E_CUDA;
}

}  // namespace sfc

#define SFC_CUDA(call)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return ::sfc::cuda_fail(e_, #call); \
  } while (0)

#define SFC_REQUIRE(cond, ...)                           \
  do {                                                   \
    if (!(cond)) {                                       \
      ::sfc::set_error(__VA_ARGS__);                     \
      return SFC_E_INVALID;                              \
    }                                                    \
  } while (0)
