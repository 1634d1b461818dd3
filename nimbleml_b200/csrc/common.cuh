// common.cuh — error reporting shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "nimbleml_tied_ce.h"

namespace nimble {

// Records `msg` as the calling thread's last error (returned by
// nimble_tied_ce_last_error) and returns `code`.
int fail(int code, const std::string& msg);

inline int elem_size(int dtype) { return (dtype == NIMBLE_DTYPE_F32 || dtype == NIMBLE_DTYPE_TF32) ? 4 : 2; }

inline bool valid_dtype(int dtype) {
  return dtype == NIMBLE_DTYPE_F32 || dtype == NIMBLE_DTYPE_F16 || dtype == NIMBLE_DTYPE_BF16;
}

}  // namespace nimble

#define NIMBLE_CUDA_TRY(expr)                                                                    \
  do {                                                                                           \
    cudaError_t e_ = (expr);                                                                     \
    if (e_ != cudaSuccess)                                                                       \
      return ::nimble::fail(NIMBLE_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)
