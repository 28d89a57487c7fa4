// Internal helpers shared by the libtcx translation units: status/error plumbing
// and CUDA error checks. Not part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/tcx.h"

namespace tcx {

// Records msg as this thread's last error and returns code (TCX_OK clears nothing).
tcx_status set_error(tcx_status code, const std::string& msg);
tcx_status set_errorf(tcx_status code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

inline std::string cuda_msg(cudaError_t e) {
  return std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
}

}  // namespace tcx

// Returns TCX_INTERNAL with a message naming the failing call.
#define TCX_CUDA_TRY(call)                                                                         \
  do {                                                                                             \
    cudaError_t tcx_e_ = (call);                                                                   \
    if (tcx_e_ != cudaSuccess) {                                                                   \
      return ::tcx::set_error(TCX_INTERNAL, std::string(#call " failed: ") + ::tcx::cuda_msg(tcx_e_)); \
    }                                                                                              \
  } while (0)
