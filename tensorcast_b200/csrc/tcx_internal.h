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

// Counts kernel launches of this library (tcx_kernel_launch_count).
void note_launches(uint64_t n);

// Kernel launchers shared between translation units (stream-ordered).
// max_ctas: cap on the persistent grid (0: 8 CTAs per SM), for copies that run
// beside other kernels.
tcx_status launch_copy_jobs(const void* d_src, void* d_dst, const tcx_copy_job* d_jobs, uint64_t n_jobs,
                            uint64_t* d_prefix, cudaStream_t stream, uint32_t max_ctas = 0);
int sm_count();
tcx_status launch_permute(const void* d_src, void* d_dst, const tcx_permute_job& pj, cudaStream_t stream);
tcx_status check_permute(const tcx_permute_job& pj);
tcx_status launch_leaf_pass(const void* d_src, uint64_t total, uint64_t leaf, uint32_t n, uint64_t seg_off,
                            uint64_t seg_len, uint32_t* states, void* d_digests, cudaStream_t stream);
// A pass over a slab buffer: bytes [seg_off, seg_off + seg_len) of leaf i (of
// the leaves [0, n) of a stream of `total` bytes cut at `leaf`) are at
// d_src + i * pitch.
tcx_status launch_leaf_pass_pitched(const void* d_src, uint64_t pitch, uint64_t total, uint64_t leaf, uint32_t n,
                                    uint64_t seg_off, uint64_t seg_len, uint32_t* states, void* d_digests,
                                    cudaStream_t stream);
tcx_status launch_merkle(const uint8_t* digests, uint64_t n, uint8_t* scratch, uint8_t* root, cudaStream_t stream);
uint64_t merkle_scratch_bytes(uint64_t n);
tcx_status preload_hash_kernels();
void encode_multihash(const uint8_t digest[32], char out[57]);

inline std::string cuda_msg(cudaError_t e) {
  return std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
}

}  // namespace tcx

// Returns TCX_INTERNAL with a message naming the failing call. The runtime's
// per-thread last error is reset (it is reported here), so that a later launch
// check on this thread does not pick up an error of this call, such as a failed
// allocation.
#define TCX_CUDA_TRY(call)                                                                         \
  do {                                                                                             \
    cudaError_t tcx_e_ = (call);                                                                   \
    if (tcx_e_ != cudaSuccess) {                                                                   \
      cudaGetLastError();                                                                          \
      return ::tcx::set_error(TCX_INTERNAL, std::string(#call " failed: ") + ::tcx::cuda_msg(tcx_e_)); \
    }                                                                                              \
  } while (0)
