// tcx_multihash_from_gpu_noalloc: the data multihash of a device buffer without
// any device or pinned allocation.
//
// Why it exists: some callers cannot call cudaMalloc at the moment they need a
// content hash. An inference or serving engine that has already reserved
// nearly all device memory for its own pool would see a new allocation fail or
// fragment that pool, and a latency-sensitive path cannot afford cudaFree,
// which waits for all work already queued on the device. This entry point
// needs nothing from the caller but the input, the output string and a stream.
//
// Its scratch (leaf digests, Merkle levels, the root) lives in the file-scope
// device array below, of a fixed size, so the number of leaves per call is
// capped at kNoAllocMaxLeaves. Every GPU that loads this library holds that
// array until the process exits.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "tcx_internal.h"

namespace tcx {
namespace {

// Most leaves one call may hash: 16384 leaves cover 64 GiB at 4 MiB leaves and
// 1 TiB (the hashing limit) at the 64 MiB maximum leaf size.
constexpr uint64_t kNoAllocMaxLeaves = 16384;
constexpr uint64_t kDigestBytes = kNoAllocMaxLeaves * 32;
// Two ping-pong Merkle level buffers of ceil(n/2) and ceil(n/4) nodes, each
// rounded up to 256 bytes (the layout launch_merkle uses), plus slack.
constexpr uint64_t kMerkleBytes = ((kNoAllocMaxLeaves / 2 + kNoAllocMaxLeaves / 4 + 2) * 32 + 255) / 256 * 256 + 256;
constexpr uint64_t kRootOffset = kDigestBytes + kMerkleBytes;
constexpr uint64_t kScratchBytes = kRootOffset + 256;

// The scratch. In host code this name is only a host-side stand-in for the
// device symbol, never a device address: the device address comes from
// cudaGetSymbolAddress, once per device, below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

// Puts the calling thread's current device back when the call returns.
struct DeviceRestore {
  int prior = -1;
  DeviceRestore() {
    if (cudaGetDevice(&prior) != cudaSuccess) {
      cudaGetLastError();
      prior = -1;
    }
  }
  ~DeviceRestore() {
    if (prior >= 0) cudaSetDevice(prior);
  }
};

struct NoAllocDevice {
  std::mutex mu;     // serialises calls on one device (the scratch is shared)
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
};
constexpr int kMaxDevices = 64;
NoAllocDevice g_devices[kMaxDevices];

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" tcx_status tcx_multihash_from_gpu_noalloc(const void* d_src, uint64_t total_bytes, int device_id,
                                                     uint64_t leaf_chunk_bytes, char* out, size_t out_capacity,
                                                     void* stream) {
  // The same argument checks, in the same order, as tcx_multihash_from_gpu.
  if (d_src == nullptr) return set_error(TCX_INVALID_ARGUMENT, "GPU pointer is null");
  if (total_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "Cannot hash empty GPU buffer");
  if (total_bytes > TCX_MAX_HASH_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "GPU buffer too large for hashing: %llu bytes",
                      static_cast<unsigned long long>(total_bytes));
  if (leaf_chunk_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "leaf_chunk_bytes must be > 0");
  if (leaf_chunk_bytes > TCX_MAX_LEAF_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "Chunk size too large: %llu (max: %llu)",
                      static_cast<unsigned long long>(leaf_chunk_bytes),
                      static_cast<unsigned long long>(TCX_MAX_LEAF_BYTES));
  if (out == nullptr || out_capacity < TCX_MULTIHASH_CHARS + 1)
    return set_error(TCX_INVALID_ARGUMENT, "output buffer needs 57 bytes");
  uint64_t leaf = 0;
  tcx_status st = tcx_leaf_policy(total_bytes, leaf_chunk_bytes, &leaf);
  if (st != TCX_OK) return st;
  const uint64_t n = (total_bytes + leaf - 1) / leaf;
  if (n > kNoAllocMaxLeaves)
    return set_errorf(TCX_INVALID_ARGUMENT,
                      "%llu leaves of %llu bytes exceed the no-alloc scratch capacity of %llu leaves "
                      "(use a larger leaf_chunk_bytes or tcx_multihash_from_gpu)",
                      static_cast<unsigned long long>(n), static_cast<unsigned long long>(leaf),
                      static_cast<unsigned long long>(kNoAllocMaxLeaves));
  if (device_id < 0 || device_id >= kMaxDevices)
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: invalid device ordinal", device_id);
  // The caller's current device is restored on every return: this entry point
  // serves engines that drive devices from their own threads.
  DeviceRestore restore;
  if (cudaError_t e = cudaSetDevice(device_id); e != cudaSuccess) {
    cudaGetLastError();
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: %s", device_id, cuda_msg(e).c_str());
  }
  const auto s = static_cast<cudaStream_t>(stream);
  if (s != nullptr) {
    int stream_dev = -1;
    if (cudaError_t e = cudaStreamGetDevice(s, &stream_dev); e != cudaSuccess) {
      cudaGetLastError();
      return set_errorf(TCX_INVALID_ARGUMENT, "cannot query the stream's device: %s", cuda_msg(e).c_str());
    }
    if (stream_dev != device_id)
      return set_errorf(TCX_INVALID_ARGUMENT, "stream belongs to device %d, not to device_id %d", stream_dev,
                        device_id);
  }
  NoAllocDevice& dev = g_devices[device_id];
  std::lock_guard<std::mutex> lock(dev.mu);
  if (dev.scratch == nullptr) {
    // Set-up, once per device, with that device current: the device address of
    // the scratch array. It is done by the first call on each device.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(TCX_INTERNAL, "GPU hashing unavailable; CPU fallback disabled: cudaGetSymbolAddress failed: " +
                                         cuda_msg(e));
    // Every kernel this entry point may launch is loaded now, so that no later
    // call, whatever its shape, needs device memory for a module load.
    if (tcx_status pst = preload_hash_kernels(); pst != TCX_OK) {
      const std::string msg = tcx_last_error();
      return set_error(pst, "GPU hashing unavailable; CPU fallback disabled: " + msg);
    }
    dev.scratch = static_cast<uint8_t*>(p);
  }
  // Nothing in the scratch has to start at zero: the leaf kernel writes every
  // digest and each Merkle level writes every node before the next level reads it.
  uint8_t* digests = dev.scratch;
  uint8_t* merkle = dev.scratch + kDigestBytes;
  uint8_t* d_root = dev.scratch + kRootOffset;
  st = launch_leaf_pass(d_src, total_bytes, leaf, static_cast<uint32_t>(n), 0, ~0ull, nullptr, digests, s);
  if (st == TCX_OK) st = launch_merkle(digests, n, merkle, d_root, s);
  uint8_t root[32];
  if (st == TCX_OK) {
    // Device to pageable host memory: returns once the 32 bytes have arrived.
    cudaError_t e = cudaMemcpyAsync(root, d_root, sizeof root, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = set_error(TCX_INTERNAL, "digest readback failed: " + cuda_msg(e));
  }
  if (st != TCX_OK) {
    const std::string msg = tcx_last_error();
    return set_error(st, "GPU hashing unavailable; CPU fallback disabled: " + msg);
  }
  encode_multihash(root, out);
  return TCX_OK;
}
