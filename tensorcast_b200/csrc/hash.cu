// Content hashing on sm_100a: per-leaf SHA-256, the Merkle reduction and the
// data-multihash entry point of the C ABI.
//
// Reference behaviour followed (core/common/artifact_hash_gpu.cc, artifact_hash_cpu.cc):
//   * leaves [i*L, min((i+1)*L, T)), 32-byte big-endian digests (kernel :384-411);
//   * pairwise Merkle tree, odd node promoted unchanged (:198-233 of the CPU file);
//   * argument checks and messages of compute_data_multihash_from_gpu (:903-957);
//   * leaf policy determine_leaf_chunk_size (artifact_hash_cpu.cc:269-303).
//
// Kernel design. SHA-256 is serial inside a leaf, so the unit of parallelism is
// the leaf: one thread owns one leaf's chain and keeps the state, the 16-word
// message window and the next block (prefetched one block ahead) in registers.
// Loads are 16-byte non-allocating vector loads; no shared memory is used.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "sha256_device.cuh"
#include "tcx_internal.h"

namespace tcx {
namespace {

constexpr int kLeafThreads = 64;       // threads (= leaves) per CTA of the leaf kernel
constexpr int kMerkleThreads = 256;    // threads per CTA of a Merkle level
constexpr uint32_t kFinishMax = 2048;  // levels at or below this size finish in one CTA
constexpr int kFinishThreads = 1024;

// ---------------------------------------------------------------------------
// Leaf kernel.
// kVec: every leaf start is 16-byte aligned (16-aligned base, L % 16 == 0).
// Otherwise each leaf start has a fixed misalignment s = addr & 3 and a block is
// assembled from 17 aligned words with funnel shifts. Every word read lies in the
// same aligned 4-byte word as at least one byte of the leaf, so no read can leave
// the pages of the buffer.
// ---------------------------------------------------------------------------
template <bool kVec>
__global__ void __launch_bounds__(kLeafThreads) sha256_leaf_kernel(const uint8_t* __restrict__ src, uint64_t total,
                                                                   uint64_t leaf, uint32_t n_leaves,
                                                                   uint8_t* __restrict__ digests) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_leaves) return;
  const uint64_t off = static_cast<uint64_t>(i) * leaf;
  const uint64_t len = min(leaf, total - off);
  const uint8_t* p = src + off;
  const uint64_t nfull = len >> 6;

  uint32_t s[8];
  dev::init_state(s);
  uint32_t w[16];

  if constexpr (kVec) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    uint4 v0, v1, v2, v3;
    if (nfull > 0) {
      v0 = dev::ldg_stream(q + 0);
      v1 = dev::ldg_stream(q + 1);
      v2 = dev::ldg_stream(q + 2);
      v3 = dev::ldg_stream(q + 3);
    }
    for (uint64_t b = 0; b < nfull; ++b) {
      dev::words_from_vec(w, v0, v1, v2, v3);
      if (b + 1 < nfull) {
        const uint4* nq = q + 4 * (b + 1);
        v0 = dev::ldg_stream(nq + 0);
        v1 = dev::ldg_stream(nq + 1);
        v2 = dev::ldg_stream(nq + 2);
        v3 = dev::ldg_stream(nq + 3);
      }
      dev::compress(s, w);
    }
  } else {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(p);
    const uint32_t shift = static_cast<uint32_t>(addr & 3u) * 8u;
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(addr & ~static_cast<uintptr_t>(3));
    for (uint64_t b = 0; b < nfull; ++b) {
      const uint32_t* bw = wp + 16 * b;
      uint32_t lo = __ldg(bw);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        // The 17th word is only needed (and only read) when the block is misaligned.
        const uint32_t hi = (shift != 0 || k < 15) ? __ldg(bw + k + 1) : 0u;
        w[k] = dev::bswap32(shift ? __funnelshift_r(lo, hi, shift) : lo);
        lo = hi;
      }
      dev::compress(s, w);
    }
  }
  dev::finish(s, p + (nfull << 6), static_cast<uint32_t>(len & 63u), len);
  dev::store_digest(digests + 32ull * i, s);
}

// ---------------------------------------------------------------------------
// Merkle reduction. node = SHA-256(left || right): one data block plus the
// constant padding block of a 64-byte message.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void hash_pair(const uint8_t* pair64, uint8_t* out32) {
  const uint4* q = reinterpret_cast<const uint4*>(pair64);
  uint32_t s[8], w[16];
  dev::init_state(s);
  dev::words_from_vec(w, q[0], q[1], q[2], q[3]);
  dev::compress(s, w);
#pragma unroll
  for (int k = 0; k < 16; ++k) w[k] = 0;
  w[0] = 0x80000000u;
  w[15] = 512u;
  dev::compress(s, w);
  dev::store_digest(out32, s);
}

// One level: dst[j] = H(src[2j] || src[2j+1]); an odd last node is copied.
__global__ void __launch_bounds__(kMerkleThreads) merkle_level_kernel(const uint8_t* __restrict__ src, uint32_t m,
                                                                      uint8_t* __restrict__ dst) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t pairs = m / 2;
  if (j < pairs) {
    hash_pair(src + 64ull * j, dst + 32ull * j);
  } else if (j == pairs && (m & 1u)) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src + 32ull * (m - 1));
    uint4* d4 = reinterpret_cast<uint4*>(dst + 32ull * j);
    d4[0] = s4[0];
    d4[1] = s4[1];
  }
}

// Remaining levels (m <= kFinishMax) inside one CTA, in shared memory; writes the root.
__global__ void __launch_bounds__(kFinishThreads) merkle_finish_kernel(const uint8_t* __restrict__ src, uint32_t m,
                                                                       uint8_t* __restrict__ root) {
  extern __shared__ uint4 smem4[];
  uint8_t* nodes = reinterpret_cast<uint8_t*>(smem4);
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  for (uint32_t k = threadIdx.x; k < 2 * m; k += blockDim.x) smem4[k] = s4[k];
  __syncthreads();
  while (m > 1) {
    const uint32_t pairs = m / 2;
    const uint32_t j = threadIdx.x;  // pairs <= kFinishMax / 2 == blockDim.x
    uint32_t s[8];
    uint4 keep0 = make_uint4(0, 0, 0, 0), keep1 = keep0;
    if (j < pairs) {
      const uint4* q = reinterpret_cast<const uint4*>(nodes + 64u * j);
      uint32_t w[16];
      dev::init_state(s);
      dev::words_from_vec(w, q[0], q[1], q[2], q[3]);
      dev::compress(s, w);
#pragma unroll
      for (int k = 0; k < 16; ++k) w[k] = 0;
      w[0] = 0x80000000u;
      w[15] = 512u;
      dev::compress(s, w);
    } else if (j == pairs && (m & 1u)) {
      keep0 = smem4[2 * (m - 1)];
      keep1 = smem4[2 * (m - 1) + 1];
    }
    __syncthreads();  // every read of this level precedes every write
    if (j < pairs) {
      dev::store_digest(nodes + 32u * j, s);
    } else if (j == pairs && (m & 1u)) {
      smem4[2 * j] = keep0;
      smem4[2 * j + 1] = keep1;
    }
    __syncthreads();
    m = pairs + (m & 1u);
  }
  if (threadIdx.x < 2) reinterpret_cast<uint4*>(root)[threadIdx.x] = smem4[threadIdx.x];
}

// ---------------------------------------------------------------------------
// Host helpers.
// ---------------------------------------------------------------------------
uint64_t div_up(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

uint64_t leaf_policy(uint64_t total, uint64_t requested) {
  uint64_t bounded = requested == 0 ? TCX_DEFAULT_LEAF_BYTES : requested;
  bounded = std::min<uint64_t>(bounded, TCX_MAX_LEAF_BYTES);
  bounded = std::max<uint64_t>(bounded, 64);
  bounded -= bounded % 64;
  if (bounded == 0) bounded = 64;
  if (requested != TCX_DEFAULT_LEAF_BYTES) return bounded;
  uint64_t adjusted = bounded;
  while (adjusted > TCX_MIN_ADAPTIVE_LEAF_BYTES && div_up(total, adjusted) < TCX_TARGET_LEAF_COUNT) {
    uint64_t candidate = adjusted / 2;
    candidate -= candidate % 64;
    if (candidate < TCX_MIN_ADAPTIVE_LEAF_BYTES) break;
    adjusted = candidate;
  }
  if (adjusted < TCX_MIN_ADAPTIVE_LEAF_BYTES) adjusted = TCX_MIN_ADAPTIVE_LEAF_BYTES;
  return adjusted == 0 ? 64 : adjusted;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

tcx_status launch_leaves(const void* d_src, uint64_t total, uint64_t leaf, uint32_t n, void* d_digests,
                         cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(div_up(n, kLeafThreads)));
  const auto* src = static_cast<const uint8_t*>(d_src);
  auto* out = static_cast<uint8_t*>(d_digests);
  if (aligned16(d_src) && leaf % 16 == 0) {
    sha256_leaf_kernel<true><<<grid, kLeafThreads, 0, stream>>>(src, total, leaf, n, out);
  } else {
    sha256_leaf_kernel<false><<<grid, kLeafThreads, 0, stream>>>(src, total, leaf, n, out);
  }
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

uint64_t merkle_scratch_bytes(uint64_t n) {
  // Two ping-pong level buffers; the largest levels are ceil(n/2) and ceil(n/4) nodes.
  const uint64_t a = div_up(n, 2), b = div_up(n, 4);
  return ((a + b + 2) * 32 + 255) & ~255ull;
}

tcx_status launch_merkle(const uint8_t* digests, uint64_t n, uint8_t* scratch, uint8_t* root, cudaStream_t stream) {
  const uint64_t a_nodes = div_up(n, 2);
  uint8_t* buf[2] = {scratch, scratch + ((a_nodes * 32 + 255) & ~255ull)};
  const uint8_t* cur = digests;
  uint64_t m = n;
  int which = 0;
  while (m > kFinishMax) {
    const uint64_t next = div_up(m, 2);
    const unsigned grid = static_cast<unsigned>(div_up(next, kMerkleThreads));
    merkle_level_kernel<<<grid, kMerkleThreads, 0, stream>>>(cur, static_cast<uint32_t>(m), buf[which]);
    TCX_CUDA_TRY(cudaGetLastError());
    cur = buf[which];
    which ^= 1;
    m = next;
  }
  const size_t smem = static_cast<size_t>(m) * 32;
  if (smem > 48 * 1024) {
    // The attribute is per device; setting it is a cheap host-side call.
    TCX_CUDA_TRY(cudaFuncSetAttribute(merkle_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kFinishMax * 32)));
  }
  merkle_finish_kernel<<<1, kFinishThreads, smem, stream>>>(cur, static_cast<uint32_t>(m), root);
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

void encode_multihash(const uint8_t digest[32], char out[57]) {
  static const char kAlphabet[] = "abcdefghijklmnopqrstuvwxyz234567";
  uint8_t mh[34];
  mh[0] = 0x12;
  mh[1] = 0x20;
  std::memcpy(mh + 2, digest, 32);
  char tmp[64];
  size_t pos = 0;
  for (size_t i = 0; i < sizeof mh;) {
    const size_t take = std::min<size_t>(5, sizeof mh - i);
    uint64_t acc = 0;
    for (size_t j = 0; j < take; ++j) acc = (acc << 8) | mh[i + j];
    acc <<= (5 - take) * 8;
    for (int sh = 35; sh >= 0; sh -= 5) tmp[pos++] = kAlphabet[(acc >> sh) & 31u];
    i += take;
  }
  out[0] = 'b';
  std::memcpy(out + 1, tmp, 55);  // ceil(34 * 8 / 5) = 55 significant characters
  out[56] = '\0';
}

// Per-device resources of tcx_multihash_from_gpu, created once and grown on demand.
struct DeviceHashContext {
  std::mutex mu;
  bool ready = false;
  cudaStream_t stream = nullptr;
  uint8_t* digests = nullptr;
  uint64_t digests_cap = 0;
  uint8_t* scratch = nullptr;
  uint64_t scratch_cap = 0;
  uint8_t* d_root = nullptr;
  uint8_t* h_root = nullptr;  // pinned
};

constexpr int kMaxDevices = 64;
DeviceHashContext g_ctx[kMaxDevices];

// Caller holds ctx.mu and has made the device current.
tcx_status ensure_context(DeviceHashContext& ctx, uint64_t n_leaves) {
  if (!ctx.ready) {
    TCX_CUDA_TRY(cudaStreamCreateWithFlags(&ctx.stream, cudaStreamNonBlocking));
    TCX_CUDA_TRY(cudaMalloc(&ctx.d_root, 256));
    TCX_CUDA_TRY(cudaMallocHost(&ctx.h_root, 256));
    cudaFuncAttributes attr;
    TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_kernel<true>));
    TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_kernel<false>));
    TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, merkle_level_kernel));
    ctx.ready = true;
  }
  const uint64_t need_d = std::max<uint64_t>(n_leaves, 1) * 32;
  if (need_d > ctx.digests_cap) {
    if (ctx.digests) TCX_CUDA_TRY(cudaFree(ctx.digests));
    ctx.digests = nullptr;
    ctx.digests_cap = 0;
    const uint64_t cap = std::max<uint64_t>(need_d, 4096 * 32);
    TCX_CUDA_TRY(cudaMalloc(&ctx.digests, cap));
    ctx.digests_cap = cap;
  }
  const uint64_t need_s = merkle_scratch_bytes(n_leaves);
  if (need_s > ctx.scratch_cap) {
    if (ctx.scratch) TCX_CUDA_TRY(cudaFree(ctx.scratch));
    ctx.scratch = nullptr;
    ctx.scratch_cap = 0;
    const uint64_t cap = std::max<uint64_t>(need_s, merkle_scratch_bytes(4096));
    TCX_CUDA_TRY(cudaMalloc(&ctx.scratch, cap));
    ctx.scratch_cap = cap;
  }
  return TCX_OK;
}

tcx_status fallback_disabled(tcx_status st) {
  if (st == TCX_OK) return st;
  const std::string msg = tcx_last_error();
  return set_error(st, "GPU hashing unavailable; CPU fallback disabled: " + msg);
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" tcx_status tcx_leaf_policy(uint64_t total_bytes, uint64_t requested_leaf_bytes, uint64_t* leaf_bytes_out) {
  if (leaf_bytes_out == nullptr) return set_error(TCX_INVALID_ARGUMENT, "leaf_bytes_out is null");
  *leaf_bytes_out = leaf_policy(total_bytes, requested_leaf_bytes);
  return TCX_OK;
}

extern "C" tcx_status tcx_sha256_leaves(const void* d_src, uint64_t total_bytes, uint64_t leaf_bytes,
                                        void* d_digests, uint64_t digest_capacity, void* stream) {
  if (d_src == nullptr) return set_error(TCX_INVALID_ARGUMENT, "GPU pointer is null");
  if (total_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "Cannot hash empty GPU buffer");
  if (total_bytes > TCX_MAX_HASH_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "GPU buffer too large for hashing: %llu bytes",
                      static_cast<unsigned long long>(total_bytes));
  if (leaf_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "leaf_chunk_bytes must be > 0");
  if (leaf_bytes > TCX_MAX_LEAF_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "Chunk size too large: %llu (max: %llu)",
                      static_cast<unsigned long long>(leaf_bytes), static_cast<unsigned long long>(TCX_MAX_LEAF_BYTES));
  const uint64_t n = div_up(total_bytes, leaf_bytes);
  if (n > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");
  if (d_digests == nullptr) return set_error(TCX_INVALID_ARGUMENT, "digest buffer is null");
  if (!aligned16(d_digests)) return set_error(TCX_INVALID_ARGUMENT, "digest buffer must be 16-byte aligned");
  if (digest_capacity < n)
    return set_errorf(TCX_INVALID_ARGUMENT, "digest buffer holds %llu digests, %llu needed",
                      static_cast<unsigned long long>(digest_capacity), static_cast<unsigned long long>(n));
  return launch_leaves(d_src, total_bytes, leaf_bytes, static_cast<uint32_t>(n), d_digests,
                       static_cast<cudaStream_t>(stream));
}

extern "C" uint64_t tcx_merkle_scratch_bytes(uint64_t n_leaves) { return merkle_scratch_bytes(n_leaves); }

extern "C" tcx_status tcx_merkle_root(const void* d_digests, uint64_t n_leaves, void* d_scratch, uint64_t scratch_bytes,
                                      void* d_root, void* stream) {
  if (d_digests == nullptr || d_root == nullptr) return set_error(TCX_INVALID_ARGUMENT, "null device pointer");
  if (n_leaves == 0) return set_error(TCX_INVALID_ARGUMENT, "Leaf digests must not be empty");
  if (n_leaves > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");
  if (!aligned16(d_digests) || !aligned16(d_root)) return set_error(TCX_INVALID_ARGUMENT, "digests and root must be 16-byte aligned");
  if (n_leaves > kFinishMax) {
    if (d_scratch == nullptr || !aligned16(d_scratch) || scratch_bytes < merkle_scratch_bytes(n_leaves))
      return set_errorf(TCX_INVALID_ARGUMENT, "Merkle scratch must be 16-byte aligned and hold %llu bytes",
                        static_cast<unsigned long long>(merkle_scratch_bytes(n_leaves)));
  }
  return launch_merkle(static_cast<const uint8_t*>(d_digests), n_leaves, static_cast<uint8_t*>(d_scratch),
                       static_cast<uint8_t*>(d_root), static_cast<cudaStream_t>(stream));
}

extern "C" tcx_status tcx_multihash_encode(const uint8_t* digest32, char* out, size_t out_capacity) {
  if (digest32 == nullptr || out == nullptr) return set_error(TCX_INVALID_ARGUMENT, "null pointer");
  if (out_capacity < TCX_MULTIHASH_CHARS + 1) return set_error(TCX_INVALID_ARGUMENT, "output buffer needs 57 bytes");
  encode_multihash(digest32, out);
  return TCX_OK;
}

extern "C" tcx_status tcx_multihash_from_gpu(const void* d_src, uint64_t total_bytes, int device_id,
                                             uint64_t leaf_chunk_bytes, char* out, size_t out_capacity) {
  // Argument checks in the order of artifact_hash_gpu.cc:907-927.
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
  if (device_id < 0 || device_id >= kMaxDevices)
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: invalid device ordinal", device_id);
  if (cudaError_t e = cudaSetDevice(device_id); e != cudaSuccess)
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: %s", device_id, cuda_msg(e).c_str());

  const uint64_t leaf = leaf_policy(total_bytes, leaf_chunk_bytes);
  const uint64_t n = div_up(total_bytes, leaf);
  if (n > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");

  DeviceHashContext& ctx = g_ctx[device_id];
  std::lock_guard<std::mutex> lock(ctx.mu);
  tcx_status st = ensure_context(ctx, n);
  if (st == TCX_OK) st = launch_leaves(d_src, total_bytes, leaf, static_cast<uint32_t>(n), ctx.digests, ctx.stream);
  if (st == TCX_OK) st = launch_merkle(ctx.digests, n, ctx.scratch, ctx.d_root, ctx.stream);
  if (st == TCX_OK) {
    cudaError_t e = cudaMemcpyAsync(ctx.h_root, ctx.d_root, 32, cudaMemcpyDeviceToHost, ctx.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx.stream);
    if (e != cudaSuccess) st = set_error(TCX_INTERNAL, "digest readback failed: " + cuda_msg(e));
  }
  if (st != TCX_OK) return fallback_disabled(st);
  encode_multihash(ctx.h_root, out);
  return TCX_OK;
}

extern "C" tcx_status tcx_prewarm_device(int device_id) {
  if (device_id < 0) return set_error(TCX_INVALID_ARGUMENT, "device_id must be >= 0");
  int count = 0;
  TCX_CUDA_TRY(cudaGetDeviceCount(&count));
  if (device_id >= count || device_id >= kMaxDevices)
    return set_errorf(TCX_INVALID_ARGUMENT, "device_id %d out of range for visible GPU count %d", device_id, count);
  int prior = -1;
  const bool have_prior = cudaGetDevice(&prior) == cudaSuccess;
  tcx_status st = TCX_OK;
  if (cudaError_t e = cudaSetDevice(device_id); e != cudaSuccess) {
    st = set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: %s", device_id, cuda_msg(e).c_str());
  } else {
    DeviceHashContext& ctx = g_ctx[device_id];
    std::lock_guard<std::mutex> lock(ctx.mu);
    st = ensure_context(ctx, TCX_TARGET_LEAF_COUNT);
  }
  if (have_prior && prior != device_id) cudaSetDevice(prior);
  return st;
}

extern "C" tcx_status tcx_prewarm_visible_devices(void) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return TCX_OK;
  if (e != cudaSuccess) return set_error(TCX_INTERNAL, "cudaGetDeviceCount failed: " + cuda_msg(e));
  for (int d = 0; d < count; ++d) {
    tcx_status st = tcx_prewarm_device(d);
    if (st != TCX_OK) {
      const std::string msg = tcx_last_error();
      return set_errorf(st, "GPU hash prewarm failed for device %d: %s", d, msg.c_str());
    }
  }
  return TCX_OK;
}
