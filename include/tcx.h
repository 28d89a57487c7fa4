/*
 * tcx.h -- C ABI of libtcx, the B200-native realization hot path for TensorCast.
 *
 * Plain C: pointers, sizes and an int status; no torch or absl types. Every entry
 * point is thread-safe. Device pointers are caller-owned. Stream arguments are
 * cudaStream_t passed as void* (NULL = the legacy default stream); stream-ordered
 * entry points return once the work is enqueued.
 *
 * Status values use absl::StatusCode numbering, so a C++ shim maps them 1:1 onto
 * absl::Status (the reference's error type). The message of the last failing call
 * on the calling thread is available from tcx_last_error().
 */
#ifndef TCX_H_
#define TCX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int tcx_status;
#define TCX_OK 0
#define TCX_CANCELLED 1
#define TCX_UNKNOWN 2
#define TCX_INVALID_ARGUMENT 3
#define TCX_DEADLINE_EXCEEDED 4
#define TCX_NOT_FOUND 5
#define TCX_RESOURCE_EXHAUSTED 8
#define TCX_FAILED_PRECONDITION 9
#define TCX_OUT_OF_RANGE 11
#define TCX_UNIMPLEMENTED 12
#define TCX_INTERNAL 13
#define TCX_UNAVAILABLE 14
#define TCX_DATA_LOSS 15

/* Limits of the content-hashing path (core/common/artifact_hash.h:16,
 * core/common/artifact_hash_internal.h:15-17, core/common/artifact_hash_gpu.cc:908-927). */
#define TCX_DEFAULT_LEAF_BYTES (4ull << 20)
#define TCX_MAX_LEAF_BYTES (64ull << 20)
#define TCX_MIN_ADAPTIVE_LEAF_BYTES (512ull << 10)
#define TCX_TARGET_LEAF_COUNT 4096ull
#define TCX_MAX_HASH_BYTES (1ull << 40)
#define TCX_MULTIHASH_CHARS 56 /* 'b' + 55 base32 characters; buffers need 57 bytes */

/* Message of the last failing tcx_* call on this thread ("" if none). */
const char* tcx_last_error(void);

/* Library version string. */
const char* tcx_version(void);

/* ---------------------------------------------------------------------------
 * Content hashing (the data multihash of an artifact).
 * ------------------------------------------------------------------------ */

/* Leaf-size policy of the GPU entry point. Replaces
 * tensorcast::common::internal::determine_leaf_chunk_size
 * (core/common/artifact_hash_cpu.cc:269-303): the request is clamped to
 * [64, 64 MiB] and aligned down to 64 B; only a request of exactly 4 MiB is
 * then halved (64 B aligned, floor 512 KiB) until there are >= 4096 leaves. */
tcx_status tcx_leaf_policy(uint64_t total_bytes, uint64_t requested_leaf_bytes, uint64_t* leaf_bytes_out);

/* Per-leaf SHA-256 on the device, stream-ordered. Leaf i covers bytes
 * [i*L, min((i+1)*L, T)) of d_src and its 32-byte big-endian digest goes to
 * d_digests + 32*i. Replaces the launch of tensorcast_sha256_leaf_kernel in
 * compute_root_via_nvrtc (core/common/artifact_hash_gpu.cc:384-411, 771-792);
 * unlike the reference it allocates nothing and does not synchronise.
 * Requirements: T in [1, 2^40], L in [1, 64 MiB], ceil(T/L) < 2^32,
 * digest_capacity >= ceil(T/L), d_digests 16-byte aligned. Any alignment of
 * d_src and any L are accepted; L % 16 == 0 with a 16-byte aligned d_src takes
 * the vectorised path. */
tcx_status tcx_sha256_leaves(const void* d_src, uint64_t total_bytes, uint64_t leaf_bytes, void* d_digests,
                             uint64_t digest_capacity, void* stream);

/* Scratch bytes tcx_merkle_root needs for n leaf digests. */
uint64_t tcx_merkle_scratch_bytes(uint64_t n_leaves);

/* Merkle root of n leaf digests on the device, stream-ordered: pairwise
 * SHA-256 of the 64-byte concatenation, an odd trailing node promoted unchanged
 * (compute_tree_hash_sha256, core/common/artifact_hash_cpu.cc:198-233).
 * d_digests is read only; d_root receives 32 bytes; d_scratch must hold
 * tcx_merkle_scratch_bytes(n) bytes, 16-byte aligned. */
tcx_status tcx_merkle_root(const void* d_digests, uint64_t n_leaves, void* d_scratch, uint64_t scratch_bytes,
                           void* d_root, void* stream);

/* 'b' + base32-lower-unpadded(0x12 0x20 || digest) into out (>= 57 bytes, NUL
 * terminated). Replaces to_multibase_multihash_sha256
 * (core/common/artifact_hash_cpu.cc:33-64, 235-254). Host only. */
tcx_status tcx_multihash_encode(const uint8_t* digest32, char* out, size_t out_capacity);

/* Data multihash of the device buffer [d_src, d_src + total_bytes) on device
 * device_id. Replaces tensorcast::common::compute_data_multihash_from_gpu
 * (core/common/artifact_hash.h:28-32, core/common/artifact_hash_gpu.cc:903-957)
 * and compute_data_multihash_from_gpu_memory
 * (core/store/materialization/dataplane/metadata/source_hash.cc:72-78):
 * same argument checks and messages, the tcx_leaf_policy leaf size, and the
 * calling thread's current device is left set to device_id. Synchronous. The
 * digest buffers and the stream are cached per device and reused across calls. */
tcx_status tcx_multihash_from_gpu(const void* d_src, uint64_t total_bytes, int device_id, uint64_t leaf_chunk_bytes,
                                  char* out, size_t out_capacity);

/* Load the hashing kernels and the per-device stream and buffers of device_id;
 * the caller's current device is restored. Replaces
 * prewarm_gpu_hash_nvrtc_for_device (core/common/artifact_hash_gpu.cc:830-854). */
tcx_status tcx_prewarm_device(int device_id);

/* tcx_prewarm_device for every visible device (OK when none is visible).
 * Replaces prewarm_gpu_hash_nvrtc_for_visible_devices (artifact_hash_gpu.cc:856-901). */
tcx_status tcx_prewarm_visible_devices(void);

#ifdef __cplusplus
}
#endif

#endif /* TCX_H_ */
