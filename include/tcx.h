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

/* Number of kernels this library has launched in this process (diagnostics:
 * lets a caller count the device work of a call). No reference counterpart. */
uint64_t tcx_kernel_launch_count(void);

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

/* One pass of streamed per-leaf SHA-256, stream-ordered: consumes bytes
 * [seg_off, seg_off + seg_len) of every leaf of d_src (leaf i at i*L), so a
 * buffer can be hashed while it is still arriving (e.g. one H2D slab per pass).
 * d_states holds 8 words per leaf and carries each chain between passes; the
 * pass that reaches a leaf's end pads it and writes its digest to d_digests.
 * Passes must run in order with seg_off = the previous seg_off + seg_len,
 * starting at 0; seg_off and seg_len are multiples of 64 (seg_len may exceed
 * the leaf). Leaves already finished are left alone. No reference
 * counterpart: the reference hashes only fully resident buffers
 * (core/common/artifact_hash_gpu.cc:693-826); this is the streamed form of the
 * same per-leaf digest. Requirements otherwise as tcx_sha256_leaves, plus
 * d_states 16-byte aligned with 32 * ceil(T/L) bytes. */
tcx_status tcx_sha256_leaves_pass(const void* d_src, uint64_t total_bytes, uint64_t leaf_bytes, uint64_t seg_off,
                                  uint64_t seg_len, void* d_states, void* d_digests, uint64_t digest_capacity,
                                  void* stream);

/* Calibration probe, stream-ordered: n_chains independent SHA-256 chains of
 * `blocks` compressions each on register-resident data (no memory traffic but
 * the 32-byte final states written to d_out). Timed by the caller, it gives the
 * compute bound of the compression (many chains) and the per-block latency of
 * one chain (32 chains). No reference counterpart (measurement aid). */
tcx_status tcx_sha256_compute_probe(uint32_t n_chains, uint32_t blocks, void* d_out, void* stream);

/* Per-leaf SHA-256 over an explicit leaf table, stream-ordered: leaf i covers
 * d_leaf_lengths[i] bytes at d_src + d_leaf_offsets[i] (device arrays); its
 * digest goes to d_digests + 32*i. For segmented inputs (e.g. one buffer per
 * sequence, each split into its own leaves) and for hashing a subset of leaves
 * (the leaf-indexed digests of verification_utils.cc:337-369). Pass
 * offsets_aligned16 = 1 only if d_src and every offset are 16-byte aligned
 * (vectorised kernels); 0 works for any alignment. */
tcx_status tcx_sha256_leaf_table(const void* d_src, const uint64_t* d_leaf_offsets, const uint32_t* d_leaf_lengths,
                                 uint64_t n_leaves, int offsets_aligned16, void* d_digests, void* stream);

/* Scratch bytes tcx_merkle_roots_segmented needs (only segments of more than
 * 2048 leaves use it). seg_first: host array of n_segments + 1 leaf indices. */
uint64_t tcx_merkle_segments_scratch_bytes(const uint64_t* seg_first, uint64_t n_segments);

/* One Merkle root per segment, stream-ordered: segment s is leaves
 * [seg_first[s], seg_first[s+1]) of d_digests and its root (tree of
 * compute_tree_hash_sha256, artifact_hash_cpu.cc:198-233) goes to
 * d_roots + 32*s. seg_first is given twice: on the host (to plan) and on the
 * device (d_seg_first, read by the kernel). Empty segments are rejected. */
tcx_status tcx_merkle_roots_segmented(const void* d_digests, const uint64_t* seg_first, const uint64_t* d_seg_first,
                                      uint64_t n_segments, void* d_scratch, uint64_t scratch_bytes, void* d_roots,
                                      void* stream);

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
 * calling thread's current device is left set to device_id. Synchronous: the
 * hash starts after the work already queued on the legacy default stream and
 * the call returns with the result. The digest buffers and the stream are
 * cached per device and reused across calls. */
tcx_status tcx_multihash_from_gpu(const void* d_src, uint64_t total_bytes, int device_id, uint64_t leaf_chunk_bytes,
                                  char* out, size_t out_capacity);

/* The data multihash of tcx_multihash_from_gpu, for callers that cannot call
 * cudaMalloc at that moment: an engine that has already reserved nearly all
 * device memory for its own pool, or a path that must not wait on cudaFree
 * (which synchronises the device). It allocates nothing, device or host: its
 * scratch is a fixed array in the library's device memory, held by every GPU
 * that loads the library until the process exits. No counterpart in the
 * reference.
 * Same arguments, checks, leaf policy and result as tcx_multihash_from_gpu,
 * plus the stream the work runs on (NULL: the legacy default stream; otherwise
 * a stream of device_id, else INVALID_ARGUMENT); returns once the result is on
 * the host. The caller's current device is restored before it returns. Limit:
 * at most 16384 leaves per call (64 GiB at the 4 MiB default leaf); more is
 * INVALID_ARGUMENT.
 * The first call on a device finds the scratch array's device address; make
 * that first call before any stream capture. Calls
 * on one device share the scratch and are serialised by the library; work that
 * overlaps them on the GPU from elsewhere with the same scratch would race. */
tcx_status tcx_multihash_from_gpu_noalloc(const void* d_src, uint64_t total_bytes, int device_id,
                                          uint64_t leaf_chunk_bytes, char* out, size_t out_capacity, void* stream);

/* Load the hashing kernels and the per-device stream and buffers of device_id;
 * the caller's current device is restored. Replaces
 * prewarm_gpu_hash_nvrtc_for_device (core/common/artifact_hash_gpu.cc:830-854). */
tcx_status tcx_prewarm_device(int device_id);

/* tcx_prewarm_device for every visible device (OK when none is visible).
 * Replaces prewarm_gpu_hash_nvrtc_for_visible_devices (artifact_hash_gpu.cc:856-901). */
tcx_status tcx_prewarm_visible_devices(void);

/* ---------------------------------------------------------------------------
 * View materialisation (tensor-parallel shards, slices and transposes).
 * ------------------------------------------------------------------------ */

#define TCX_MAX_DIMS 8

/* One strided byte copy: `rows` rows of `row_bytes` bytes, row k read from
 * src + src_off + k*src_pitch and written to dst + dst_off + k*dst_pitch.
 * An identity or dim-0 narrowed tensor is one row; a narrow along dim d > 0 is
 * prod(shape[:d]) rows of length*prod(shape[d+1:])*esize bytes at source pitch
 * shape[d]*prod(shape[d+1:])*esize -- the `outer` blocks of
 * compute_bidirectional_internal (view_planner.cc:466-524). */
typedef struct tcx_copy_job {
  uint64_t src_off;
  uint64_t dst_off;
  uint64_t src_pitch;
  uint64_t dst_pitch;
  uint64_t row_bytes;
  uint64_t rows;
} tcx_copy_job;

/* A compact tensor of `shape` (element size esize) at src + src_off, written
 * permuted to dst + dst_off: output dim i is input dim perm[i], i.e.
 * torch permute(perm).contiguous() (view_transform_executor.cc:116-131). */
typedef struct tcx_permute_job {
  uint64_t src_off;
  uint64_t dst_off;
  uint32_t esize;
  uint32_t ndim;
  int64_t shape[TCX_MAX_DIMS];
  int32_t perm[TCX_MAX_DIMS];
} tcx_permute_job;

/* Device scratch bytes tcx_copy_jobs needs for n jobs. */
uint64_t tcx_copy_jobs_scratch_bytes(uint64_t n_jobs);

/* Runs n copy jobs (d_jobs: device array) from d_src to d_dst in one
 * stream-ordered launch pair. Destination ranges must not overlap each other
 * or the source. Replaces the GenericByteRangeExecutor data copies and the
 * cudaMemcpy2DAsync column packs of execute_dim1_tensor
 * (core/store/replica/collective_disk_loader.cc:4488-4508). */
tcx_status tcx_copy_jobs(const void* d_src, void* d_dst, const tcx_copy_job* d_jobs, uint64_t n_jobs,
                         void* d_scratch, uint64_t scratch_bytes, void* stream);

/* One out-of-place permute (job in host memory), stream-ordered. Replaces the
 * GPU branch of execute_transform
 * (core/store/materialization/dataplane/view/view_transform_executor.cc:74-133). */
tcx_status tcx_permute(const void* d_src, void* d_dst, const tcx_permute_job* job, void* stream);

/* ---------------------------------------------------------------------------
 * Collective from-disk load: each rank stages 1/N of the canonical byte space
 * (leaf-aligned) into its own VRAM, hashes the leaves it staged, and the ranks
 * exchange over NVLink (NCCL grouped send/recv) exactly the bytes each peer's
 * view needs; every rank then holds its view and the artifact's Merkle root.
 * Replaces try_collective_disk_load / execute_group_collective
 * (core/store/replica/collective_disk_loader.h:120-142,
 * collective_disk_loader.cc:5538-5816) and the verification-stage hash of the
 * loaded replica (core/store/materialization/runtime/pipeline/
 * verification_stage.cc:55-128).
 * ------------------------------------------------------------------------ */

#define TCX_UNIQUE_ID_BYTES 128

typedef struct tcx_group tcx_group;

/* A file range to read into pinned memory: `length` bytes at `file_offset` of
 * `path` land at dst_offset of the destination buffer. */
typedef struct tcx_file_segment {
  const char* path;
  uint64_t file_offset;
  uint64_t dst_offset;
  uint64_t length;
} tcx_file_segment;

/* Everything a rank needs to know about one collective load; identical on
 * every rank except the buffers. */
typedef struct tcx_load_plan {
  uint64_t total_bytes;          /* T: size of the canonical byte space */
  uint64_t leaf_bytes;           /* hash leaf size L (used as given) */
  const uint64_t* stage_bounds;  /* world+1 offsets, multiples of L, bounds[world] = T:
                                    rank r stages [bounds[r], bounds[r+1]) */
  const tcx_copy_job* jobs;      /* every rank's view: src_off in the canonical space,
                                    dst_off/dst_pitch in that rank's view buffer */
  const uint64_t* job_offsets;   /* world+1: rank r's jobs are jobs[off[r], off[r+1]) */
  const tcx_permute_job* permutes; /* this rank's in-place permutes of view regions, run
                                      after the exchange (src_off == dst_off) */
  uint64_t n_permutes;
  uint64_t view_bytes;           /* bytes of this rank's view buffer */
  uint64_t slab_bytes;           /* bytes per leaf per H2D/hash slab (0: 256 KiB) */
  uint64_t window_bytes;         /* bytes per peer per exchange round; bounds the send/receive
                                    scratch to about 2*(N-1) windows (0: 512 MiB) */
  uint64_t flags;                /* TCX_LOAD_* bits */
  const uint64_t* target_ranges; /* TCX_LOAD_TARGETS: n_targets (offset, length) pairs of this
                                    rank's view space that are writable; NULL otherwise */
  uint64_t n_targets;
  uint64_t push_nccl_permille;   /* with TCX_LOAD_PEER_PUSH: this share (per mille, whole pieces in
                                    view order) of every (sender, receiver) pair's bytes goes over
                                    NCCL send/recv at the same time as the copy engines push the rest
                                    (0: the copy engines carry everything) */
} tcx_load_plan;

/* tcx_load_plan.flags: also compute the data multihash of this rank's finished
 * view (leaf size from tcx_leaf_policy(view_bytes, 4 MiB)), as the reference's
 * ViewHashComputer::hash_replica_view does for a GPU-resident view
 * (core/store/materialization/common/view_hash_utils.cc:38-82). */
#define TCX_LOAD_VIEW_HASH 1ull

/* tcx_load_plan.flags: exchange by pushing over peer memory instead of NCCL
 * send/recv: every rank maps every peer's view (CUDA IPC; d_view must be memory
 * this process allocated with cudaMalloc) and copies the peers' view pieces
 * from its staged bytes directly into those views over NVLink with the copy
 * engines (one 2-D copy per piece, one stream per peer; a peer that is a thread
 * of this process is written through its own pointer), so extraction and
 * transfer are one pass with no pack or receive buffers and no SM time is taken
 * from the leaf hash running at the same time. NCCL carries only the handle
 * exchange and two one-word barriers. */
#define TCX_LOAD_PEER_PUSH 2ull

/* tcx_load_plan.flags: exchange by a windowed all-gather instead of the shard
 * exchange: round k broadcasts every rank's staged bytes [bounds[r] + k*W,
 * bounds[r] + (k+1)*W) to all ranks (W = window_bytes; one ncclBroadcast per
 * root in one group) and each rank copies its view pieces out of the peers'
 * windows. Every rank then has seen every byte (T*(N-1)/N received per rank),
 * the reference's collective shape (collective_disk_loader.cc:4276-4554: chunks
 * broadcast from their owner); the default shard exchange moves only each view's
 * bytes. Excludes TCX_LOAD_PEER_PUSH. */
#define TCX_LOAD_ALLGATHER 8ull

/* tcx_load_plan.flags: the view is a set of separate caller tensors (the
 * reference's bind_into / mapped-target load, collective_disk_loader.cc:7909-8157,
 * 5818-6293): d_view is the lowest target's address, view offsets are device
 * addresses relative to it, and target_ranges lists the writable (offset,
 * length) ranges. Every job and permute of this rank must lie inside one
 * target; bytes between targets are never touched (no gap zero-fill). Not
 * combinable with TCX_LOAD_VIEW_HASH or TCX_LOAD_PEER_PUSH (the exchange is
 * the NCCL send/recv shard exchange or TCX_LOAD_ALLGATHER). */
#define TCX_LOAD_TARGETS 4ull

/* Per-peer sizes and job lists of the exchange for one rank (host-only planning).
 * Capacities: tcx_plan_exchange_capacity(). pack_jobs move this rank's staged
 * bytes (src offsets relative to the staged range) into the send buffer;
 * local_jobs move them straight into the view; scatter_jobs move received
 * bytes from the receive buffer into the view, for peers whose bytes do not
 * land contiguously (direct[p] == 0). direct[p] == 1: the bytes from peer p are
 * received straight into the view at recv_view_off[p]. */
typedef struct tcx_exchange_plan {
  tcx_copy_job* pack_jobs;
  uint64_t n_pack;
  tcx_copy_job* local_jobs;
  uint64_t n_local;
  tcx_copy_job* scatter_jobs;
  uint64_t n_scatter;
  uint64_t* send_offsets;   /* world+1 offsets into the send buffer */
  uint64_t* recv_offsets;   /* world+1 offsets into the receive buffer (non-direct peers) */
  uint64_t* recv_counts;    /* world: bytes received from each peer */
  uint64_t* recv_view_off;  /* world: view offset of a direct receive */
  uint8_t* direct;          /* world flags */
  uint64_t* gaps;           /* 2*capacity entries: (offset, length) pairs of view bytes no job
                               writes; the load zero-fills them */
  uint64_t n_gaps;
} tcx_exchange_plan;

/* Upper bound on each job count and gap count tcx_plan_exchange may produce
 * (each job array needs this many entries, gaps twice as many). */
uint64_t tcx_plan_exchange_capacity(const tcx_load_plan* plan, int world);

/* Host-only: the exchange schedule of `rank` in a `world`-rank load. */
tcx_status tcx_plan_exchange(const tcx_load_plan* plan, int world, int rank, tcx_exchange_plan* out);

/* Capacity of each output job array of tcx_plan_push_split. */
uint64_t tcx_plan_push_split_capacity(const tcx_load_plan* plan, int world);

/* Host-only: the split tcx_group_load makes of a push exchange with
 * push_nccl_permille > 0 (no reference counterpart: the reference moves every
 * peer's bytes with NCCL). For every (sender p, receiver r) pair, r's jobs clipped
 * to p's staged range are taken in order; pieces go to NCCL until nccl_permille of
 * the pair's bytes is reached, the rest to the copy engines. nccl_jobs receives
 * every receiver's NCCL pieces (canonical source offsets, the receiver's view
 * offsets; receiver r's at nccl_job_offsets[r..r+1]) -- a load plan of only those
 * pieces gives the NCCL rounds; ce_jobs receives this rank's copy-engine pieces
 * (source offsets relative to its staged range), receiver r's at ce_offsets[r..r+1].
 * Every rank computes the same nccl_jobs from the same plan. */
tcx_status tcx_plan_push_split(const tcx_load_plan* plan, int world, int rank, uint64_t nccl_permille,
                               tcx_copy_job* nccl_jobs, uint64_t* nccl_job_offsets, tcx_copy_job* ce_jobs,
                               uint64_t* ce_offsets, uint64_t capacity);

/* Reads segments into dst (pinned or pageable host memory) with `threads`
 * parallel preads; a short read is DATA_LOSS (source_hash.cc:44-51).
 * Equivalent to tcx_read_segments_ex(segs, n, dst, threads, 0). */
tcx_status tcx_read_segments(const tcx_file_segment* segs, uint64_t n, void* dst, int threads);

/* tcx_read_segments_ex flag: bypass the page cache (O_DIRECT) for cold reads;
 * files on a file system that refuses O_DIRECT are read buffered. */
#define TCX_READ_DIRECT 1ull

/* tcx_read_segments with flags. Pieces are read in source order (file, then
 * offset), each thread reading forward, whatever order the segments are listed
 * in: the source-ordered windows of the reference's safetensors readers
 * (PreadMultiSafetensorsSource / DirectAlignedSafetensorsSource,
 * collective_disk_loader.cc:1571-2200). With TCX_READ_DIRECT, nearby pieces
 * (gaps up to 256 KiB) are read as one 4 KiB-aligned window of at most 16 MiB
 * into an aligned bounce buffer and copied out, so segments need no alignment. */
tcx_status tcx_read_segments_ex(const tcx_file_segment* segs, uint64_t n, void* dst, int threads, uint64_t flags);

/* Progress of a streamed hash: bytes whose leaves are hashed so far, of total. */
typedef void (*tcx_progress_fn)(uint64_t processed_bytes, uint64_t total_bytes, void* ctx);

/* Data multihash of a byte stream stored in files, hashed on `device`.
 * Replaces compute_data_multihash_from_seekable_source
 * (core/store/materialization/dataplane/metadata/source_hash.cc:19-61) as
 * called by compute_data_multihash_from_disk_dir (disk_dir_hash.cc:47-104):
 * the stream [0, total) is given as file segments in stream order (dst_offset
 * = stream offset; they must tile [0, total) exactly), cut into leaves of
 * leaf_bytes (used as given, no adaptive policy, as the CPU path), SHA-256 per
 * leaf, Merkle tree, multihash. Leaves of at least two 64 KiB pieces are
 * streamed: in waves of up to 4096 leaves, read_threads reader threads (0 = up
 * to 16) pread piece j (up to 256 KiB) of a few consecutive leaves into a pinned
 * buffer and copy it at once into one of three device slab buffers; one pass
 * of the leaf kernel per slab advances every chain of the wave. Otherwise (or
 * with TCX_READ_DIRECT in read_flags, as tcx_read_segments_ex, or the
 * environment variable TCX_STAGE=slabs), groups of whole leaves (group_bytes,
 * 0 = 1 GiB) are read by parallel preads into `depth` pinned slots (0 = 4),
 * copied and hashed on one stream per slot. Either way reads, copies and
 * hashing overlap. The buffers stay allocated per device for the next call
 * (tcx_file_hash_release frees them); calls on one device are serialised. Synchronous; restores the caller's current device. Errors as
 * the reference: total 0 or leaf 0 is
 * INVALID_ARGUMENT, a short read DATA_LOSS "short read while hashing source".
 * root_out (optional) receives the 32-byte root; out (>= 57 bytes) the
 * multihash. progress (optional) is called on the calling thread. */
tcx_status tcx_multihash_from_file_segments(const tcx_file_segment* segs, uint64_t n_segs, uint64_t total,
                                            uint64_t leaf_bytes, int device, uint64_t group_bytes, int depth,
                                            int read_threads, uint64_t read_flags, tcx_progress_fn progress,
                                            void* progress_ctx, uint8_t* root_out, char* out, uint64_t out_len);

/* Frees the pinned and device buffers tcx_multihash_from_file_segments keeps for
 * `device` (-1: every device). No counterpart in the reference (it allocates per
 * call). */
tcx_status tcx_file_hash_release(int device);

/* Maps [offset, offset + length) of a file into host memory and, when
 * register_pinned != 0, page-locks the mapping (cudaHostRegister; a read-only
 * mapping registered read-only where the driver accepts it, else a shared
 * read-write mapping that is never written) so that host-to-device copies
 * read the file's page-cache pages directly: a
 * tmpfs-resident artifact can be staged without a second host copy. *host_ptr
 * is the first mapped byte; release with tcx_host_unmap_file(handle).
 * UNAVAILABLE if the driver refuses to register the mapping. Replaces the
 * pread-into-pinned-pool staging of collective_disk_loader.cc:4254-4261. */
tcx_status tcx_host_map_file(const char* path, uint64_t offset, uint64_t length, int register_pinned,
                             void** host_ptr, void** handle);

/* Unregisters and unmaps a mapping made by tcx_host_map_file. */
tcx_status tcx_host_unmap_file(void* handle);

/* Binds the calling thread to the CPUs local to CUDA device `device` (sysfs
 * local_cpulist of its PCI function), so pinned staging buffers it allocates
 * and touches afterwards live on the GPU's NUMA node; *n_cpus_out (may be
 * NULL) receives the CPU count. Stands in for the NUMA options of the
 * reference's pinned pool (core/common/memory/). */
tcx_status tcx_bind_device_cpus(int device, int* n_cpus_out);

/* A new NCCL unique id (rank 0 creates it; the caller distributes the bytes). */
tcx_status tcx_group_unique_id(uint8_t* out128);

/* Joins rank `rank` of a `world`-rank group on CUDA device `device`
 * (unique_id may be NULL when world == 1). Waits at most timeout_ms for the
 * other ranks (DEADLINE_EXCEEDED, communicator aborted). Replaces the
 * NcclClique of collective_disk_loader.cc:209-306 (one process per GPU here
 * instead of one leader thread driving every GPU). */
tcx_status tcx_group_create(const uint8_t* unique_id, int world, int rank, int device, int64_t timeout_ms,
                            tcx_group** out);

/* tcx_group_create for rank threads of one process, the reference daemon's model
 * (try_collective_disk_load called by N rank threads that rendezvous on group_id,
 * collective_disk_loader.cc:8159-8277; clique over the local GPUs, :229-247):
 * the first thread to join `group_id` creates the NCCL unique id and every rank
 * thread of the group takes it from an in-process table, then joins as
 * tcx_group_create does (one communicator per thread, waiting at most timeout_ms
 * for the others). A rank joining twice, or a different world size under the same
 * id, is INVALID_ARGUMENT; an id whose ranks did not all join within timeout_ms
 * starts a new generation at its next join. Loads of such groups may use
 * TCX_LOAD_PEER_PUSH: peers in the same process are written through their own
 * pointers (peer access enabled), peers in other processes through CUDA IPC. */
tcx_status tcx_group_join(const char* group_id, int world, int rank, int device, int64_t timeout_ms,
                          tcx_group** out);

/* Releases the group's communicator, streams and device buffers. */
tcx_status tcx_group_destroy(tcx_group* g);

typedef struct tcx_load_result {
  uint8_t root[32];     /* Merkle root over all ranks' leaves */
  char multihash[64];   /* data multihash of the root (NUL terminated) */
  uint64_t leaves;      /* total leaf count */
  uint64_t h2d_bytes;   /* host-to-device bytes of this rank */
  uint64_t peer_send_bytes, peer_recv_bytes;
  float h2d_ms, hash_ms, exchange_ms, total_ms;  /* device-timed phases on this rank */
  char view_multihash[64];  /* with TCX_LOAD_VIEW_HASH: data multihash of this rank's view, else "" */
  uint64_t view_leaf_bytes; /* leaf size used for view_multihash */
  float stage_read_ms;      /* tcx_group_load_files: host time from the first read to the last slab read */
  float transfer_ms;        /* device time of this rank's peer transfer: its pushes, or the NCCL rounds */
} tcx_load_result;

/* Runs one collective load on every rank of g (all ranks call it with the same
 * plan). h_stage: this rank's staged bytes in pinned host memory, or NULL when
 * d_stage already holds them (device-resident load: no H2D). d_view may equal
 * d_stage when every job of this rank is an in-place identity. The load starts
 * after the work already queued on `stream` (the caller's stream, NULL = the
 * legacy default stream) and the call returns once it is complete.
 * expected_root (32 bytes, may be NULL): a mismatch returns DATA_LOSS
 * (verification_stage.cc:130-141). Loads on one group run one at a time
 * (concurrent calls wait); different groups are independent. */
tcx_status tcx_group_load(tcx_group* g, const tcx_load_plan* plan, const void* h_stage, void* d_stage, void* d_view,
                          const uint8_t* expected_root, tcx_load_result* out, void* stream);

/* Where tcx_group_load_files reads this rank's staged range from. */
typedef struct tcx_file_stage {
  const tcx_file_segment* segments; /* the staged range [bounds[rank], bounds[rank+1]) as file ranges,
                                       dst_offset relative to bounds[rank]; bytes no segment covers
                                       are zero (the canonical space's alignment pads) */
  uint64_t n_segments;
  int read_threads;                 /* host reader threads (0: the CPUs the caller may run on, shared among
                                       the groups alive in this process, 2 to 32) */
  int ring_slots;                   /* slab staging: pinned slabs read ahead (0: 4) */
  uint64_t slot_bytes;              /* slab staging: pinned bytes per slab when plan->slab_bytes is 0
                                       (0: 512 MiB) */
} tcx_file_stage;

/* tcx_group_load with the staged range read from files inside the call, so
 * reads, host-to-device copies and the streamed SHA-256 passes overlap (the
 * reference's read -> pinned -> H2D chunk loop with its two-deep
 * ChunkPrefetcher, collective_disk_loader.cc:2277-2383, 5538-5816). Slab j is
 * bytes [j*S, (j+1)*S) of every leaf of the range, and its hash pass runs once
 * it is on the device.
 *  - Leaves of at least two pieces (plan->slab_bytes 0): piece staging. S is a
 *    piece of up to 256 KiB and at most half a leaf; a reader thread preads the pieces of slab j of a few
 *    consecutive leaves (about 4 MiB) into one of its two pinned buffers and at
 *    once queues their 2-D copy on its own stream.
 *  - Otherwise (or with the environment variable TCX_STAGE=slabs): the readers
 *    pread slab j into pinned slot j % ring_slots, copied with one 2-D copy.
 * The pinned buffers and the threads stay with the group for later loads. A
 * file that cannot be opened is NOT_FOUND, a short read DATA_LOSS; total_ms
 * then covers the reads as well. */
tcx_status tcx_group_load_files(tcx_group* g, const tcx_load_plan* plan, const tcx_file_stage* files, void* d_stage,
                                void* d_view, const uint8_t* expected_root, tcx_load_result* out, void* stream);

/* ---------------------------------------------------------------------------
 * Paged KV-cache gather (no reference counterpart: the reference stores
 * engine-owned KV as opaque byte artifacts, tests/python/test_kvcache_adapter.py).
 * ------------------------------------------------------------------------ */

/* Gathers each sequence's pages from a paged pool into one contiguous buffer,
 * stream-ordered. Pool page p of plane k: d_pool + (k*pool_pages + p) *
 * page_tokens*token_bytes. Sequence s has d_seq_tokens[s] tokens in pages
 * d_page_table[d_page_offsets[s] .. d_page_offsets[s+1]) and is written at
 * d_out + d_out_offsets[s] as [plane][token][token_bytes]. total_pages =
 * d_page_offsets[n_seq] (host copy). Table entries are checked on the device:
 * a bad one skips that page and leaves a non-zero code in *d_status (1 slot out
 * of the pool, 2 page past the sequence's tokens, 3 output past out_bytes);
 * *d_status must be zero before the call. */
tcx_status tcx_kv_gather(const void* d_pool, uint32_t planes, uint64_t pool_pages, uint32_t page_tokens,
                         uint64_t token_bytes, const uint32_t* d_page_table, const uint64_t* d_page_offsets,
                         const uint32_t* d_seq_tokens, const uint64_t* d_out_offsets, uint64_t n_seq,
                         uint64_t total_pages, void* d_out, uint64_t out_bytes, uint32_t* d_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TCX_H_ */
