// Data multihash of byte ranges of files, hashed on the GPU.
//
// The reference hashes an artifact directory on the CPU
// (compute_data_multihash_from_disk_dir, disk_dir_hash.cc:47-104, through
// compute_data_multihash_from_seekable_source, source_hash.cc:19-61): the
// files' bytes form one stream (safetensors payloads in file-name order, or
// numbered partitions in numeric order), cut into fixed leaves, one SHA-256
// per leaf on one core, then the Merkle tree. Here the caller resolves the
// stream to file segments and this entry point streams it through the GPU:
//
//   host threads: pread group k+1 into pinned slot (k+1) % depth
//   slot stream:  H2D of group k, then the leaf kernel over its whole leaves
//   end:          Merkle root of all leaf digests on the device, 32 bytes back
//
// A group is a whole number of leaves, so every leaf is hashed in one launch
// and groups are independent; `depth` slots (pinned + device buffer + stream)
// keep reads, copies and hashing of different groups in flight at once.
//
// Leaves of two pieces or more are streamed instead (hash_file_segments_streamed):
// the leaves go in waves of up to 4096, and slab j of a wave is the 256 KiB piece
// j of each of its leaves. Reader threads pread the pieces of a few consecutive
// leaves into one of their own pinned buffers and queue its copy into a device
// slab buffer at once (as the collective load does); once a slab is on the
// device one pass of the leaf kernel advances every chain of the wave over it,
// so thousands of chains hash at once from a ring of three slab buffers instead
// of a few hundred per 1 GiB group.
//
// The buffers stay allocated per device between calls (tcx_file_hash_release
// frees them); calls on one device are serialised.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "staging.h"
#include "tcx_internal.h"

namespace tcx {
namespace {

constexpr uint64_t kDefaultGroupBytes = 1ull << 30;
constexpr int kDefaultDepth = 4;

// Streamed hashing: bytes of one leaf per slab, bytes per host-to-device copy,
// pinned buffers per reader thread, device slab buffers and their total bytes.
constexpr uint64_t kPieceBytes = 256ull << 10;
constexpr uint64_t kMinPieceBytes = 64ull << 10;
constexpr uint64_t kPieceCopy = 4ull << 20;
constexpr int kPieceBufs = 2;
constexpr int kSlabRing = 3;
constexpr uint64_t kSlabRingBytes = 3ull << 30;  // TCX_HASH_WAVE_LEAVES overrides the leaves per wave

struct Slot {
  uint8_t* host = nullptr;
  uint8_t* dev = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t hashed = nullptr;  // leaf digests of the slot's group written
  int64_t group = -1;
};

// Per-device buffers, kept between calls (page-locking gigabytes of host memory
// costs far more than one hash of them) until tcx_file_hash_release.
struct FileHashContext {
  std::mutex mu;
  std::vector<Slot> slots;
  uint64_t slot_bytes = 0;
  uint8_t* digests = nullptr;
  uint64_t digest_bytes = 0;
  uint8_t* scratch = nullptr;
  uint64_t scratch_bytes = 0;
  uint8_t* root = nullptr;
  // Streamed hashing.
  std::unique_ptr<ReadPool> readers;
  PieceBuffers pieces;
  uint8_t* ring = nullptr;  // kSlabRing slab buffers
  uint64_t ring_bytes = 0;
  std::vector<cudaEvent_t> ring_free;  // per slab buffer: the pass that last read it
  std::vector<cudaEvent_t> wave_done;  // per wave: its leaf digests written
  cudaStream_t s_hash = nullptr;
  uint32_t* states = nullptr;
  uint64_t states_bytes = 0;

  void free_stream() {
    readers.reset();  // joins the reader threads before their buffers go away
    pieces.release();
    if (s_hash) cudaStreamSynchronize(s_hash);
    for (auto* v : {&ring_free, &wave_done}) {
      for (cudaEvent_t e : *v) cudaEventDestroy(e);
      v->clear();
    }
    if (s_hash) cudaStreamDestroy(s_hash);
    s_hash = nullptr;
    if (ring) cudaFree(ring);
    ring = nullptr;
    ring_bytes = 0;
    if (states) cudaFree(states);
    states = nullptr;
    states_bytes = 0;
  }
  tcx_status ensure_stream(int n_readers, uint64_t piece_buf, uint64_t ring_total, uint64_t n_states_bytes,
                           uint64_t n_waves) {
    if (!readers || readers->size() != n_readers) {
      readers.reset();
      readers = std::make_unique<ReadPool>(n_readers);
    }
    if (tcx_status st = pieces.ensure(n_readers, piece_buf, kPieceBufs); st != TCX_OK) return st;
    if (s_hash == nullptr) TCX_CUDA_TRY(cudaStreamCreateWithFlags(&s_hash, cudaStreamNonBlocking));
    while (ring_free.size() < static_cast<size_t>(kSlabRing) || wave_done.size() < n_waves) {
      cudaEvent_t e;
      TCX_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      (ring_free.size() < static_cast<size_t>(kSlabRing) ? ring_free : wave_done).push_back(e);
    }
    if (ring_bytes < ring_total) {
      if (ring) cudaFree(ring);
      ring = nullptr;
      ring_bytes = 0;
      if (cudaError_t e = cudaMalloc(&ring, ring_total); e != cudaSuccess) {
        cudaGetLastError();
        return set_errorf(TCX_RESOURCE_EXHAUSTED, "file hash slab buffers of %llu bytes: %s",
                          static_cast<unsigned long long>(ring_total), cuda_msg(e).c_str());
      }
      ring_bytes = ring_total;
    }
    if (states_bytes < n_states_bytes) {
      if (states) cudaFree(states);
      states = nullptr;
      states_bytes = 0;
      TCX_CUDA_TRY(cudaMalloc(&states, n_states_bytes));
      states_bytes = n_states_bytes;
    }
    return TCX_OK;
  }

  void free_slots() {
    for (auto& s : slots) {
      if (s.stream) cudaStreamSynchronize(s.stream);
      if (s.hashed) cudaEventDestroy(s.hashed);
      if (s.stream) cudaStreamDestroy(s.stream);
      if (s.host) cudaFreeHost(s.host);
      if (s.dev) cudaFree(s.dev);
    }
    slots.clear();
    slot_bytes = 0;
  }
  void free_all() {
    free_stream();
    free_slots();
    if (digests) cudaFree(digests);
    if (scratch) cudaFree(scratch);
    if (root) cudaFree(root);
    digests = scratch = root = nullptr;
    digest_bytes = scratch_bytes = 0;
  }
  tcx_status ensure_common(uint64_t n_digest_bytes, uint64_t n_scratch_bytes) {
    if (digest_bytes < n_digest_bytes) {
      if (digests) cudaFree(digests);
      digests = nullptr;
      digest_bytes = 0;
      TCX_CUDA_TRY(cudaMalloc(&digests, n_digest_bytes));
      digest_bytes = n_digest_bytes;
    }
    if (scratch_bytes < n_scratch_bytes) {
      if (scratch) cudaFree(scratch);
      scratch = nullptr;
      scratch_bytes = 0;
      TCX_CUDA_TRY(cudaMalloc(&scratch, n_scratch_bytes));
      scratch_bytes = n_scratch_bytes;
    }
    if (root == nullptr) TCX_CUDA_TRY(cudaMalloc(&root, 256));
    return TCX_OK;
  }
  tcx_status ensure(int n_slots, uint64_t bytes, uint64_t n_digest_bytes, uint64_t n_scratch_bytes) {
    if (static_cast<int>(slots.size()) < n_slots || slot_bytes < bytes) {
      free_slots();
      slots.resize(n_slots);
      slot_bytes = bytes;
      for (auto& s : slots) {
        cudaError_t e = cudaMallocHost(&s.host, bytes);
        if (e == cudaSuccess) e = cudaMalloc(&s.dev, bytes);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.hashed, cudaEventDisableTiming);
        if (e != cudaSuccess) {
          cudaGetLastError();
          free_slots();
          return set_error(e == cudaErrorMemoryAllocation ? TCX_RESOURCE_EXHAUSTED : TCX_INTERNAL,
                           std::string("file hash buffers: ") + cudaGetErrorString(e));
        }
      }
    }
    for (auto& s : slots) s.group = -1;
    return ensure_common(n_digest_bytes, n_scratch_bytes);
  }
  // After an error: nothing of this call may still run when the buffers are next used.
  void drain() {
    for (auto& s : slots)
      if (s.stream) cudaStreamSynchronize(s.stream);
    pieces.sync();
    if (s_hash) cudaStreamSynchronize(s_hash);
  }
};

std::mutex g_contexts_mu;
std::map<int, std::unique_ptr<FileHashContext>> g_contexts;

FileHashContext* context_for(int device) {
  std::lock_guard<std::mutex> lock(g_contexts_mu);
  auto& c = g_contexts[device];
  if (!c) c = std::make_unique<FileHashContext>();
  return c.get();
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

tcx_status hash_file_segments(FileHashContext& r, const tcx_file_segment* segs, uint64_t n_segs, uint64_t total,
                              uint64_t leaf_bytes, uint64_t group_bytes, int depth, int read_threads,
                              uint64_t read_flags, tcx_progress_fn progress, void* progress_ctx, uint8_t root[32]) {
  const uint64_t n_leaves = (total + leaf_bytes - 1) / leaf_bytes;
  uint64_t G = std::max<uint64_t>(1, (group_bytes ? group_bytes : kDefaultGroupBytes) / leaf_bytes);
  G = std::min<uint64_t>(G, n_leaves);
  const uint64_t gbytes = G * leaf_bytes;
  const uint64_t n_groups = (n_leaves + G - 1) / G;
  const int D = static_cast<int>(std::min<uint64_t>(std::max(1, depth > 0 ? depth : kDefaultDepth), n_groups));
  const int threads = read_threads > 0 ? read_threads
                                       : std::max(1, std::min(16, static_cast<int>(std::thread::hardware_concurrency())));
  if (tcx_status st = r.ensure(D, gbytes, n_leaves * 32, std::max<uint64_t>(merkle_scratch_bytes(n_leaves), 256));
      st != TCX_OK)
    return st;

  if (progress) progress(0, total, progress_ctx);
  uint64_t reported = 0;  // groups whose digests are known to be written, reported in order
  // Reports groups [reported, limit) as their hashes complete; `wait` blocks on each.
  auto report_done = [&](uint64_t limit, bool wait) -> tcx_status {
    while (reported < limit) {
      const Slot& s = r.slots[reported % D];
      if (s.group != static_cast<int64_t>(reported)) break;  // not enqueued yet
      const cudaError_t q = wait ? cudaEventSynchronize(s.hashed) : cudaEventQuery(s.hashed);
      if (q == cudaErrorNotReady) break;
      if (q != cudaSuccess) return set_error(TCX_INTERNAL, std::string("leaf hashing failed: ") + cudaGetErrorString(q));
      ++reported;
      if (progress) progress(std::min(total, reported * gbytes), total, progress_ctx);
    }
    return TCX_OK;
  };

  std::vector<tcx_file_segment> piece;
  uint64_t seg_i = 0;
  for (uint64_t k = 0; k < n_groups; ++k) {
    Slot& s = r.slots[k % D];
    if (s.group >= 0) {
      // The slot's previous group (k - depth) is hashed (so also copied out of the
      // pinned buffer) and reported before the slot's event is recorded again.
      if (tcx_status st = report_done(k - D + 1, true); st != TCX_OK) return st;
    }
    const uint64_t g0 = k * gbytes, g1 = std::min(total, g0 + gbytes);
    piece.clear();
    while (seg_i < n_segs && segs[seg_i].dst_offset + segs[seg_i].length <= g0) ++seg_i;
    for (uint64_t i = seg_i; i < n_segs && segs[i].dst_offset < g1; ++i) {
      const uint64_t a = std::max(g0, segs[i].dst_offset), b = std::min(g1, segs[i].dst_offset + segs[i].length);
      if (a >= b) continue;
      piece.push_back({segs[i].path, segs[i].file_offset + (a - segs[i].dst_offset), a - g0, b - a});
    }
    tcx_status st = tcx_read_segments_ex(piece.data(), piece.size(), s.host, threads, read_flags);
    if (st == TCX_DATA_LOSS) return set_error(TCX_DATA_LOSS, "short read while hashing source");
    if (st != TCX_OK) return st;
    const uint64_t len = g1 - g0;
    TCX_CUDA_TRY(cudaMemcpyAsync(s.dev, s.host, len, cudaMemcpyHostToDevice, s.stream));
    const uint64_t first = k * G, n = (len + leaf_bytes - 1) / leaf_bytes;
    st = launch_leaf_pass(s.dev, len, leaf_bytes, static_cast<uint32_t>(n), 0, ~0ull, nullptr,
                          r.digests + first * 32, s.stream);
    if (st != TCX_OK) return st;
    TCX_CUDA_TRY(cudaEventRecord(s.hashed, s.stream));
    s.group = static_cast<int64_t>(k);
    if (tcx_status st2 = report_done(k, false); st2 != TCX_OK) return st2;
  }
  // Merkle root on slot 0's stream once every group's digests are written.
  cudaStream_t fin = r.slots[0].stream;
  for (int i = 1; i < D; ++i) TCX_CUDA_TRY(cudaStreamWaitEvent(fin, r.slots[i].hashed, 0));
  if (tcx_status st = launch_merkle(r.digests, n_leaves, r.scratch, r.root, fin); st != TCX_OK) return st;
  TCX_CUDA_TRY(cudaMemcpyAsync(root, r.root, 32, cudaMemcpyDeviceToHost, fin));
  TCX_CUDA_TRY(cudaStreamSynchronize(fin));
  return report_done(n_groups, true);
}

// Piece size for leaves of `leaf` bytes in a stream of `total`, 0 for the group
// path: a power of two from 64 KiB up to 256 KiB and at most half a leaf.
uint64_t stream_piece_bytes(uint64_t leaf, uint64_t total, uint64_t read_flags) {
  if (read_flags & TCX_READ_DIRECT) return 0;  // O_DIRECT windows go through the group path
  if (const char* m = std::getenv("TCX_STAGE"); m != nullptr && std::strcmp(m, "slabs") == 0) return 0;
  const uint64_t span = std::min(leaf, total);
  uint64_t S = kMinPieceBytes;
  while (S * 2 <= kPieceBytes && S * 4 <= span) S *= 2;
  return S * 2 <= span ? S : 0;
}

tcx_status hash_file_segments_streamed(FileHashContext& r, const tcx_file_segment* segs, uint64_t n_segs,
                                       uint64_t total, uint64_t L, uint64_t S, int read_threads, int device,
                                       tcx_progress_fn progress, void* progress_ctx, uint8_t root[32]) {
  const uint64_t n_full = total / L, tail = total - n_full * L;
  const uint64_t n_leaves = n_full + (tail > 0 ? 1 : 0);
  const uint64_t J = (std::min(L, total) + S - 1) / S;  // slabs per wave
  uint64_t W = std::max<uint64_t>(1, kSlabRingBytes / (kSlabRing * S));  // leaves per wave
  if (const char* v = std::getenv("TCX_HASH_WAVE_LEAVES")) W = std::max<uint64_t>(1, std::strtoull(v, nullptr, 0));
  W = std::min<uint64_t>(W, n_leaves);
  const uint64_t n_waves = (n_leaves + W - 1) / W;
  const uint64_t k = std::max<uint64_t>(1, std::min<uint64_t>(W, kPieceCopy / S));  // leaves per copy
  const uint64_t slab_bytes = W * S;
  const int nt = read_threads > 0 ? read_threads : std::max(1, std::min(16, affinity_cpus()));
  if (tcx_status st = r.ensure_common(n_leaves * 32, std::max<uint64_t>(merkle_scratch_bytes(n_leaves), 256));
      st != TCX_OK)
    return st;
  if (tcx_status st = r.ensure_stream(nt, k * S, kSlabRing * slab_bytes, W * 32, n_waves); st != TCX_OK) return st;
  auto ctx = std::make_shared<FileStageCtx>();
  if (tcx_status st = open_stage_files(segs, n_segs, total, ctx.get()); st != TCX_OK) return st;
  // The call has no deadline of its own (the CPU path it replaces blocks until
  // its reads return); this bounds only the wait for a stuck copy.
  const auto deadline = StageClock::now() + std::chrono::hours(24);

  PieceBuffers& pb = r.pieces;
  const uint64_t Q = n_waves * J;  // slabs in stream order: wave-major
  std::vector<std::shared_ptr<ReadBatch>> batches(Q);
  auto submit = [&](uint64_t q) {
    const uint64_t w = q / J, j = q % J, w0 = w * W, ww = std::min(W, n_leaves - w0);
    uint8_t* slab = r.ring + (q % kSlabRing) * slab_bytes;
    cudaEvent_t free_ev = r.ring_free[q % kSlabRing];
    auto b = std::make_shared<ReadBatch>();
    b->n = (ww + k - 1) / k;
    b->fn = [&pb, ctx, slab, free_ev, w0, ww, j, S, L, n_full, tail, k, device, deadline](uint64_t i,
                                                                                         ReadBatch& bb) -> bool {
      const uint64_t off = j * S, r0 = i * k, r1 = std::min(ww, r0 + k);
      uint64_t used = 0;  // rows of the item up to the last one with bytes in this slab
      for (uint64_t r = r0; r < r1; ++r)
        if ((w0 + r < n_full ? L : tail) > off) used = r - r0 + 1;
      if (used == 0) return true;
      const int t = reader_for_copies(pb, device, bb);
      if (t < 0) return false;
      uint64_t slot = 0;
      uint8_t* buf = pb.acquire(t, deadline, bb, &slot);
      if (buf == nullptr) return false;
      for (uint64_t r = r0; r < r0 + used; ++r) {
        const uint64_t len = w0 + r < n_full ? L : tail;
        if (len > off && !read_stage_range(*ctx, (w0 + r) * L + off, std::min(S, len - off), buf + (r - r0) * S, bb))
          return false;
      }
      // Rows at pitch S on both sides: one copy; the bytes past a short leaf's end
      // are never read by the pass.
      cudaStream_t st = pb.streams[t];
      cudaError_t e = cudaStreamWaitEvent(st, free_ev, 0);
      if (e == cudaSuccess) e = cudaMemcpyAsync(slab + r0 * S, buf, used * S, cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) {
        cudaGetLastError();
        bb.fail(TCX_INTERNAL, "queueing the host-to-device copy of hashed pieces: " + cuda_msg(e));
        return false;
      }
      return pb.queued(t, slot, bb);
    };
    batches[q] = b;
    r.readers->submit(b);
  };

  if (progress) progress(0, total, progress_ctx);
  uint64_t reported = 0;  // waves whose digests are known to be written
  auto report_done = [&](uint64_t limit, bool wait) -> tcx_status {
    while (reported < limit) {
      const cudaError_t q = wait ? cudaEventSynchronize(r.wave_done[reported]) : cudaEventQuery(r.wave_done[reported]);
      if (q == cudaErrorNotReady) break;
      if (q != cudaSuccess) return set_error(TCX_INTERNAL, std::string("leaf hashing failed: ") + cudaGetErrorString(q));
      ++reported;
      if (progress) progress(std::min(total, reported * W * L), total, progress_ctx);
    }
    return TCX_OK;
  };

  tcx_status st = TCX_OK;
  uint64_t submitted = 0;
  for (; submitted < std::min<uint64_t>(Q, kSlabRing); ++submitted) submit(submitted);
  for (uint64_t q = 0; q < Q && st == TCX_OK; ++q) {
    const uint64_t w = q / J, j = q % J, w0 = w * W, ww = std::min(W, n_leaves - w0);
    if (!ReadPool::wait(*batches[q], deadline)) {
      st = set_error(TCX_DEADLINE_EXCEEDED, "reading the hashed files timed out");
      break;
    }
    if (batches[q]->failed) {
      std::lock_guard<std::mutex> lk(batches[q]->mu);
      st = batches[q]->code == TCX_DATA_LOSS ? set_error(TCX_DATA_LOSS, "short read while hashing source")
                                             : set_error(batches[q]->code != TCX_OK ? batches[q]->code : TCX_INTERNAL,
                                                         batches[q]->err);
      break;
    }
    if ((st = pb.join(r.s_hash)) != TCX_OK) break;
    st = launch_leaf_pass_pitched(r.ring + (q % kSlabRing) * slab_bytes, S, total - w0 * L, L,
                                  static_cast<uint32_t>(ww), j * S, S, r.states, r.digests + w0 * 32, r.s_hash);
    if (st != TCX_OK) break;
    if (cudaError_t e = cudaEventRecord(r.ring_free[q % kSlabRing], r.s_hash); e != cudaSuccess) {
      cudaGetLastError();
      st = set_error(TCX_INTERNAL, "recording a slab pass: " + cuda_msg(e));
      break;
    }
    if (j == J - 1) {
      if (cudaError_t e = cudaEventRecord(r.wave_done[w], r.s_hash); e != cudaSuccess) {
        cudaGetLastError();
        st = set_error(TCX_INTERNAL, "recording a wave: " + cuda_msg(e));
        break;
      }
    }
    // The slab buffer of q is free for slab q + kSlabRing once this pass has run;
    // its readers' copies wait for the event just recorded.
    if (submitted < Q) submit(submitted++);
    if ((st = report_done(j == J - 1 ? w + 1 : w, false)) != TCX_OK) break;
  }
  if (st != TCX_OK) {
    for (uint64_t q = 0; q < submitted; ++q) batches[q]->failed = true;
    for (uint64_t q = 0; q < submitted; ++q)
      ReadPool::wait(*batches[q], StageClock::now() + std::chrono::minutes(10));
    pb.sync();
    cudaStreamSynchronize(r.s_hash);
    cudaGetLastError();
    return st;
  }
  if ((st = launch_merkle(r.digests, n_leaves, r.scratch, r.root, r.s_hash)) != TCX_OK) return st;
  TCX_CUDA_TRY(cudaMemcpyAsync(root, r.root, 32, cudaMemcpyDeviceToHost, r.s_hash));
  TCX_CUDA_TRY(cudaStreamSynchronize(r.s_hash));
  return report_done(n_waves, true);
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" tcx_status tcx_multihash_from_file_segments(const tcx_file_segment* segs, uint64_t n_segs, uint64_t total,
                                                       uint64_t leaf_bytes, int device, uint64_t group_bytes,
                                                       int depth, int read_threads, uint64_t read_flags,
                                                       tcx_progress_fn progress,
                                                       void* progress_ctx, uint8_t* root_out, char* out,
                                                       uint64_t out_len) {
  if (total == 0) return set_error(TCX_INVALID_ARGUMENT, "total_size must be > 0");
  if (leaf_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "leaf_chunk_bytes must be > 0");
  if (leaf_bytes > 0xFFFFFFFFull) return set_error(TCX_INVALID_ARGUMENT, "leaf_chunk_bytes must fit in 32 bits");
  if (out == nullptr || out_len < 57) return set_error(TCX_INVALID_ARGUMENT, "output buffer must hold 57 bytes");
  if (segs == nullptr && n_segs > 0) return set_error(TCX_INVALID_ARGUMENT, "null segment list");
  // The segments must tile [0, total) in stream order.
  uint64_t cursor = 0;
  for (uint64_t i = 0; i < n_segs; ++i) {
    if (segs[i].path == nullptr) return set_error(TCX_INVALID_ARGUMENT, "segment without a path");
    if (segs[i].dst_offset != cursor)
      return set_errorf(TCX_INVALID_ARGUMENT, "segment %llu starts at %llu, expected %llu",
                        static_cast<unsigned long long>(i), static_cast<unsigned long long>(segs[i].dst_offset),
                        static_cast<unsigned long long>(cursor));
    cursor += segs[i].length;
  }
  if (cursor != total)
    return set_errorf(TCX_INVALID_ARGUMENT, "segments cover %llu bytes, total_size is %llu",
                      static_cast<unsigned long long>(cursor), static_cast<unsigned long long>(total));
  int n_dev = 0;
  TCX_CUDA_TRY(cudaGetDeviceCount(&n_dev));
  if (device < 0 || device >= n_dev) return set_error(TCX_INVALID_ARGUMENT, "device_id out of range");

  const uint64_t n_leaves = (total + leaf_bytes - 1) / leaf_bytes;
  if (n_leaves >= (1ull << 32)) return set_error(TCX_INVALID_ARGUMENT, "too many leaves");

  DeviceGuard guard(device);
  FileHashContext* ctx = context_for(device);
  std::lock_guard<std::mutex> lock(ctx->mu);
  uint8_t root[32];
  const uint64_t piece = stream_piece_bytes(leaf_bytes, total, read_flags);
  const tcx_status st =
      piece > 0 ? hash_file_segments_streamed(*ctx, segs, n_segs, total, leaf_bytes, piece, read_threads, device,
                                              progress, progress_ctx, root)
                : hash_file_segments(*ctx, segs, n_segs, total, leaf_bytes, group_bytes, depth, read_threads,
                                     read_flags, progress, progress_ctx, root);
  if (st != TCX_OK) {
    ctx->drain();
    return st;
  }
  if (root_out) std::memcpy(root_out, root, 32);
  encode_multihash(root, out);
  return TCX_OK;
}

extern "C" tcx_status tcx_file_hash_release(int device) {
  std::lock_guard<std::mutex> lock(g_contexts_mu);
  for (auto& [dev, ctx] : g_contexts) {
    if (device >= 0 && dev != device) continue;
    DeviceGuard guard(dev);
    std::lock_guard<std::mutex> l(ctx->mu);
    ctx->free_all();
  }
  return TCX_OK;
}
