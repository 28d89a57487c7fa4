// Collective load engine: one process (one tcx_group) per GPU.
//
// Per rank, three streams carry the pipeline of tcx_group_load:
//   copy:  pinned host -> HBM of this rank's staged range, in slabs laid across
//          all of its leaves at once (one 2-D copy per slab: width = slab,
//          pitch = leaf), so every leaf's SHA-256 chain advances as soon as a
//          slab lands instead of leaves completing one after another;
//   hash:  one streamed SHA-256 pass per slab over all leaves of the range;
//   comm:  after the last slab: zero-fill of view gaps, pack of each peer's
//          bytes, local extraction into the view, one NCCL group of
//          send/recv (personalised all-to-all over NVLink), scatter of
//          non-contiguous receives, in-place permutes; then the leaf digests
//          of all ranks (NCCL all-gather), the Merkle root and a 32-byte
//          device-to-host read.
// Reference: collective_disk_loader.cc:5538-5816 runs read -> H2D to one root
// GPU -> ncclBroadcast/ncclSend per chunk with a host synchronize after every
// chunk; verification_stage.cc:55-128 hashes the replica afterwards.
#include <cuda.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <nccl.h>
#include <sched.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cctype>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "staging.h"
#include "tcx_internal.h"

namespace tcx {
tcx_status validate_load_plan(const tcx_load_plan* plan, int world);
void clip_jobs(const tcx_copy_job* jobs, uint64_t n, uint64_t lo, uint64_t hi, std::vector<tcx_copy_job>& out);
}

namespace {

using namespace tcx;
using Clock = std::chrono::steady_clock;

// Groups alive in this process (rank threads of one process each hold one): the
// default reader count of a load splits the process's CPUs among them.
std::atomic<int> g_live_groups{0};

constexpr uint64_t kDefaultSlab = 256 * 1024;
constexpr uint64_t kDefaultWindow = 512ull << 20;  // bytes per peer per exchange round
constexpr uint64_t kDefaultSlotBytes = 512ull << 20;  // pinned bytes per slab when staging from files
constexpr uint64_t kDefaultRingSlots = 4;            // slabs read ahead when staging from files

// Piece staging from files (the pieces of a few leaves copied to the device as
// soon as they are read): bytes per leaf piece, bytes per copy, and pinned
// buffers per reader thread. It is used for leaves of at least two pieces;
// TCX_STAGE=slabs selects the slab ring instead, and TCX_STAGE_PIECE,
// TCX_STAGE_COPY and TCX_STAGE_PIECE_BUFS override the defaults. Measured on
// B200 (16 GB artifact of 4 MiB leaves, tmpfs, 16 readers): 47.4-50.7 GB/s from
// the file against 41.6-42.5 GB/s with 512 MiB slab slots, where every slab is
// written to host DRAM in full before its copy reads it back; 2 MiB or 8 MiB
// copies, 128 or 512 KiB pieces and 3 buffers per reader measured slower.
constexpr uint64_t kDefaultPieceBytes = 256ull << 10;
constexpr uint64_t kDefaultPieceCopy = 4ull << 20;
constexpr int kDefaultPieceBufs = 2;
constexpr uint64_t kMinPieceBytes = 64ull << 10;

// Piece size for leaves of `span` bytes, 0 for slab staging: a power of two,
// at most half the leaf (so that every leaf's chain advances over several slabs).
uint64_t piece_bytes_for(uint64_t span) {
  const char* mode = std::getenv("TCX_STAGE");
  if (mode != nullptr && std::strcmp(mode, "slabs") == 0) return 0;
  uint64_t want = kDefaultPieceBytes;
  if (const char* v = std::getenv("TCX_STAGE_PIECE")) want = std::strtoull(v, nullptr, 0);
  uint64_t S = kMinPieceBytes;
  while (S * 2 <= want && S * 4 <= span) S *= 2;
  return S * 2 <= span ? S : 0;
}

// Leaves per work item: about kDefaultPieceCopy bytes per host-to-device copy
// (TCX_STAGE_COPY overrides), at least one leaf and at most n_rows.
uint64_t piece_rows_for(uint64_t S, uint64_t n_rows) {
  uint64_t want = kDefaultPieceCopy;
  if (const char* v = std::getenv("TCX_STAGE_COPY")) want = std::strtoull(v, nullptr, 0);
  return std::max<uint64_t>(1, std::min<uint64_t>(n_rows, want / S));
}

int piece_buffers() {
  if (const char* v = std::getenv("TCX_STAGE_PIECE_BUFS")) return std::max(1, std::min(64, std::atoi(v)));
  return kDefaultPieceBufs;
}

// The local extraction copy of a load runs while the leaf hash is still going.
// With fewer chains than about one consumer warp per SMSP the hash is bound by
// each warp's own instruction issue, and a full 8-CTA-per-SM copy grid sharing
// those SMSPs slows every chain (measured with the same grid pushing to peers:
// the 70B TP-4 hash went from about 74 to 135 ms); a quarter of the SMs' worth
// of CTAs still copies several hundred GB/s within HBM. With more chains than
// that the hash is throughput-bound like the copy, which keeps the full grid.
// (The NCCL path's pack and scatter kernels keep the full grid: they gate the
// exchange, which is the longer leg of the 70B loads at N=2 and 4.)
// The cap applies only while the capped copy still ends inside the hash: measured
// on the Llama-3-70B TP-2 load (16.8k chains, 35 GB of local pieces per rank), the
// quarter grid moved about 220 GB/s and set the step (159 ms against a 125 ms hash),
// while the full grid finished beside the hash (step 127 ms, hash unchanged). So the
// full grid is used once the local bytes at 220 GB/s would take more than 60% of one
// chain's time (about 1 us per 64-byte block).
uint32_t load_copy_ctas(uint64_t n_chains, uint64_t local_bytes, uint64_t leaf_bytes) {
  // TCX_LOCAL_COPY_CTAS overrides the cap (0 = the full grid) for measurements.
  if (const char* v = std::getenv("TCX_LOCAL_COPY_CTAS")) return static_cast<uint32_t>(std::strtoul(v, nullptr, 10));
  const uint64_t sms = static_cast<uint64_t>(sm_count());
  if (n_chains >= sms * 128) return 0u;
  const double chain_s = static_cast<double>(leaf_bytes / 64) * 1e-6;
  const double capped_s = static_cast<double>(local_bytes) / 220e9;
  if (capped_s > 0.6 * chain_s) return 0u;
  return static_cast<uint32_t>(std::max<uint64_t>(8, sms / 4));
}

// TCX_LOCAL_COPY=ce moves this rank's own view pieces with the copy engines (one
// 2-D copy per piece) instead of the copy kernel (measurement knob).
bool local_copy_on_copy_engines() {
  const char* v = std::getenv("TCX_LOCAL_COPY");
  return v != nullptr && std::strcmp(v, "ce") == 0;
}

std::string nccl_msg(ncclResult_t r) { return std::string(ncclGetErrorString(r)); }

struct DevBuf {
  void* p = nullptr;
  uint64_t cap = 0;
  tcx_status grow(uint64_t bytes) {
    if (bytes <= cap) return TCX_OK;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    const uint64_t want = std::max<uint64_t>(bytes, 256);
    if (cudaError_t e = cudaMalloc(&p, want); e != cudaSuccess) {
      cudaGetLastError();  // reported here; keep it from later launch checks
      return set_errorf(TCX_RESOURCE_EXHAUSTED, "cudaMalloc(%llu) failed: %s",
                        static_cast<unsigned long long>(want), cuda_msg(e).c_str());
    }
    cap = want;
    return TCX_OK;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
  uint8_t* bytes() const { return static_cast<uint8_t*>(p); }
};


}  // namespace

struct tcx_group {
  std::mutex mu;  // one load at a time per group (the buffers and streams below are shared)
  int world = 1, rank = 0, device = 0;
  int64_t timeout_ms = 60000;
  ncclComm_t comm = nullptr;
  cudaStream_t s_copy = nullptr, s_hash = nullptr, s_comm = nullptr, s_pack = nullptr;
  cudaStream_t s_local = nullptr;  // this rank's own view pieces, beside the exchange (world > 1)
  cudaEvent_t ev_local = nullptr;
  cudaEvent_t ev_xfer0 = nullptr, ev_xfer1 = nullptr;  // timed: the peer transfer (pushes or NCCL rounds)
  DevBuf digests_mine, states, digests_all, digests_compact, merkle_scratch, root, send, recv, perm_scratch, jobs,
      prefix, view_digests, view_scratch;
  uint8_t* h_root = nullptr;
  tcx_copy_job* h_jobs = nullptr;
  uint64_t h_jobs_cap = 0;
  std::vector<cudaEvent_t> slab_events, packed_events, sent_events;
  cudaEvent_t ev_start = nullptr, ev_h2d = nullptr, ev_hash = nullptr, ev_exch = nullptr, ev_end = nullptr;
  // Peer view mappings for the push exchange (CUDA IPC), re-validated on every load.
  struct PeerView {
    cudaIpcMemHandle_t handle{};
    void* base = nullptr;  // allocation base, mapped into this process (or the peer's own pointer)
    uint64_t offset = 0;   // view start inside the peer's allocation
    uint64_t size = 0;     // peer's view bytes
    bool open = false;     // an opened IPC mapping (another process's memory)
    bool local = false;    // the peer is a thread of this process: its pointer is used as is
  };
  std::vector<PeerView> peer_views;
  // One stream per peer for the push copies (copy engines), so the pushes to
  // different peers run at once on different engines.
  std::vector<cudaStream_t> s_peer;
  std::vector<cudaEvent_t> peer_done;
  cudaEvent_t ev_push = nullptr;
  DevBuf ipc_records, barrier_word;
  uint8_t* h_ipc = nullptr;  // pinned, world records
  // Streamed staging from files (tcx_group_load_files): a ring of pinned slots,
  // kept between loads like the reference's pinned buffer pool, and the reader
  // threads that fill them.
  uint8_t* h_ring = nullptr;
  uint64_t h_ring_bytes = 0;
  std::unique_ptr<ReadPool> readers;
  // Piece staging: per reader thread a stream and pinned buffers for the pieces
  // of a few leaves, each with the event of the copy that last read it.
  PieceBuffers pieces;
};

namespace {

// Waits until a non-blocking communicator has no operation in progress.
tcx_status nccl_settle(tcx_group* g, Clock::time_point deadline, const char* what) {
  for (;;) {
    ncclResult_t state = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(g->comm, &state);
    if (r != ncclSuccess) return set_errorf(TCX_INTERNAL, "%s: ncclCommGetAsyncError: %s", what, nccl_msg(r).c_str());
    if (state == ncclSuccess) return TCX_OK;
    if (state != ncclInProgress) return set_errorf(TCX_INTERNAL, "%s: %s", what, nccl_msg(state).c_str());
    if (Clock::now() > deadline) {
      ncclCommAbort(g->comm);
      g->comm = nullptr;
      return set_errorf(TCX_DEADLINE_EXCEEDED, "%s: timed out waiting for peers", what);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

tcx_status nccl_check(tcx_group* g, ncclResult_t r, Clock::time_point deadline, const char* what) {
  if (r == ncclSuccess) return TCX_OK;
  if (r == ncclInProgress) return nccl_settle(g, deadline, what);
  return set_errorf(TCX_INTERNAL, "%s: %s", what, nccl_msg(r).c_str());
}

// Waits for ev with a deadline, watching the communicator for asynchronous errors.
tcx_status wait_event(tcx_group* g, cudaEvent_t ev, Clock::time_point deadline) {
  if (g->comm == nullptr) {
    TCX_CUDA_TRY(cudaEventSynchronize(ev));
    return TCX_OK;
  }
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return TCX_OK;
    if (e != cudaErrorNotReady) return set_error(TCX_INTERNAL, "load failed on the device: " + cuda_msg(e));
    ncclResult_t state = ncclSuccess;
    ncclCommGetAsyncError(g->comm, &state);
    if (state != ncclSuccess && state != ncclInProgress) {
      ncclCommAbort(g->comm);
      g->comm = nullptr;
      return set_errorf(TCX_INTERNAL, "NCCL error during load: %s", nccl_msg(state).c_str());
    }
    if (Clock::now() > deadline) {
      ncclCommAbort(g->comm);
      g->comm = nullptr;
      return set_error(TCX_DEADLINE_EXCEEDED, "collective load timed out (a peer did not take part)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

tcx_status ensure_events(std::vector<cudaEvent_t>& v, uint64_t n) {
  while (v.size() < n) {
    cudaEvent_t e;
    TCX_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    v.push_back(e);
  }
  return TCX_OK;
}

// One rank's advertisement of its view buffer for the push exchange.
struct IpcRecord {
  cudaIpcMemHandle_t handle;  // 64 bytes: the allocation holding the view
  uint64_t offset;            // view start inside that allocation
  uint64_t size;              // view bytes
  uint64_t valid;
  uint64_t process;           // token of the advertising process (same token: a thread of this process)
  uint64_t base;              // allocation base in the advertising process
  uint64_t device;            // the advertising rank's CUDA device
};
static_assert(sizeof(IpcRecord) == 112, "IPC record layout");

// A random token that tells this process apart from every other one on the node
// (ranks that are threads of one process share memory without CUDA IPC, which
// cannot open a handle exported by the same process).
uint64_t process_token() {
  static const uint64_t token = [] {
    std::random_device rd;
    uint64_t t = (static_cast<uint64_t>(rd()) << 32) ^ rd() ^ static_cast<uint64_t>(getpid());
    return t == 0 ? 1 : t;
  }();
  return token;
}

// Stream-ordered barrier: completes on every rank only after every rank's earlier
// work on its comm stream has completed.
tcx_status nccl_barrier(tcx_group* g, Clock::time_point deadline) {
  return nccl_check(g, ncclAllReduce(g->barrier_word.p, g->barrier_word.p, 1, ncclInt32, ncclSum, g->comm, g->s_comm),
                    deadline, "barrier");
}

// Exchanges view handles (NCCL all-gather of one IpcRecord per rank) and maps every
// peer's view into this process, reusing mappings whose handle has not changed.
tcx_status map_peer_views(tcx_group* g, void* d_view, uint64_t view_bytes, Clock::time_point deadline) {
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (get_range == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    TCX_CUDA_TRY(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(TCX_UNAVAILABLE, "cuMemGetAddressRange is unavailable");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  CUdeviceptr base = 0;
  size_t alloc = 0;
  if (get_range(&base, &alloc, reinterpret_cast<CUdeviceptr>(d_view)) != CUDA_SUCCESS)
    return set_error(TCX_INVALID_ARGUMENT, "d_view is not device memory this process allocated");
  const uint64_t offset = reinterpret_cast<uint64_t>(d_view) - static_cast<uint64_t>(base);
  if (offset + view_bytes > alloc) return set_error(TCX_INVALID_ARGUMENT, "view exceeds its allocation");
  IpcRecord mine{};
  TCX_CUDA_TRY(cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void*>(base)));
  mine.offset = offset;
  mine.size = view_bytes;
  mine.valid = 1;
  mine.process = process_token();
  mine.base = static_cast<uint64_t>(base);
  mine.device = static_cast<uint64_t>(g->device);
  const uint64_t rec = sizeof(IpcRecord), world = static_cast<uint64_t>(g->world);
  tcx_status st;
  if ((st = g->ipc_records.grow((world + 1) * rec)) != TCX_OK) return st;
  if (g->h_ipc == nullptr) TCX_CUDA_TRY(cudaMallocHost(&g->h_ipc, (world + 1) * rec));
  std::memcpy(g->h_ipc + world * rec, &mine, rec);
  TCX_CUDA_TRY(cudaMemcpyAsync(g->ipc_records.bytes() + world * rec, g->h_ipc + world * rec, rec,
                               cudaMemcpyHostToDevice, g->s_comm));
  st = nccl_check(g, ncclAllGather(g->ipc_records.bytes() + world * rec, g->ipc_records.p, rec, ncclUint8, g->comm,
                                   g->s_comm), deadline, "view handle exchange");
  if (st != TCX_OK) return st;
  TCX_CUDA_TRY(cudaMemcpyAsync(g->h_ipc, g->ipc_records.p, world * rec, cudaMemcpyDeviceToHost, g->s_comm));
  TCX_CUDA_TRY(cudaEventRecord(g->ev_exch, g->s_comm));
  if ((st = wait_event(g, g->ev_exch, deadline)) != TCX_OK) return st;
  g->peer_views.resize(world);
  for (int p = 0; p < g->world; ++p) {
    if (p == g->rank) continue;
    IpcRecord r;
    std::memcpy(&r, g->h_ipc + static_cast<uint64_t>(p) * rec, rec);
    if (!r.valid) return set_errorf(TCX_INTERNAL, "rank %d sent no view handle", p);
    auto& pv = g->peer_views[p];
    if (r.process == mine.process) {
      // A thread of this process: write through its own pointer (unified addressing)
      // once this device may access the peer's.
      if (pv.open) cudaIpcCloseMemHandle(pv.base);
      pv.open = false;
      if (!pv.local || pv.base != reinterpret_cast<void*>(r.base)) {
        const int peer_dev = static_cast<int>(r.device);
        if (peer_dev != g->device) {
          int can = 0;
          TCX_CUDA_TRY(cudaDeviceCanAccessPeer(&can, g->device, peer_dev));
          if (can) {
            const cudaError_t e = cudaDeviceEnablePeerAccess(peer_dev, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
              return set_errorf(TCX_INTERNAL, "cudaDeviceEnablePeerAccess(%d): %s", peer_dev, cuda_msg(e).c_str());
            cudaGetLastError();
          }
        }
        pv.base = reinterpret_cast<void*>(r.base);
        pv.local = true;
      }
    } else if (!pv.open || std::memcmp(&pv.handle, &r.handle, sizeof r.handle) != 0) {
      if (pv.open) cudaIpcCloseMemHandle(pv.base);
      pv.open = false;
      pv.local = false;
      TCX_CUDA_TRY(cudaIpcOpenMemHandle(&pv.base, r.handle, cudaIpcMemLazyEnablePeerAccess));
      pv.handle = r.handle;
      pv.open = true;
    }
    pv.offset = r.offset;
    pv.size = r.size;
  }
  return TCX_OK;
}

tcx_copy_job swap_ends(tcx_copy_job j) {
  std::swap(j.src_off, j.dst_off);
  std::swap(j.src_pitch, j.dst_pitch);
  return j;
}

// Every byte this rank's jobs and permutes write lies inside its view and, for a
// load into separate target tensors, inside one of the targets.
tcx_status check_destinations(const tcx_load_plan* plan, int rank) {
  const bool targets = (plan->flags & TCX_LOAD_TARGETS) != 0;
  std::vector<std::pair<uint64_t, uint64_t>> t;
  if (targets) {
    if (plan->flags & (TCX_LOAD_VIEW_HASH | TCX_LOAD_PEER_PUSH))
      return set_error(TCX_INVALID_ARGUMENT, "a load into target tensors takes neither the view hash nor peer push");
    if (plan->n_targets == 0 || plan->target_ranges == nullptr)
      return set_error(TCX_INVALID_ARGUMENT, "TCX_LOAD_TARGETS needs target_ranges");
    for (uint64_t i = 0; i < plan->n_targets; ++i)
      t.emplace_back(plan->target_ranges[2 * i], plan->target_ranges[2 * i + 1]);
    std::sort(t.begin(), t.end());
    for (size_t i = 0; i < t.size(); ++i) {
      if (t[i].first + t[i].second > plan->view_bytes || t[i].first + t[i].second < t[i].first)
        return set_error(TCX_INVALID_ARGUMENT, "a target range exceeds view_bytes");
      if (i > 0 && t[i].first < t[i - 1].first + t[i - 1].second)
        return set_error(TCX_INVALID_ARGUMENT, "target ranges overlap");
    }
  }
  auto inside = [&](uint64_t a, uint64_t e) {
    if (e < a || e > plan->view_bytes) return false;
    if (!targets) return true;
    auto it = std::upper_bound(t.begin(), t.end(), std::make_pair(a, ~uint64_t{0}));
    if (it == t.begin()) return false;
    --it;
    return e <= it->first + it->second;
  };
  for (uint64_t i = plan->job_offsets[rank]; i < plan->job_offsets[rank + 1]; ++i) {
    const tcx_copy_job& j = plan->jobs[i];
    if (j.rows == 0 || j.row_bytes == 0) continue;
    const uint64_t e = j.dst_off + (j.rows - 1) * (j.rows > 1 ? j.dst_pitch : 0) + j.row_bytes;
    if (!inside(j.dst_off, e))
      return set_errorf(TCX_INVALID_ARGUMENT, "job %llu writes outside %s", static_cast<unsigned long long>(i),
                        targets ? "its target" : "the view");
  }
  for (uint64_t i = 0; i < plan->n_permutes; ++i) {
    const tcx_permute_job& pj = plan->permutes[i];
    if (pj.ndim == 0 || pj.ndim > TCX_MAX_DIMS) continue;  // rejected by check_permute
    uint64_t bytes = pj.esize;
    for (uint32_t d = 0; d < pj.ndim; ++d) bytes *= static_cast<uint64_t>(pj.shape[d] < 0 ? 0 : pj.shape[d]);
    if (bytes && !inside(pj.dst_off, pj.dst_off + bytes))
      return set_errorf(TCX_INVALID_ARGUMENT, "permute %llu lies outside %s", static_cast<unsigned long long>(i),
                        targets ? "one target" : "the view");
  }
  return TCX_OK;
}

float elapsed_ms(cudaEvent_t a, cudaEvent_t b) {
  float ms = 0;
  if (cudaEventElapsedTime(&ms, a, b) != cudaSuccess) return -1.f;
  return ms;
}

}  // namespace

extern "C" tcx_status tcx_group_unique_id(uint8_t* out128) {
  if (out128 == nullptr) return set_error(TCX_INVALID_ARGUMENT, "out is null");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_errorf(TCX_INTERNAL, "ncclGetUniqueId: %s", nccl_msg(r).c_str());
  static_assert(sizeof(id) == TCX_UNIQUE_ID_BYTES, "NCCL unique id size");
  std::memcpy(out128, &id, sizeof id);
  return TCX_OK;
}

extern "C" tcx_status tcx_group_create(const uint8_t* unique_id, int world, int rank, int device, int64_t timeout_ms,
                                       tcx_group** out) {
  if (out == nullptr) return set_error(TCX_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return set_error(TCX_INVALID_ARGUMENT, "rank/world out of range");
  if (world > 1 && unique_id == nullptr) return set_error(TCX_INVALID_ARGUMENT, "unique_id is required for world > 1");
  if (cudaError_t e = cudaSetDevice(device); e != cudaSuccess)
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: %s", device, cuda_msg(e).c_str());
  auto* g = new tcx_group();
  g_live_groups.fetch_add(1);
  g->world = world;
  g->rank = rank;
  g->device = device;
  g->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  auto fail = [&](tcx_status st) {
    tcx_group_destroy(g);
    return st;
  };
  if (cudaStreamCreateWithFlags(&g->s_copy, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&g->s_hash, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&g->s_comm, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&g->s_pack, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&g->s_local, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&g->ev_local, cudaEventDisableTiming) != cudaSuccess)
    return fail(set_error(TCX_INTERNAL, "stream creation failed"));
  for (cudaEvent_t* ev : {&g->ev_start, &g->ev_h2d, &g->ev_hash, &g->ev_exch, &g->ev_end, &g->ev_xfer0, &g->ev_xfer1})
    if (cudaEventCreate(ev) != cudaSuccess) return fail(set_error(TCX_INTERNAL, "event creation failed"));
  if (cudaMallocHost(&g->h_root, 256) != cudaSuccess) return fail(set_error(TCX_INTERNAL, "pinned alloc failed"));
  if (world > 1) {
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    const auto deadline = Clock::now() + std::chrono::milliseconds(g->timeout_ms);
    ncclResult_t r = ncclCommInitRankConfig(&g->comm, world, id, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress)
      return fail(set_errorf(TCX_INTERNAL, "ncclCommInitRankConfig: %s", nccl_msg(r).c_str()));
    tcx_status st = nccl_settle(g, deadline, "communicator init");
    if (st != TCX_OK) return fail(st);
  }
  *out = g;
  return TCX_OK;
}

namespace {
// In-process rendezvous of tcx_group_join: the first rank thread of a group id
// creates the NCCL unique id, the others take it; an entry lives until every rank
// has taken it or its deadline passes (a later join of the same id then starts a
// new generation).
struct JoinEntry {
  uint8_t uid[TCX_UNIQUE_ID_BYTES];
  int world = 0;
  std::vector<bool> taken;
  int n_taken = 0;
  Clock::time_point expires;
};
std::mutex g_join_mu;
std::map<std::string, JoinEntry> g_joins;
}  // namespace

extern "C" tcx_status tcx_group_join(const char* group_id, int world, int rank, int device, int64_t timeout_ms,
                                     tcx_group** out) {
  if (out == nullptr) return set_error(TCX_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (group_id == nullptr) return set_error(TCX_INVALID_ARGUMENT, "group_id is null");
  if (world < 1 || rank < 0 || rank >= world) return set_error(TCX_INVALID_ARGUMENT, "rank/world out of range");
  if (world == 1) return tcx_group_create(nullptr, 1, 0, device, timeout_ms, out);
  uint8_t uid[TCX_UNIQUE_ID_BYTES];
  {
    std::lock_guard<std::mutex> lk(g_join_mu);
    const auto now = Clock::now();
    auto it = g_joins.find(group_id);
    if (it != g_joins.end() && now > it->second.expires) {
      g_joins.erase(it);
      it = g_joins.end();
    }
    if (it == g_joins.end()) {
      JoinEntry e;
      tcx_status st = tcx_group_unique_id(e.uid);
      if (st != TCX_OK) return st;
      e.world = world;
      e.taken.assign(world, false);
      e.expires = now + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 60000);
      it = g_joins.emplace(group_id, std::move(e)).first;
    }
    JoinEntry& e = it->second;
    if (e.world != world)
      return set_errorf(TCX_INVALID_ARGUMENT, "group %s is being joined with world sizes %d and %d", group_id,
                        e.world, world);
    if (e.taken[rank]) return set_errorf(TCX_INVALID_ARGUMENT, "rank %d of group %s joined twice", rank, group_id);
    e.taken[rank] = true;
    std::memcpy(uid, e.uid, sizeof uid);
    if (++e.n_taken == world) g_joins.erase(it);
  }
  return tcx_group_create(uid, world, rank, device, timeout_ms, out);
}

extern "C" tcx_status tcx_group_destroy(tcx_group* g) {
  if (g == nullptr) return TCX_OK;
  cudaSetDevice(g->device);
  for (cudaStream_t s : {g->s_copy, g->s_hash, g->s_comm, g->s_pack, g->s_local})
    if (s) cudaStreamSynchronize(s);
  if (g->comm) {
    ncclCommFinalize(g->comm);
    const auto deadline = Clock::now() + std::chrono::milliseconds(g->timeout_ms);
    if (nccl_settle(g, deadline, "communicator finalize") == TCX_OK && g->comm) ncclCommDestroy(g->comm);
    g->comm = nullptr;
  }
  for (DevBuf* b : {&g->digests_mine, &g->states, &g->digests_all, &g->digests_compact, &g->merkle_scratch, &g->root,
                    &g->send, &g->recv, &g->perm_scratch, &g->jobs, &g->prefix, &g->view_digests, &g->view_scratch})
    b->release();
  for (cudaStream_t s : g->s_peer)
    if (s) cudaStreamSynchronize(s);
  for (auto& pv : g->peer_views)
    if (pv.open && !pv.local) cudaIpcCloseMemHandle(pv.base);
  g->peer_views.clear();
  for (cudaEvent_t e : g->peer_done)
    if (e) cudaEventDestroy(e);
  if (g->ev_push) cudaEventDestroy(g->ev_push);
  for (cudaStream_t s : g->s_peer)
    if (s) cudaStreamDestroy(s);
  g->readers.reset();  // joins the reader threads before their buffers go away
  g->pieces.release();
  if (g->h_ring) cudaFreeHost(g->h_ring);
  g->ipc_records.release();
  g->barrier_word.release();
  if (g->h_ipc) cudaFreeHost(g->h_ipc);
  if (g->h_root) cudaFreeHost(g->h_root);
  if (g->h_jobs) cudaFreeHost(g->h_jobs);
  for (auto* v : {&g->slab_events, &g->packed_events, &g->sent_events})
    for (cudaEvent_t e : *v) cudaEventDestroy(e);
  for (cudaEvent_t e : {g->ev_start, g->ev_h2d, g->ev_hash, g->ev_exch, g->ev_end, g->ev_xfer0, g->ev_xfer1})
    if (e) cudaEventDestroy(e);
  if (g->ev_local) cudaEventDestroy(g->ev_local);
  for (cudaStream_t s : {g->s_copy, g->s_hash, g->s_comm, g->s_pack, g->s_local})
    if (s) cudaStreamDestroy(s);
  delete g;
  g_live_groups.fetch_sub(1);
  return TCX_OK;
}

namespace {

// The group's reader pool with nt threads (kept between loads).
void ensure_readers(tcx_group* g, int nt) {
  if (!g->readers || g->readers->size() != nt) {
    g->readers.reset();
    g->readers = std::make_unique<ReadPool>(nt);
  }
}

// fs.read_threads, or this process's CPUs shared among its live groups (2 to 32).
int reader_count(const tcx_file_stage& fs) {
  if (fs.read_threads > 0) return fs.read_threads;
  return std::max(2, std::min(32, affinity_cpus() / std::max(1, g_live_groups.load())));
}

template <class Enqueue>
tcx_status stage_from_files(tcx_group* g, const tcx_file_stage& fs, uint64_t mine, uint64_t L, uint64_t S, uint64_t J,
                            uint64_t n_full, uint64_t tail, Enqueue&& enqueue_slab, Clock::time_point deadline) {
  auto ctx = std::make_shared<FileStageCtx>();
  if (tcx_status st = open_stage_files(fs.segments, fs.n_segments, mine, ctx.get()); st != TCX_OK) return st;

  const uint64_t n_rows = n_full + (tail > 0 ? 1 : 0);
  const uint64_t slot = n_rows * S;
  const uint64_t K = std::min<uint64_t>(J, fs.ring_slots > 0 ? static_cast<uint64_t>(fs.ring_slots) : kDefaultRingSlots);
  if (g->h_ring_bytes < K * slot) {
    if (g->h_ring) cudaFreeHost(g->h_ring);
    g->h_ring = nullptr;
    g->h_ring_bytes = 0;
    if (cudaError_t e = cudaHostAlloc(&g->h_ring, K * slot, cudaHostAllocPortable); e != cudaSuccess) {
      cudaGetLastError();
      return set_errorf(TCX_RESOURCE_EXHAUSTED, "pinned staging ring of %llu bytes: %s",
                        static_cast<unsigned long long>(K * slot), cuda_msg(e).c_str());
    }
    g->h_ring_bytes = K * slot;
  }
  ensure_readers(g, reader_count(fs));

  std::vector<std::shared_ptr<ReadBatch>> batches(J);
  uint64_t dispatched = 0;
  tcx_status st = TCX_OK;
  for (uint64_t j = 0; j < J && st == TCX_OK; ++j) {
    while (dispatched < J && dispatched < j + K) {
      if (dispatched >= K && (st = wait_event(g, g->slab_events[dispatched - K], deadline)) != TCX_OK) break;
      auto b = std::make_shared<ReadBatch>();
      const uint64_t jj = dispatched, off = jj * S;
      uint8_t* dst = g->h_ring + (jj % K) * slot;
      b->n = n_rows;
      b->fn = [ctx, jj, off, dst, S, L, n_full, tail](uint64_t r, ReadBatch& bb) {
        (void)jj;
        if (r < n_full) return read_stage_range(*ctx, r * L + off, std::min(S, L - off), dst + r * S, bb);
        if (tail <= off) return true;
        return read_stage_range(*ctx, n_full * L + off, std::min(S, tail - off), dst + r * S, bb);
      };
      batches[jj] = b;
      g->readers->submit(b);
      ++dispatched;
    }
    if (st != TCX_OK) break;
    if (!ReadPool::wait(*batches[j], deadline)) {
      st = set_error(TCX_DEADLINE_EXCEEDED, "reading the staged range from files timed out");
      break;
    }
    if (batches[j]->failed) {
      std::lock_guard<std::mutex> lk(batches[j]->mu);
      st = set_error(batches[j]->code != TCX_OK ? batches[j]->code : TCX_INTERNAL, batches[j]->err);
      break;
    }
    uint8_t* src = g->h_ring + (j % K) * slot;
    st = enqueue_slab(j, src, S, src + n_full * S);
  }
  if (st != TCX_OK) {
    // Nothing of this load may still write into the ring once the call returns:
    // skip what is not started and wait for reads in progress and queued copies.
    for (uint64_t k = 0; k < dispatched; ++k) batches[k]->failed = true;
    for (uint64_t k = 0; k < dispatched; ++k)
      ReadPool::wait(*batches[k], Clock::now() + std::chrono::milliseconds(g->timeout_ms));
    cudaStreamSynchronize(g->s_copy);
    cudaGetLastError();
  }
  return st;
}

// Streams this rank's staged range from files in leaf pieces: piece (r, j) is
// bytes [j*S, (j+1)*S) of leaf r, and a work item is the pieces of `k`
// consecutive leaves in slab j. A reader thread preads an item's pieces into one
// of its own pinned buffers (k*S bytes) and at once queues one 2-D host-to-device
// copy of them on its own stream, so copies of a few MiB follow the reads within
// microseconds and the data crosses host memory while it is still cache-warm; a
// thread reuses a buffer only after the copy that last read it is done, so no
// reader runs more than `bufs` items ahead of its copies. Slab j is complete once
// every reader has queued its items of it: s_copy then waits for all readers'
// streams, and on_slab(j) queues the slab's hash pass.
template <class OnSlab>
tcx_status stage_pieces_from_files(tcx_group* g, const tcx_file_stage& fs, uint8_t* stage, uint64_t mine, uint64_t L,
                                   uint64_t S, uint64_t J, uint64_t n_full, uint64_t tail, uint64_t k, int bufs,
                                   OnSlab&& on_slab, Clock::time_point deadline) {
  auto ctx = std::make_shared<FileStageCtx>();
  if (tcx_status st = open_stage_files(fs.segments, fs.n_segments, mine, ctx.get()); st != TCX_OK) return st;
  const int nt = reader_count(fs);
  ensure_readers(g, nt);
  PieceBuffers& pb = g->pieces;
  if (tcx_status st = pb.ensure(nt, k * S, bufs); st != TCX_OK) return st;
  // The copies into the staged buffer wait for the caller's earlier work on it.
  if (tcx_status st = pb.wait_on(g->ev_start); st != TCX_OK) return st;

  const uint64_t n_rows = n_full + (tail > 0 ? 1 : 0);
  const uint64_t n_items = (n_rows + k - 1) / k;
  const int device = g->device;
  std::vector<std::shared_ptr<ReadBatch>> batches(J);
  for (uint64_t j = 0; j < J; ++j) {
    auto b = std::make_shared<ReadBatch>();
    b->n = n_items;
    b->fn = [&pb, ctx, stage, j, S, L, n_full, n_rows, tail, k, device, deadline](uint64_t i, ReadBatch& bb) -> bool {
      const uint64_t off = j * S, r0 = i * k, r1 = std::min(r0 + k, n_rows);
      const uint64_t full1 = std::min(r1, n_full);  // full leaves of the item: [r0, full1)
      const bool full_part = r0 < full1 && off < L;
      const bool tail_part = r1 > n_full && tail > off;  // the short last leaf is in the item
      if (!full_part && !tail_part) return true;
      const int t = reader_for_copies(pb, device, bb);
      if (t < 0) return false;
      uint64_t slot = 0;
      uint8_t* buf = pb.acquire(t, deadline, bb, &slot);
      if (buf == nullptr) return false;
      const uint64_t w = full_part ? std::min(S, L - off) : 0;
      const uint64_t wt = tail_part ? std::min(S, tail - off) : 0;
      for (uint64_t r = r0; r < full1 && full_part; ++r)
        if (!read_stage_range(*ctx, r * L + off, w, buf + (r - r0) * S, bb)) return false;
      if (tail_part && !read_stage_range(*ctx, n_full * L + off, wt, buf + (n_full - r0) * S, bb)) return false;
      cudaStream_t s = pb.streams[t];
      cudaError_t e = cudaSuccess;
      if (full_part)
        e = full1 - r0 == 1 ? cudaMemcpyAsync(stage + r0 * L + off, buf, w, cudaMemcpyHostToDevice, s)
                            : cudaMemcpy2DAsync(stage + r0 * L + off, L, buf, S, w, full1 - r0, cudaMemcpyHostToDevice, s);
      if (e == cudaSuccess && tail_part)
        e = cudaMemcpyAsync(stage + n_full * L + off, buf + (n_full - r0) * S, wt, cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) {
        cudaGetLastError();
        bb.fail(TCX_INTERNAL, "queueing the host-to-device copy of staged pieces: " + cuda_msg(e));
        return false;
      }
      return pb.queued(t, slot, bb);
    };
    batches[j] = b;
    g->readers->submit(b);
  }
  tcx_status st = TCX_OK;
  for (uint64_t j = 0; j < J && st == TCX_OK; ++j) {
    if (!ReadPool::wait(*batches[j], deadline)) {
      st = set_error(TCX_DEADLINE_EXCEEDED, "reading the staged range from files timed out");
      break;
    }
    if (batches[j]->failed) {
      std::lock_guard<std::mutex> lk(batches[j]->mu);
      st = set_error(batches[j]->code != TCX_OK ? batches[j]->code : TCX_INTERNAL, batches[j]->err);
      break;
    }
    st = pb.join(g->s_copy);
    if (st == TCX_OK) st = on_slab(j);
  }
  if (st != TCX_OK) {
    // Nothing of this load may still write into the piece buffers or the staged
    // buffer once the call returns: skip what is not started, wait for reads in
    // progress and for every queued copy.
    for (auto& b : batches) b->failed = true;
    for (auto& b : batches) ReadPool::wait(*b, Clock::now() + std::chrono::milliseconds(g->timeout_ms));
    pb.sync();
    cudaStreamSynchronize(g->s_copy);
    cudaGetLastError();
  }
  return st;
}

tcx_status group_load(tcx_group* g, const tcx_load_plan* plan, const void* h_stage, const tcx_file_stage* files,
                      void* d_stage, void* d_view, const uint8_t* expected_root, tcx_load_result* out, void* stream) {
  if (g == nullptr) return set_error(TCX_INVALID_ARGUMENT, "group is null");
  std::lock_guard<std::mutex> lock(g->mu);
  if (g->world > 1 && g->comm == nullptr)
    return set_error(TCX_FAILED_PRECONDITION, "group communicator was aborted by an earlier failure");
  tcx_status st = validate_load_plan(plan, g->world);
  if (st != TCX_OK) return st;
  if (d_stage == nullptr || d_view == nullptr || out == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "d_stage, d_view and out are required");
  if ((st = check_destinations(plan, g->rank)) != TCX_OK) return st;
  TCX_CUDA_TRY(cudaSetDevice(g->device));
  const int world = g->world, rank = g->rank;
  const uint64_t* b = plan->stage_bounds;
  const uint64_t L = plan->leaf_bytes, T = plan->total_bytes;
  const uint64_t lo = b[rank], hi = b[rank + 1], mine = hi - lo;
  auto n_of = [&](int r) { return (b[r + 1] - b[r] + L - 1) / L; };
  const uint64_t n_mine = n_of(rank);
  uint64_t max_n = 0;
  for (int r = 0; r < world; ++r) max_n = std::max(max_n, n_of(r));
  const uint64_t n_total = (T + L - 1) / L;
  if (n_total > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");

  // --- host planning ------------------------------------------------------
  const uint64_t cap = tcx_plan_exchange_capacity(plan, world);
  std::vector<tcx_copy_job> pack(cap), local(cap), scatter(cap);
  std::vector<uint64_t> send_off(world + 1), recv_off(world + 1), recv_counts(world), recv_view(world), gaps(2 * cap);
  std::vector<uint8_t> direct(world);
  tcx_exchange_plan xp{pack.data(), 0, local.data(), 0, scatter.data(), 0, send_off.data(), recv_off.data(),
                       recv_counts.data(), recv_view.data(), direct.data(), gaps.data(), 0};
  st = tcx_plan_exchange(plan, world, rank, &xp);
  if (st != TCX_OK) return st;
  // A view buffer may alias the staged buffer only for a one-rank load whose
  // local copies are all in place (an identity view): nothing is then copied,
  // and gap zero-fill waits for the hash passes that read the same bytes.
  const auto* vb = static_cast<const uint8_t*>(d_view);
  const auto* sb = static_cast<const uint8_t*>(d_stage);
  bool alias = vb < sb + std::max<uint64_t>(mine, 1) && sb < vb + std::max<uint64_t>(plan->view_bytes, 1);
  if (plan->flags & TCX_LOAD_TARGETS) {  // only the targets themselves belong to the view
    alias = false;
    for (uint64_t i = 0; i < plan->n_targets; ++i) {
      const uint8_t* t0 = vb + plan->target_ranges[2 * i];
      const uint64_t tl = std::max<uint64_t>(plan->target_ranges[2 * i + 1], 1);
      alias = alias || (t0 < sb + std::max<uint64_t>(mine, 1) && sb < t0 + tl);
    }
  }
  std::vector<tcx_copy_job> local_kept;
  for (uint64_t i = 0; i < xp.n_local; ++i) {
    const tcx_copy_job& j = local[i];
    const bool in_place = d_view == d_stage && j.src_off == j.dst_off && (j.rows == 1 || j.src_pitch == j.dst_pitch);
    if (!in_place) local_kept.push_back(j);
  }
  if (alias && (world > 1 || !local_kept.empty() || d_view != d_stage))
    return set_error(TCX_INVALID_ARGUMENT, "d_view may alias d_stage only for a one-rank identity view");
  std::vector<tcx_copy_job> compact;
  if (world > 1) {
    for (int r = 0; r < world; ++r) {
      const uint64_t nr = n_of(r);
      if (nr == 0) continue;
      compact.push_back({static_cast<uint64_t>(r) * max_n * 32, (b[r] / L) * 32, nr * 32, nr * 32, nr * 32, 1});
    }
  }
  uint64_t perm_bytes = 0;
  for (uint64_t i = 0; i < plan->n_permutes; ++i) {
    const tcx_permute_job& pj = plan->permutes[i];
    st = check_permute(pj);
    if (st != TCX_OK) return st;
    if (pj.src_off != pj.dst_off) return set_error(TCX_INVALID_ARGUMENT, "load permutes are in place (src_off == dst_off)");
    uint64_t bytes = pj.esize;
    for (uint32_t d = 0; d < pj.ndim; ++d) bytes *= static_cast<uint64_t>(pj.shape[d]);
    if (pj.dst_off + bytes > plan->view_bytes) return set_error(TCX_INVALID_ARGUMENT, "permute outside the view");
    perm_bytes = std::max(perm_bytes, bytes);
  }

  // --- push / NCCL split ----------------------------------------------------
  // With the push exchange, a share of every (sender, receiver) pair's pieces
  // (plan->push_nccl_permille of its bytes, whole pieces in view order) can go
  // over NCCL send/recv while the rest is copied by the copy engines: the copy
  // engines of a GPU top out near 390 GB/s in an all-to-all among 4 GPUs, and
  // NCCL's SM-driven transfer adds its own bandwidth beside them. Every rank
  // derives the same split from the same plan; the NCCL part is planned as a
  // load of only those pieces.
  const bool push = world > 1 && (plan->flags & TCX_LOAD_PEER_PUSH) != 0;
  const uint64_t nccl_share = push ? std::min<uint64_t>(plan->push_nccl_permille, 1000) : 0;
  const std::vector<uint64_t> recv_counts_all(recv_counts.begin(), recv_counts.end());
  std::vector<tcx_copy_job> ce_jobs;  // hybrid: this rank's copy-engine pieces, grouped by receiver
  std::vector<uint64_t> ce_off(world + 1, 0);
  std::vector<tcx_copy_job> nccl_jobs;
  std::vector<uint64_t> nccl_job_off(world + 1, 0);
  if (nccl_share > 0) {
    const uint64_t scap = tcx_plan_push_split_capacity(plan, world);
    nccl_jobs.resize(scap);
    ce_jobs.resize(scap);
    if ((st = tcx_plan_push_split(plan, world, rank, nccl_share, nccl_jobs.data(), nccl_job_off.data(), ce_jobs.data(),
                                  ce_off.data(), scap)) != TCX_OK)
      return st;
    nccl_jobs.resize(nccl_job_off[world]);
    ce_jobs.resize(ce_off[world]);
    tcx_load_plan nplan = *plan;
    nplan.jobs = nccl_jobs.data();
    nplan.job_offsets = nccl_job_off.data();
    nplan.permutes = nullptr;
    nplan.n_permutes = 0;
    nplan.flags = 0;
    const uint64_t ncap = tcx_plan_exchange_capacity(&nplan, world);
    std::vector<tcx_copy_job> npack(ncap), nlocal(ncap), nscatter(ncap);
    std::vector<uint64_t> nsend(world + 1), nrecv_off(world + 1), nrecv_counts(world), nrecv_view(world), ngaps(2 * ncap);
    std::vector<uint8_t> ndirect(world);
    tcx_exchange_plan nxp{npack.data(), 0, nlocal.data(), 0, nscatter.data(), 0, nsend.data(), nrecv_off.data(),
                          nrecv_counts.data(), nrecv_view.data(), ndirect.data(), ngaps.data(), 0};
    if ((st = tcx_plan_exchange(&nplan, world, rank, &nxp)) != TCX_OK) return st;
    // The NCCL rounds below are built from the split's plan; this rank's own
    // pieces and the view's gaps stay those of the full plan.
    pack.swap(npack);
    scatter.swap(nscatter);
    send_off.swap(nsend);
    recv_off.swap(nrecv_off);
    recv_counts.swap(nrecv_counts);
    recv_view.swap(nrecv_view);
    direct.swap(ndirect);
    xp.n_pack = nxp.n_pack;
    xp.n_scatter = nxp.n_scatter;
  }

  // --- exchange rounds ------------------------------------------------------
  // Each (sender, receiver) pair's bytes form one stream of send_off/recv_counts
  // bytes, moved in rounds of at most W bytes. Both sides cut the stream at the
  // same offsets, so round k of a pair is in round k on both ranks.
  uint64_t W = plan->window_bytes ? plan->window_bytes : kDefaultWindow;
  W = std::max<uint64_t>(256, W - W % 256);
  std::vector<int> peers;
  for (int p = 0; p < world; ++p)
    if (p != rank) peers.push_back(p);
  uint64_t rounds = 0, max_send = 0, max_recv_buf = 0;
  for (int p : peers) {
    const uint64_t sp = send_off[p + 1] - send_off[p];
    rounds = std::max(rounds, (sp + W - 1) / W);
    rounds = std::max(rounds, (recv_counts[p] + W - 1) / W);
    max_send = std::max(max_send, sp);
    if (!direct[p]) max_recv_buf = std::max(max_recv_buf, recv_counts[p]);
  }
  const uint64_t send_slot = std::min(W, std::max<uint64_t>(max_send, 1));
  const uint64_t recv_slot = std::min(W, std::max<uint64_t>(max_recv_buf, 1));
  std::vector<uint64_t> pack_off(rounds + 1, 0), scat_off(rounds + 1, 0);
  std::vector<tcx_copy_job> round_pack, round_scatter, tmp;
  for (uint64_t k = 0; k < rounds; ++k) {
    const uint64_t buf = k % 2;
    for (size_t si = 0; si < peers.size(); ++si) {
      const int p = peers[si];
      const uint64_t sp = send_off[p + 1] - send_off[p];
      if (k * W < sp) {
        const uint64_t lo_w = send_off[p] + k * W, hi_w = send_off[p] + std::min(sp, (k + 1) * W);
        tmp.clear();
        for (uint64_t i = 0; i < xp.n_pack; ++i) {
          if (pack[i].dst_off >= hi_w || pack[i].dst_off + pack[i].rows * pack[i].row_bytes <= lo_w) continue;
          const tcx_copy_job sw = swap_ends(pack[i]);
          clip_jobs(&sw, 1, lo_w, hi_w, tmp);
        }
        for (auto& j : tmp) {
          tcx_copy_job r = swap_ends(j);
          r.dst_off = r.dst_off - lo_w + (buf * peers.size() + si) * send_slot;
          round_pack.push_back(r);
        }
      }
      if (!direct[p] && k * W < recv_counts[p]) {
        const uint64_t lo_w = recv_off[p] + k * W, hi_w = recv_off[p] + std::min(recv_counts[p], (k + 1) * W);
        tmp.clear();
        clip_jobs(scatter.data(), xp.n_scatter, lo_w, hi_w, tmp);
        for (auto& j : tmp) {
          j.src_off = j.src_off - lo_w + (buf * peers.size() + si) * recv_slot;
          round_scatter.push_back(j);
        }
      }
    }
    pack_off[k + 1] = round_pack.size();
    scat_off[k + 1] = round_scatter.size();
  }

  // Push exchange: this rank copies each peer's view pieces from its staged range
  // straight into the peer's view over NVLink (no pack or receive buffers).
  std::vector<tcx_copy_job> push_jobs;
  std::vector<uint64_t> push_off(world + 1, 0);
  uint64_t push_bytes = 0;
  if (push && nccl_share > 0) {
    push_jobs = ce_jobs;
    push_off = ce_off;
    for (const auto& j : push_jobs) push_bytes += j.rows * j.row_bytes;
  } else if (push) {
    rounds = 0;
    round_pack.clear();
    round_scatter.clear();
    std::fill(pack_off.begin(), pack_off.end(), 0);
    std::fill(scat_off.begin(), scat_off.end(), 0);
    for (int p = 0; p < world; ++p) {
      push_off[p] = push_jobs.size();
      if (p == rank) continue;
      tmp.clear();
      clip_jobs(plan->jobs + plan->job_offsets[p], plan->job_offsets[p + 1] - plan->job_offsets[p], lo, hi, tmp);
      for (auto j : tmp) {
        j.src_off -= lo;
        push_bytes += j.rows * j.row_bytes;
        push_jobs.push_back(j);
      }
    }
    push_off[world] = push_jobs.size();
  }

  // Windowed all-gather exchange: round k broadcasts every rank's staged bytes
  // [b[r] + k*W, b[r] + (k+1)*W) to all ranks (one ncclBroadcast per root in a
  // group, the root's own range in place), and each rank copies its view pieces
  // out of every peer's window. Every rank receives every byte (T·(N-1)/N per
  // rank instead of only its view's bytes).
  const bool gather_all = world > 1 && (plan->flags & TCX_LOAD_ALLGATHER) != 0;
  if (gather_all && push) return set_error(TCX_INVALID_ARGUMENT, "TCX_LOAD_ALLGATHER and TCX_LOAD_PEER_PUSH exclude each other");
  uint64_t ag_rounds = 0, ag_slot = 0;
  std::vector<uint64_t> ag_off;
  std::vector<tcx_copy_job> ag_jobs;
  auto ag_count = [&](int r, uint64_t k) -> uint64_t {
    const uint64_t w0 = b[r] + k * W;
    return w0 >= b[r + 1] ? 0 : std::min(W, b[r + 1] - w0);
  };
  if (gather_all) {
    rounds = 0;
    round_pack.clear();
    round_scatter.clear();
    std::fill(pack_off.begin(), pack_off.end(), 0);
    std::fill(scat_off.begin(), scat_off.end(), 0);
    uint64_t max_stage = 0;
    for (int r = 0; r < world; ++r) max_stage = std::max(max_stage, b[r + 1] - b[r]);
    ag_rounds = (max_stage + W - 1) / W;
    ag_slot = std::min(W, std::max<uint64_t>(max_stage, 1));
    ag_off.assign(ag_rounds + 1, 0);
    const tcx_copy_job* my_jobs = plan->jobs + plan->job_offsets[rank];
    const uint64_t n_my = plan->job_offsets[rank + 1] - plan->job_offsets[rank];
    for (uint64_t k = 0; k < ag_rounds; ++k) {
      for (int r = 0; r < world; ++r) {
        const uint64_t n = ag_count(r, k);
        if (r == rank || n == 0) continue;
        const uint64_t w0 = b[r] + k * W;
        tmp.clear();
        clip_jobs(my_jobs, n_my, w0, w0 + n, tmp);
        for (auto j : tmp) {
          j.src_off = j.src_off - w0 + ((k % 2) * static_cast<uint64_t>(world) + static_cast<uint64_t>(r)) * ag_slot;
          ag_jobs.push_back(j);
        }
      }
      ag_off[k + 1] = ag_jobs.size();
    }
  }

  // --- buffers --------------------------------------------------------------
  const uint64_t n_jobs_all =
      round_pack.size() + local_kept.size() + round_scatter.size() + compact.size() + ag_jobs.size();
  const uint64_t n_launches = 2 * rounds + 2 + ag_rounds;
  if ((st = g->digests_mine.grow(std::max<uint64_t>(max_n, 1) * 32)) != TCX_OK) return st;
  if ((st = g->states.grow(std::max<uint64_t>(n_mine, 1) * 32)) != TCX_OK) return st;
  if ((st = g->merkle_scratch.grow(merkle_scratch_bytes(n_total))) != TCX_OK) return st;
  if ((st = g->root.grow(256)) != TCX_OK) return st;
  if ((st = g->jobs.grow(std::max<uint64_t>(n_jobs_all, 1) * sizeof(tcx_copy_job))) != TCX_OK) return st;
  if ((st = g->prefix.grow((n_jobs_all + n_launches + 1) * 8)) != TCX_OK) return st;
  if (rounds && max_send && (st = g->send.grow(2 * peers.size() * send_slot)) != TCX_OK) return st;
  if (rounds && max_recv_buf && (st = g->recv.grow(2 * peers.size() * recv_slot)) != TCX_OK) return st;
  if (perm_bytes && (st = g->perm_scratch.grow(perm_bytes)) != TCX_OK) return st;
  if (push && (st = g->barrier_word.grow(256)) != TCX_OK) return st;
  if (ag_rounds && (st = g->recv.grow(2 * static_cast<uint64_t>(world) * ag_slot)) != TCX_OK) return st;
  if (world > 1) {
    if ((st = g->digests_all.grow(static_cast<uint64_t>(world) * max_n * 32)) != TCX_OK) return st;
    if ((st = g->digests_compact.grow(n_total * 32)) != TCX_OK) return st;
  }
  const bool view_hash = (plan->flags & TCX_LOAD_VIEW_HASH) != 0 && plan->view_bytes > 0;
  uint64_t view_leaf = 0, view_n = 0;
  if (view_hash) {
    if ((st = tcx_leaf_policy(plan->view_bytes, TCX_DEFAULT_LEAF_BYTES, &view_leaf)) != TCX_OK) return st;
    view_n = (plan->view_bytes + view_leaf - 1) / view_leaf;
    if ((st = g->view_digests.grow(view_n * 32)) != TCX_OK) return st;
    if ((st = g->view_scratch.grow(merkle_scratch_bytes(view_n) + 256)) != TCX_OK) return st;
  }
  if ((st = ensure_events(g->packed_events, std::max(rounds, ag_rounds))) != TCX_OK) return st;
  if ((st = ensure_events(g->sent_events, std::max(rounds, ag_rounds))) != TCX_OK) return st;
  if (n_jobs_all > g->h_jobs_cap) {
    if (g->h_jobs) cudaFreeHost(g->h_jobs);
    g->h_jobs = nullptr;
    g->h_jobs_cap = 0;
    TCX_CUDA_TRY(cudaMallocHost(&g->h_jobs, n_jobs_all * sizeof(tcx_copy_job)));
    g->h_jobs_cap = n_jobs_all;
  }
  tcx_copy_job* hj = g->h_jobs;
  const uint64_t o_pack = 0, o_local = round_pack.size(), o_scatter = o_local + local_kept.size(),
                 o_compact = o_scatter + round_scatter.size(), o_ag = o_compact + compact.size();
  std::copy(round_pack.begin(), round_pack.end(), hj + o_pack);
  std::copy(local_kept.begin(), local_kept.end(), hj + o_local);
  std::copy(round_scatter.begin(), round_scatter.end(), hj + o_scatter);
  std::copy(compact.begin(), compact.end(), hj + o_compact);
  std::copy(ag_jobs.begin(), ag_jobs.end(), hj + o_ag);
  auto* dj = static_cast<tcx_copy_job*>(g->jobs.p);
  auto* dprefix = static_cast<uint64_t*>(g->prefix.p);
  // Each copy-job launch gets its own prefix region, handed out in launch order
  // (launches run on two streams at once, so regions must never overlap).
  uint64_t prefix_cursor = 0;
  auto prefix_for = [&](uint64_t n_jobs) {
    uint64_t* r = dprefix + prefix_cursor;
    prefix_cursor += n_jobs + 1;
    return r;
  };
  auto* view = static_cast<uint8_t*>(d_view);
  auto* stage = static_cast<uint8_t*>(d_stage);
  const auto* hstage = static_cast<const uint8_t*>(h_stage);

  const auto deadline = Clock::now() + std::chrono::milliseconds(g->timeout_ms);
  if (push) {
    // Map every peer's view (collective) and check that each push stays inside it.
    if ((st = map_peer_views(g, d_view, plan->view_bytes, deadline)) != TCX_OK) return st;
    if (g->s_peer.empty()) {
      g->s_peer.assign(world, nullptr);
      g->peer_done.assign(world, nullptr);
      for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        TCX_CUDA_TRY(cudaStreamCreateWithFlags(&g->s_peer[p], cudaStreamNonBlocking));
        TCX_CUDA_TRY(cudaEventCreateWithFlags(&g->peer_done[p], cudaEventDisableTiming));
      }
      TCX_CUDA_TRY(cudaEventCreateWithFlags(&g->ev_push, cudaEventDisableTiming));
    }
    for (int p = 0; p < world; ++p) {
      if (p == rank) continue;
      for (uint64_t i = push_off[p]; i < push_off[p + 1]; ++i) {
        const tcx_copy_job& j = push_jobs[i];
        const uint64_t end = j.dst_off + (j.rows - 1) * j.dst_pitch + j.row_bytes;
        if (end > g->peer_views[p].size)
          return set_errorf(TCX_INVALID_ARGUMENT, "rank %d's view (%llu bytes) is smaller than its jobs need", p,
                            static_cast<unsigned long long>(g->peer_views[p].size));
      }
    }
  }

  // --- H2D + hashing ---------------------------------------------------------
  // Everything queued on the caller's stream before this call (writes into the
  // staged or view buffers, for instance) completes before the load touches them.
  TCX_CUDA_TRY(cudaEventRecord(g->ev_start, static_cast<cudaStream_t>(stream)));
  TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_copy, g->ev_start, 0));
  TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_hash, g->ev_start, 0));
  TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->ev_start, 0));
  uint64_t h2d_bytes = 0;
  float read_ms = 0.f;
  if (mine > 0) {
    if (hstage != nullptr || files != nullptr) {
      // Slabs: slab j is bytes [j*S, (j+1)*S) of every leaf of the range (one 2-D
      // copy: n_full rows at pitch L, plus the short last leaf), so every leaf's
      // chain advances as each slab lands.
      const uint64_t n_full = mine / L, tail = mine - n_full * L;
      const uint64_t span = n_full > 0 ? L : tail;  // bytes per leaf to cover
      const uint64_t n_rows = n_full + (tail > 0 ? 1 : 0);
      // From files, leaves of at least 2 pieces are staged piece by piece (each
      // piece's copy queued as soon as it is read, see stage_pieces_from_files).
      const uint64_t piece = files != nullptr ? piece_bytes_for(span) : 0;
      uint64_t S = plan->slab_bytes;
      if (piece > 0 && S == 0) S = piece;
      if (S == 0 && files != nullptr) {
        // From files, a slab is one pinned slot: about slot_bytes per slab.
        // S is a power of two from 64 bytes up to the leaf.
        const uint64_t want = files->slot_bytes ? files->slot_bytes : kDefaultSlotBytes;
        S = 64;
        while (S * 2 <= span && S * 2 * n_rows <= want) S *= 2;
      }
      if (S == 0) S = kDefaultSlab;
      S = std::max<uint64_t>(64, S - S % 64);
      const uint64_t J = (span + S - 1) / S;
      if ((st = ensure_events(g->slab_events, J)) != TCX_OK) return st;
      // H2D of slab j from src (rows at src_pitch; the short leaf's piece at tsrc),
      // then the streamed hash pass over it.
      // The streamed hash pass over slab j, once everything queued on s_copy is done.
      auto hash_slab = [&](uint64_t j) -> tcx_status {
        TCX_CUDA_TRY(cudaEventRecord(g->slab_events[j], g->s_copy));
        TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_hash, g->slab_events[j], 0));
        return launch_leaf_pass(stage, mine, L, static_cast<uint32_t>(n_mine), j * S, S,
                                static_cast<uint32_t*>(g->states.p), g->digests_mine.p, g->s_hash);
      };
      auto enqueue_slab = [&](uint64_t j, const uint8_t* src, uint64_t src_pitch, const uint8_t* tsrc) -> tcx_status {
        const uint64_t off = j * S;
        if (n_full > 0 && off < L) {
          const uint64_t w = std::min(S, L - off);
          TCX_CUDA_TRY(cudaMemcpy2DAsync(stage + off, L, src, src_pitch, w, n_full, cudaMemcpyHostToDevice, g->s_copy));
        }
        if (tail > off) {
          const uint64_t w = std::min(S, tail - off);
          TCX_CUDA_TRY(cudaMemcpyAsync(stage + n_full * L + off, tsrc, w, cudaMemcpyHostToDevice, g->s_copy));
        }
        return hash_slab(j);
      };
      if (files == nullptr) {
        for (uint64_t j = 0; j < J; ++j) {
          if ((st = enqueue_slab(j, hstage + j * S, L, hstage + n_full * L + j * S)) != TCX_OK) return st;
        }
      } else {
        const auto t_read = Clock::now();
        if (piece > 0 && S == piece)
          st = stage_pieces_from_files(g, *files, stage, mine, L, S, J, n_full, tail, piece_rows_for(S, n_rows),
                                       piece_buffers(), hash_slab, deadline);
        else
          st = stage_from_files(g, *files, mine, L, S, J, n_full, tail, enqueue_slab, deadline);
        read_ms = std::chrono::duration<float, std::milli>(Clock::now() - t_read).count();
        if (st != TCX_OK) return st;
      }
      h2d_bytes = mine;
    } else {
      st = launch_leaf_pass(stage, mine, L, static_cast<uint32_t>(n_mine), 0, ~0ull, nullptr, g->digests_mine.p,
                            g->s_hash);
      if (st != TCX_OK) return st;
    }
  }
  TCX_CUDA_TRY(cudaEventRecord(g->ev_h2d, g->s_copy));
  TCX_CUDA_TRY(cudaEventRecord(g->ev_hash, g->s_hash));

  // --- exchange and view extraction ------------------------------------------
  TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, alias ? g->ev_hash : g->ev_h2d, 0));
  if (n_jobs_all > 0)
    TCX_CUDA_TRY(cudaMemcpyAsync(dj, hj, n_jobs_all * sizeof(tcx_copy_job), cudaMemcpyHostToDevice, g->s_comm));
  TCX_CUDA_TRY(cudaEventRecord(g->ev_exch, g->s_comm));  // job tables uploaded, staged bytes complete
  TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_pack, g->ev_exch, 0));
  // View bytes no job writes are zero-filled, as a fresh view buffer is; bytes
  // between target tensors belong to no one and are left alone.
  if ((plan->flags & TCX_LOAD_TARGETS) == 0)
    for (uint64_t k = 0; k < xp.n_gaps; ++k)
      TCX_CUDA_TRY(cudaMemsetAsync(view + gaps[2 * k], 0, gaps[2 * k + 1], g->s_comm));
  // This rank's own view pieces: at N > 1 on their own stream, so that they are
  // copied while the exchange (push copies or NCCL rounds) runs; the permutes and
  // the view hash below wait for them.
  cudaStream_t s_loc = world > 1 ? g->s_local : g->s_comm;
  if (world > 1) TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_local, g->ev_exch, 0));
  if (!local_kept.empty() && world > 1 && local_copy_on_copy_engines()) {
    for (const tcx_copy_job& j : local_kept) {
      if (j.rows == 0 || j.row_bytes == 0) continue;
      if (j.rows == 1)
        TCX_CUDA_TRY(cudaMemcpyAsync(view + j.dst_off, stage + j.src_off, j.row_bytes, cudaMemcpyDeviceToDevice, s_loc));
      else
        TCX_CUDA_TRY(cudaMemcpy2DAsync(view + j.dst_off, j.dst_pitch, stage + j.src_off, j.src_pitch, j.row_bytes,
                                       j.rows, cudaMemcpyDeviceToDevice, s_loc));
    }
  } else if (!local_kept.empty()) {
    uint64_t local_bytes = 0;
    for (const tcx_copy_job& j : local_kept) local_bytes += j.rows * j.row_bytes;
    if ((st = launch_copy_jobs(stage, view, dj + o_local, local_kept.size(), prefix_for(local_kept.size()), s_loc,
                               load_copy_ctas(n_mine, local_bytes, L))) != TCX_OK)
      return st;
  }
  if (world > 1) TCX_CUDA_TRY(cudaEventRecord(g->ev_local, g->s_local));
  uint64_t sent = 0, received = 0;
  if (push) {
    // Every rank's view is ready to be written (its gaps cleared, its earlier loads done).
    if ((st = nccl_barrier(g, deadline)) != TCX_OK) return st;
    TCX_CUDA_TRY(cudaEventRecord(g->ev_push, g->s_comm));
    TCX_CUDA_TRY(cudaEventRecord(g->ev_xfer0, g->s_comm));
    // The pushes run on the copy engines, one stream per peer: no SM time is
    // taken from the leaf hash that is still running, and the peers' transfers
    // proceed side by side. A job is one 2-D copy (rows at the source and
    // destination pitches) from the staged range straight into the peer's view.
    for (int p = 0; p < world; ++p) {
      if (p == rank || push_off[p + 1] == push_off[p]) continue;
      cudaStream_t sp = g->s_peer[p];
      TCX_CUDA_TRY(cudaStreamWaitEvent(sp, g->ev_push, 0));
      uint8_t* peer_view = static_cast<uint8_t*>(g->peer_views[p].base) + g->peer_views[p].offset;
      for (uint64_t i = push_off[p]; i < push_off[p + 1]; ++i) {
        const tcx_copy_job& j = push_jobs[i];
        if (j.rows == 0 || j.row_bytes == 0) continue;
        if (j.rows == 1)
          TCX_CUDA_TRY(cudaMemcpyAsync(peer_view + j.dst_off, stage + j.src_off, j.row_bytes, cudaMemcpyDeviceToDevice, sp));
        else
          TCX_CUDA_TRY(cudaMemcpy2DAsync(peer_view + j.dst_off, j.dst_pitch, stage + j.src_off, j.src_pitch, j.row_bytes,
                                         j.rows, cudaMemcpyDeviceToDevice, sp));
      }
      TCX_CUDA_TRY(cudaEventRecord(g->peer_done[p], sp));
    }
  }
  if (rounds && !push) TCX_CUDA_TRY(cudaEventRecord(g->ev_xfer0, g->s_comm));
  for (uint64_t k = 0; k < rounds; ++k) {
    const uint64_t buf = k % 2;
    // pack round k on the pack stream once round k-2 (same buffer) has been sent
    if (k >= 2) TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_pack, g->sent_events[k - 2], 0));
    const uint64_t np = pack_off[k + 1] - pack_off[k];
    if (np && (st = launch_copy_jobs(stage, g->send.p, dj + o_pack + pack_off[k], np,
                                     prefix_for(np), g->s_pack)) != TCX_OK)
      return st;
    TCX_CUDA_TRY(cudaEventRecord(g->packed_events[k], g->s_pack));
    TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->packed_events[k], 0));
    if ((st = nccl_check(g, ncclGroupStart(), deadline, "ncclGroupStart")) != TCX_OK) return st;
    for (size_t si = 0; si < peers.size(); ++si) {
      const int p = peers[si];
      const uint64_t sp = send_off[p + 1] - send_off[p];
      if (k * W < sp) {
        const uint64_t n = std::min(W, sp - k * W);
        st = nccl_check(g, ncclSend(g->send.bytes() + (buf * peers.size() + si) * send_slot, n, ncclUint8, p, g->comm,
                                    g->s_comm), deadline, "ncclSend");
        if (st != TCX_OK) return st;
        sent += n;
      }
      if (k * W < recv_counts[p]) {
        const uint64_t n = std::min(W, recv_counts[p] - k * W);
        uint8_t* dst = direct[p] ? view + recv_view[p] + k * W : g->recv.bytes() + (buf * peers.size() + si) * recv_slot;
        st = nccl_check(g, ncclRecv(dst, n, ncclUint8, p, g->comm, g->s_comm), deadline, "ncclRecv");
        if (st != TCX_OK) return st;
        received += n;
      }
    }
    if ((st = nccl_check(g, ncclGroupEnd(), deadline, "exchange")) != TCX_OK) return st;
    TCX_CUDA_TRY(cudaEventRecord(g->sent_events[k], g->s_comm));
    if (k + 1 == rounds && !push) TCX_CUDA_TRY(cudaEventRecord(g->ev_xfer1, g->s_comm));
    const uint64_t ns = scat_off[k + 1] - scat_off[k];
    if (ns && (st = launch_copy_jobs(g->recv.p, view, dj + o_scatter + scat_off[k], ns,
                                     prefix_for(ns), g->s_comm)) != TCX_OK)
      return st;
  }
  if (push) {
    for (int p = 0; p < world; ++p)
      if (p != rank && push_off[p + 1] != push_off[p])
        TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->peer_done[p], 0));
    TCX_CUDA_TRY(cudaEventRecord(g->ev_xfer1, g->s_comm));  // this rank's pushes (and NCCL rounds) are done
    // Every peer has finished writing into this rank's view.
    if ((st = nccl_barrier(g, deadline)) != TCX_OK) return st;
    sent += push_bytes;
    received = 0;
    for (int p = 0; p < world; ++p)
      if (p != rank) received += recv_counts_all[p];
  }
  if (ag_rounds) TCX_CUDA_TRY(cudaEventRecord(g->ev_xfer0, g->s_comm));
  for (uint64_t k = 0; k < ag_rounds; ++k) {
    // The window slots of round k were last read by the extraction of round k-2.
    if (k >= 2) TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->packed_events[k - 2], 0));
    if ((st = nccl_check(g, ncclGroupStart(), deadline, "ncclGroupStart")) != TCX_OK) return st;
    for (int r = 0; r < world; ++r) {
      const uint64_t n = ag_count(r, k);
      if (n == 0) continue;
      uint8_t* buf = r == rank ? stage + k * W
                               : g->recv.bytes() + ((k % 2) * static_cast<uint64_t>(world) + static_cast<uint64_t>(r)) * ag_slot;
      st = nccl_check(g, ncclBroadcast(buf, buf, n, ncclUint8, r, g->comm, g->s_comm), deadline, "ncclBroadcast");
      if (st != TCX_OK) return st;
      if (r == rank) sent += n * static_cast<uint64_t>(world - 1);
      else received += n;
    }
    if ((st = nccl_check(g, ncclGroupEnd(), deadline, "exchange")) != TCX_OK) return st;
    TCX_CUDA_TRY(cudaEventRecord(g->sent_events[k], g->s_comm));
    if (k + 1 == ag_rounds) TCX_CUDA_TRY(cudaEventRecord(g->ev_xfer1, g->s_comm));
    TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_pack, g->sent_events[k], 0));
    const uint64_t ne = ag_off[k + 1] - ag_off[k];
    if (ne && (st = launch_copy_jobs(g->recv.p, view, dj + o_ag + ag_off[k], ne, prefix_for(ne), g->s_pack,
                                     load_copy_ctas(n_mine, 0, L))) != TCX_OK)
      return st;
    TCX_CUDA_TRY(cudaEventRecord(g->packed_events[k], g->s_pack));
  }
  if (ag_rounds) TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->packed_events[ag_rounds - 1], 0));
  if (world > 1) TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->ev_local, 0));
  for (uint64_t i = 0; i < plan->n_permutes; ++i) {
    tcx_permute_job pj = plan->permutes[i];
    uint64_t bytes = pj.esize;
    for (uint32_t d = 0; d < pj.ndim; ++d) bytes *= static_cast<uint64_t>(pj.shape[d]);
    const uint64_t off = pj.dst_off;
    pj.src_off = off;
    pj.dst_off = 0;
    if ((st = launch_permute(view, g->perm_scratch.p, pj, g->s_comm)) != TCX_OK) return st;
    TCX_CUDA_TRY(cudaMemcpyAsync(view + off, g->perm_scratch.p, bytes, cudaMemcpyDeviceToDevice, g->s_comm));
  }
  if (view_hash) {
    // View multihash: the view is final here; its root lands after the artifact root.
    if ((st = launch_leaf_pass(view, plan->view_bytes, view_leaf, static_cast<uint32_t>(view_n), 0, ~0ull, nullptr,
                               g->view_digests.p, g->s_comm)) != TCX_OK)
      return st;
    if ((st = launch_merkle(g->view_digests.bytes(), view_n, g->view_scratch.bytes(), g->root.bytes() + 64,
                            g->s_comm)) != TCX_OK)
      return st;
  }
  TCX_CUDA_TRY(cudaEventRecord(g->ev_exch, g->s_comm));

  // --- digests of every rank, Merkle root ------------------------------------
  TCX_CUDA_TRY(cudaStreamWaitEvent(g->s_comm, g->ev_hash, 0));
  const uint8_t* leaf_digests = g->digests_mine.bytes();
  if (world > 1) {
    st = nccl_check(g, ncclAllGather(g->digests_mine.p, g->digests_all.p, max_n * 32, ncclUint8, g->comm, g->s_comm),
                    deadline, "digest all-gather");
    if (st != TCX_OK) return st;
    if ((st = launch_copy_jobs(g->digests_all.p, g->digests_compact.p, dj + o_compact, compact.size(),
                               prefix_for(compact.size()), g->s_comm)) != TCX_OK)
      return st;
    leaf_digests = g->digests_compact.bytes();
  }
  if ((st = launch_merkle(leaf_digests, n_total, g->merkle_scratch.bytes(), g->root.bytes(), g->s_comm)) != TCX_OK)
    return st;
  TCX_CUDA_TRY(cudaMemcpyAsync(g->h_root, g->root.p, view_hash ? 96 : 32, cudaMemcpyDeviceToHost, g->s_comm));
  TCX_CUDA_TRY(cudaEventRecord(g->ev_end, g->s_comm));
  if ((st = wait_event(g, g->ev_end, deadline)) != TCX_OK) return st;

  std::memset(out, 0, sizeof *out);
  std::memcpy(out->root, g->h_root, 32);
  encode_multihash(out->root, out->multihash);
  out->leaves = n_total;
  out->h2d_bytes = h2d_bytes;
  out->peer_send_bytes = sent;
  out->peer_recv_bytes = received;
  out->h2d_ms = elapsed_ms(g->ev_start, g->ev_h2d);
  out->hash_ms = elapsed_ms(g->ev_start, g->ev_hash);
  out->exchange_ms = elapsed_ms(g->ev_h2d, g->ev_exch);
  out->total_ms = elapsed_ms(g->ev_start, g->ev_end);
  out->stage_read_ms = read_ms;
  out->transfer_ms = (push || rounds || ag_rounds) ? elapsed_ms(g->ev_xfer0, g->ev_xfer1) : 0.f;
  if (view_hash) {
    encode_multihash(g->h_root + 64, out->view_multihash);
    out->view_leaf_bytes = view_leaf;
  }
  if (expected_root != nullptr && std::memcmp(expected_root, out->root, 32) != 0)
    return set_error(TCX_DATA_LOSS, "ARTIFACT_ID_MISMATCH: data multihash of the loaded bytes differs from the expected one");
  return TCX_OK;
}

}  // namespace

extern "C" tcx_status tcx_group_load(tcx_group* g, const tcx_load_plan* plan, const void* h_stage, void* d_stage,
                                     void* d_view, const uint8_t* expected_root, tcx_load_result* out,
                                     void* stream) {
  return group_load(g, plan, h_stage, nullptr, d_stage, d_view, expected_root, out, stream);
}

extern "C" tcx_status tcx_group_load_files(tcx_group* g, const tcx_load_plan* plan, const tcx_file_stage* files,
                                           void* d_stage, void* d_view, const uint8_t* expected_root,
                                           tcx_load_result* out, void* stream) {
  if (files == nullptr) return set_error(TCX_INVALID_ARGUMENT, "files is null");
  return group_load(g, plan, nullptr, files, d_stage, d_view, expected_root, out, stream);
}

namespace {
struct FileMapping {
  void* base = nullptr;
  uint64_t length = 0;
  bool registered = false;
};
}  // namespace

extern "C" tcx_status tcx_host_map_file(const char* path, uint64_t offset, uint64_t length, int register_pinned,
                                        void** host_ptr, void** handle) {
  if (path == nullptr || host_ptr == nullptr || handle == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "path, host_ptr and handle are required");
  *host_ptr = nullptr;
  *handle = nullptr;
  if (length == 0) return set_error(TCX_INVALID_ARGUMENT, "length must be > 0");
  const long page = sysconf(_SC_PAGESIZE);
  const uint64_t aligned_off = offset - offset % static_cast<uint64_t>(page);
  const uint64_t map_len = length + (offset - aligned_off);
  // Read-only mapping registered read-only first; where the driver refuses that, a
  // shared read-write mapping (never written) registered normally.
  void* base = MAP_FAILED;
  bool registered = false;
  std::string why;
  for (int attempt = 0; attempt < (register_pinned ? 2 : 1) && !registered; ++attempt) {
    const bool rw = attempt == 1;
    const int fd = open(path, (rw ? O_RDWR : O_RDONLY) | O_CLOEXEC);
    if (fd < 0) {
      if (attempt == 0) return set_errorf(TCX_NOT_FOUND, "open failed: %s", path);
      break;
    }
    const off_t size = lseek(fd, 0, SEEK_END);
    if (size < 0 || static_cast<uint64_t>(size) < offset + length) {
      close(fd);
      return set_errorf(TCX_OUT_OF_RANGE, "%s is shorter than the mapped range", path);
    }
    base = mmap(nullptr, map_len, rw ? (PROT_READ | PROT_WRITE) : PROT_READ, MAP_SHARED | MAP_POPULATE, fd,
                static_cast<off_t>(aligned_off));
    close(fd);
    if (base == MAP_FAILED)
      return set_errorf(TCX_RESOURCE_EXHAUSTED, "mmap of %llu bytes failed", static_cast<unsigned long long>(map_len));
    if (!register_pinned) break;
    const cudaError_t e =
        cudaHostRegister(base, map_len, rw ? cudaHostRegisterPortable : (cudaHostRegisterReadOnly | cudaHostRegisterPortable));
    if (e == cudaSuccess) {
      registered = true;
    } else {
      why += (why.empty() ? "" : "; ") + cuda_msg(e);
      cudaGetLastError();
      munmap(base, map_len);
      base = MAP_FAILED;
    }
  }
  if (register_pinned && !registered)
    return set_error(TCX_UNAVAILABLE, "cudaHostRegister of the file mapping failed: " + why);
  auto* m = new FileMapping{base, map_len, registered};
  *host_ptr = static_cast<uint8_t*>(base) + (offset - aligned_off);
  *handle = m;
  return TCX_OK;
}

extern "C" tcx_status tcx_host_unmap_file(void* handle) {
  if (handle == nullptr) return TCX_OK;
  auto* m = static_cast<FileMapping*>(handle);
  tcx_status st = TCX_OK;
  if (m->registered) {
    cudaError_t e = cudaHostUnregister(m->base);
    if (e != cudaSuccess) st = set_error(TCX_INTERNAL, "cudaHostUnregister failed: " + cuda_msg(e));
  }
  munmap(m->base, m->length);
  delete m;
  return st;
}

extern "C" tcx_status tcx_bind_device_cpus(int device, int* n_cpus_out) {
  // The CPUs on the GPU's side of the PCIe hierarchy (sysfs local_cpulist). Binding
  // the calling thread there before it allocates pinned buffers places them, by
  // first touch, on the GPU's NUMA node; threads it starts afterwards inherit it.
  char bus[64] = {0};
  TCX_CUDA_TRY(cudaDeviceGetPCIBusId(bus, sizeof bus, device));
  for (char* c = bus; *c; ++c) *c = static_cast<char>(tolower(*c));
  const std::string path = std::string("/sys/bus/pci/devices/") + bus + "/local_cpulist";
  FILE* f = fopen(path.c_str(), "r");
  if (f == nullptr) return set_errorf(TCX_NOT_FOUND, "cannot read %s", path.c_str());
  char list[4096] = {0};
  const size_t got = fread(list, 1, sizeof list - 1, f);
  fclose(f);
  list[got] = 0;
  cpu_set_t set;
  CPU_ZERO(&set);
  int count = 0;
  for (char* tok = strtok(list, ",\n"); tok != nullptr; tok = strtok(nullptr, ",\n")) {
    int a = -1, b = -1;
    if (sscanf(tok, "%d-%d", &a, &b) == 2) {
    } else if (sscanf(tok, "%d", &a) == 1) {
      b = a;
    } else {
      continue;
    }
    for (int c = a; c <= b && c < CPU_SETSIZE; ++c) {
      CPU_SET(c, &set);
      ++count;
    }
  }
  if (count == 0) return set_errorf(TCX_NOT_FOUND, "no CPUs listed in %s", path.c_str());
  if (sched_setaffinity(0, sizeof set, &set) != 0) return set_error(TCX_INTERNAL, "sched_setaffinity failed");
  if (n_cpus_out) *n_cpus_out = count;
  return TCX_OK;
}
