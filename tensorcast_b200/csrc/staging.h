// Host-side staging shared by the collective load (loader.cc) and the file hash
// (disk_hash.cc): a pool of reader threads, the file segments of a byte range,
// and per-reader pinned piece buffers whose host-to-device copies each reader
// queues on its own stream as soon as it has read them. Not part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "tcx_internal.h"

namespace tcx {

using StageClock = std::chrono::steady_clock;

// One unit of host reading: fn(i) for i in [0, n), run by the reader pool's
// threads; fn returns false (with code/err set under mu) on failure, after which
// the remaining items are skipped.
struct ReadBatch {
  std::function<bool(uint64_t, ReadBatch&)> fn;
  uint64_t n = 0;
  std::atomic<uint64_t> done{0};
  std::atomic<bool> failed{false};
  uint64_t next = 0;  // next item to hand out (guarded by the pool's mutex)
  std::mutex mu;
  std::condition_variable cv;
  tcx_status code = TCX_OK;
  std::string err;
  void fail(tcx_status c, const std::string& m);
};

// Index of the pool thread that runs the current item (-1 outside a pool).
int reader_index();

// Persistent host threads that read file pieces into pinned memory. Batches are
// served in submission order; a thread that finds every item of the oldest batch
// handed out moves on to the next one, so several batches are read at once.
class ReadPool {
 public:
  explicit ReadPool(int n);
  ~ReadPool();
  int size() const { return static_cast<int>(threads_.size()); }
  void submit(const std::shared_ptr<ReadBatch>& b);
  // True once every item of b has run (or been skipped after a failure); false at the deadline.
  static bool wait(ReadBatch& b, StageClock::time_point deadline);

 private:
  void work(int index);
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::shared_ptr<ReadBatch>> q_;
  std::vector<std::thread> threads_;
  bool stop_ = false;
};

// CPUs this process may run on.
int affinity_cpus();

// The file segments of a staged byte range, shared by the reader threads (held
// by every batch that reads them, so it outlives any piece in flight).
struct FileStageCtx {
  std::vector<tcx_file_segment> segs;  // sorted by dst_offset, non-overlapping; paths point into `paths`
  std::vector<std::string> paths;
  std::vector<int> fds;                // per segment
  std::vector<int> owned;              // distinct descriptors to close
  ~FileStageCtx();
};

// Checks, sorts and opens segments covering parts of [0, range): a missing file
// is NOT_FOUND, overlapping or out-of-range segments INVALID_ARGUMENT.
tcx_status open_stage_files(const tcx_file_segment* segments, uint64_t n_segments, uint64_t range,
                            FileStageCtx* ctx);

// Reads range bytes [a, a + w) into dst: file bytes where a segment covers them,
// zero elsewhere. A short read records DATA_LOSS in b and returns false.
bool read_stage_range(const FileStageCtx& c, uint64_t a, uint64_t w, uint8_t* dst, ReadBatch& b);

// Per reader thread: a stream and `bufs` pinned buffers, each with the event of
// the copy that last read it. Released explicitly (never from a destructor, so
// that nothing calls CUDA during static destruction).
struct PieceBuffers {
  uint8_t* host = nullptr;  // readers x bufs buffers of buf_bytes
  uint64_t buf_bytes = 0;
  int bufs = 0;
  std::vector<cudaStream_t> streams;  // per reader
  std::vector<cudaEvent_t> copied;    // per buffer
  std::vector<cudaEvent_t> marks;     // per reader: joins its stream into another
  std::vector<uint8_t> used;          // per buffer: a copy was queued from it
  std::vector<uint64_t> count;        // per reader: buffers taken (picks the next one)

  int readers() const { return static_cast<int>(streams.size()); }
  // Allocates for `n_readers` readers, `n_bufs` buffers of at least `bytes` each
  // (kept when already large enough).
  tcx_status ensure(int n_readers, uint64_t bytes, int n_bufs);
  void release();
  // Waits for every copy queued on the readers' streams.
  void sync();
  // Makes every reader stream wait for ev before its next copy.
  tcx_status wait_on(cudaEvent_t ev);
  // Reader t's next buffer, once the copy that last read it is done (polled up
  // to the deadline); nullptr with the failure recorded in b. *slot names it for
  // queued().
  uint8_t* acquire(int t, StageClock::time_point deadline, ReadBatch& b, uint64_t* slot);
  // Records, after the copies reader t has just queued from buffer `slot`, the
  // event acquire() waits for before that buffer is reused.
  bool queued(int t, uint64_t slot, ReadBatch& b);
  // Stream s waits for everything queued so far on the readers' streams.
  tcx_status join(cudaStream_t s);
};

// The calling reader thread's index in its pool, checked against the buffers,
// with the device made current for its copies; -1 with the failure in b.
int reader_for_copies(const PieceBuffers& pb, int device, ReadBatch& b);

}  // namespace tcx
