// Host-side staging shared by the collective load and the file hash: reader
// threads, file segments of a byte range, per-reader pinned piece buffers.
#include "staging.h"

#include <fcntl.h>
#include <sched.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <map>

namespace tcx {

namespace {
thread_local int t_reader = -1;
}  // namespace

int reader_index() { return t_reader; }

void ReadBatch::fail(tcx_status c, const std::string& m) {
  std::lock_guard<std::mutex> lk(mu);
  if (code == TCX_OK) {
    code = c;
    err = m;
  }
  failed = true;
}

ReadPool::ReadPool(int n) {
  for (int i = 0; i < n; ++i) threads_.emplace_back([this, i] { work(i); });
}

ReadPool::~ReadPool() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : threads_) t.join();
}

void ReadPool::submit(const std::shared_ptr<ReadBatch>& b) {
  if (b->n == 0) return;
  {
    std::lock_guard<std::mutex> lk(mu_);
    q_.push_back(b);
  }
  cv_.notify_all();
}

bool ReadPool::wait(ReadBatch& b, StageClock::time_point deadline) {
  std::unique_lock<std::mutex> lk(b.mu);
  return b.cv.wait_until(lk, deadline, [&] { return b.done.load() == b.n; });
}

void ReadPool::work(int index) {
  t_reader = index;
  for (;;) {
    std::shared_ptr<ReadBatch> b;
    uint64_t i = 0;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return stop_ || !q_.empty(); });
      if (q_.empty()) return;  // stop_ with nothing queued
      b = q_.front();
      i = b->next++;
      if (b->next >= b->n) q_.pop_front();
    }
    if (!b->failed.load()) {
      if (!b->fn(i, *b)) b->failed = true;
    }
    if (b->done.fetch_add(1) + 1 == b->n) {
      std::lock_guard<std::mutex> lk(b->mu);
      b->cv.notify_all();
    }
  }
}

int affinity_cpus() {
  cpu_set_t set;
  CPU_ZERO(&set);
  if (sched_getaffinity(0, sizeof set, &set) != 0) return 8;
  return std::max(1, CPU_COUNT(&set));
}

FileStageCtx::~FileStageCtx() {
  for (int fd : owned) close(fd);
}

tcx_status open_stage_files(const tcx_file_segment* segments, uint64_t n_segments, uint64_t range,
                            FileStageCtx* ctx) {
  if (n_segments > 0 && segments == nullptr) return set_error(TCX_INVALID_ARGUMENT, "segments is null");
  ctx->segs.reserve(n_segments);
  ctx->paths.reserve(n_segments);
  for (uint64_t i = 0; i < n_segments; ++i) {
    const tcx_file_segment& x = segments[i];
    if (x.path == nullptr)
      return set_errorf(TCX_INVALID_ARGUMENT, "segment %llu has no path", static_cast<unsigned long long>(i));
    if (x.length == 0) continue;
    if (x.dst_offset > range || x.length > range - x.dst_offset)
      return set_errorf(TCX_INVALID_ARGUMENT, "segment %llu lies outside the staged range of %llu bytes",
                        static_cast<unsigned long long>(i), static_cast<unsigned long long>(range));
    ctx->paths.emplace_back(x.path);
    ctx->segs.push_back(x);
  }
  for (size_t i = 0; i < ctx->segs.size(); ++i) ctx->segs[i].path = ctx->paths[i].c_str();
  std::sort(ctx->segs.begin(), ctx->segs.end(),
            [](const tcx_file_segment& x, const tcx_file_segment& y) { return x.dst_offset < y.dst_offset; });
  for (size_t i = 1; i < ctx->segs.size(); ++i)
    if (ctx->segs[i].dst_offset < ctx->segs[i - 1].dst_offset + ctx->segs[i - 1].length)
      return set_error(TCX_INVALID_ARGUMENT, "segments overlap in the staged range");
  std::map<std::string, int> opened;
  ctx->fds.resize(ctx->segs.size());
  for (size_t i = 0; i < ctx->segs.size(); ++i) {
    auto it = opened.find(ctx->segs[i].path);
    if (it == opened.end()) {
      const int fd = open(ctx->segs[i].path, O_RDONLY | O_CLOEXEC);
      if (fd < 0) return set_errorf(TCX_NOT_FOUND, "open failed: %s", ctx->segs[i].path);
      ctx->owned.push_back(fd);
      it = opened.emplace(ctx->segs[i].path, fd).first;
    }
    ctx->fds[i] = it->second;
  }
  return TCX_OK;
}

bool read_stage_range(const FileStageCtx& c, uint64_t a, uint64_t w, uint8_t* dst, ReadBatch& b) {
  const auto& sg = c.segs;
  size_t k = std::partition_point(sg.begin(), sg.end(),
                                  [&](const tcx_file_segment& x) { return x.dst_offset + x.length <= a; }) -
             sg.begin();
  uint64_t pos = a;
  const uint64_t end = a + w;
  while (pos < end) {
    if (k >= sg.size() || sg[k].dst_offset >= end) {
      std::memset(dst + (pos - a), 0, end - pos);
      break;
    }
    const tcx_file_segment& x = sg[k];
    if (x.dst_offset > pos) {
      std::memset(dst + (pos - a), 0, x.dst_offset - pos);
      pos = x.dst_offset;
    }
    const uint64_t e = std::min(end, x.dst_offset + x.length);
    uint64_t got = 0;
    const uint64_t want = e - pos, foff = x.file_offset + (pos - x.dst_offset);
    while (got < want) {
      const ssize_t r = pread(c.fds[k], dst + (pos - a) + got, want - got, static_cast<off_t>(foff + got));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) {
        char msg[512];
        snprintf(msg, sizeof msg, "short read while staging %s at offset %llu (%llu of %llu bytes)", x.path,
                 static_cast<unsigned long long>(foff + got), static_cast<unsigned long long>(got),
                 static_cast<unsigned long long>(want));
        b.fail(TCX_DATA_LOSS, msg);
        return false;
      }
      got += static_cast<uint64_t>(r);
    }
    pos = e;
    ++k;
  }
  return true;
}

tcx_status PieceBuffers::ensure(int n_readers, uint64_t bytes, int n_bufs) {
  if (readers() == n_readers && bufs == n_bufs && buf_bytes >= bytes) return TCX_OK;
  release();
  const uint64_t n = static_cast<uint64_t>(n_readers) * n_bufs;
  if (cudaError_t e = cudaHostAlloc(&host, n * bytes, cudaHostAllocPortable); e != cudaSuccess) {
    cudaGetLastError();
    host = nullptr;
    return set_errorf(TCX_RESOURCE_EXHAUSTED, "pinned piece buffers of %llu bytes: %s",
                      static_cast<unsigned long long>(n * bytes), cuda_msg(e).c_str());
  }
  buf_bytes = bytes;
  bufs = n_bufs;
  for (int t = 0; t < n_readers; ++t) {
    cudaStream_t s;
    TCX_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    streams.push_back(s);
  }
  for (uint64_t i = 0; i < n + n_readers; ++i) {
    cudaEvent_t e;
    TCX_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    (i < n ? copied : marks).push_back(e);
  }
  used.assign(n, 0);
  count.assign(n_readers, 0);
  return TCX_OK;
}

void PieceBuffers::release() {
  sync();
  for (auto* v : {&copied, &marks}) {
    for (cudaEvent_t e : *v) cudaEventDestroy(e);
    v->clear();
  }
  for (cudaStream_t s : streams) cudaStreamDestroy(s);
  streams.clear();
  if (host) cudaFreeHost(host);
  host = nullptr;
  buf_bytes = 0;
  bufs = 0;
  used.clear();
  count.clear();
}

void PieceBuffers::sync() {
  for (cudaStream_t s : streams) cudaStreamSynchronize(s);
}

tcx_status PieceBuffers::wait_on(cudaEvent_t ev) {
  for (cudaStream_t s : streams) TCX_CUDA_TRY(cudaStreamWaitEvent(s, ev, 0));
  return TCX_OK;
}

uint8_t* PieceBuffers::acquire(int t, StageClock::time_point deadline, ReadBatch& b, uint64_t* slot) {
  const uint64_t k = static_cast<uint64_t>(t) * bufs + count[t]++ % bufs;
  if (used[k]) {
    for (;;) {
      const cudaError_t q = cudaEventQuery(copied[k]);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) {
        cudaGetLastError();
        b.fail(TCX_INTERNAL, "host-to-device copy of a staged piece failed: " + cuda_msg(q));
        return nullptr;
      }
      if (StageClock::now() > deadline) {
        b.fail(TCX_DEADLINE_EXCEEDED, "host-to-device copy of a staged piece timed out");
        return nullptr;
      }
      std::this_thread::yield();
    }
  }
  *slot = k;
  return host + k * buf_bytes;
}

bool PieceBuffers::queued(int t, uint64_t slot, ReadBatch& b) {
  if (cudaError_t e = cudaEventRecord(copied[slot], streams[t]); e != cudaSuccess) {
    cudaGetLastError();
    b.fail(TCX_INTERNAL, "recording the copy of staged pieces: " + cuda_msg(e));
    return false;
  }
  used[slot] = 1;
  return true;
}

tcx_status PieceBuffers::join(cudaStream_t s) {
  for (int t = 0; t < readers(); ++t) {
    TCX_CUDA_TRY(cudaEventRecord(marks[t], streams[t]));
    TCX_CUDA_TRY(cudaStreamWaitEvent(s, marks[t], 0));
  }
  return TCX_OK;
}

int reader_for_copies(const PieceBuffers& pb, int device, ReadBatch& b) {
  const int t = reader_index();
  if (t < 0 || t >= pb.readers()) {
    b.fail(TCX_INTERNAL, "staged piece read outside the reader threads");
    return -1;
  }
  if (cudaError_t e = cudaSetDevice(device); e != cudaSuccess) {
    cudaGetLastError();
    b.fail(TCX_INTERNAL, "reader thread cudaSetDevice: " + cuda_msg(e));
    return -1;
  }
  return t;
}

}  // namespace tcx
