// Host reads of file segments into (pinned) memory for the staging pipeline.
//
// Segments name a file range and its place in the destination. They are cut
// into pieces of at most 64 MiB, put in source order (file, then offset: the
// payload order of a safetensors file, which differs from the canonical order
// the caller lists them in) and spread over a pool of threads, so every thread
// reads forward through its files (the source-ordered windows of the
// reference's safetensors reader, collective_disk_loader.cc:1571-2200).
//
// TCX_READ_DIRECT bypasses the page cache (O_DIRECT) for cold reads from a
// block device: O_DIRECT needs 4 KiB-aligned file offsets, lengths and buffer
// addresses, which arbitrary tensor ranges do not have, so nearby pieces of a
// file (gaps up to 256 KiB) are grouped into windows of at most 16 MiB, each
// window is read block-aligned into a per-thread aligned bounce buffer and its
// pieces are copied out to their destinations. A file system that refuses
// O_DIRECT (tmpfs) is read buffered instead.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "tcx_internal.h"

namespace tcx {
namespace {

constexpr uint64_t kPiece = 64ull << 20;
constexpr uint64_t kAlign = 4096;
constexpr uint64_t kDirectWindow = 16ull << 20;
constexpr uint64_t kDirectGap = 256ull << 10;

struct Piece {
  const char* path;
  uint64_t file_off, dst_off, len;
};

// A run of pieces of one file read together; [begin, end) of the piece list.
struct Window {
  size_t begin, end;
};

struct Fd {
  int fd = -1;
  std::string path;
  bool direct = false;
  ~Fd() {
    if (fd >= 0) close(fd);
  }
  // Opens `p` (O_DIRECT when asked and accepted); false on failure.
  bool open_for(const char* p, bool want_direct) {
    if (fd >= 0 && path == p && direct == want_direct) return true;
    if (fd >= 0) close(fd);
    fd = -1;
    path = p;
    direct = false;
    if (want_direct) {
      fd = ::open(p, O_RDONLY | O_CLOEXEC | O_DIRECT);
      if (fd >= 0) {
        direct = true;
        return true;
      }
      if (errno != EINVAL) return false;
    }
    fd = ::open(p, O_RDONLY | O_CLOEXEC);
    return fd >= 0;
  }
};

bool read_full(int fd, uint8_t* dst, uint64_t len, uint64_t off, uint64_t* got_out) {
  uint64_t got = 0;
  while (got < len) {
    const ssize_t r = pread(fd, dst + got, len - got, off + got);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) break;
    got += static_cast<uint64_t>(r);
  }
  *got_out = got;
  return got == len;
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" tcx_status tcx_read_segments_ex(const tcx_file_segment* segs, uint64_t n, void* dst, int threads,
                                           uint64_t flags) {
  if (n == 0) return TCX_OK;
  if (segs == nullptr || dst == nullptr) return set_error(TCX_INVALID_ARGUMENT, "null pointer");
  const bool direct = (flags & TCX_READ_DIRECT) != 0;
  // A direct-read piece must fit one bounce window with its block-alignment head.
  const uint64_t piece_max = direct ? kDirectWindow - kAlign : kPiece;
  std::vector<Piece> pieces;
  for (uint64_t i = 0; i < n; ++i) {
    if (segs[i].length && segs[i].path == nullptr) return set_error(TCX_INVALID_ARGUMENT, "segment without a path");
    for (uint64_t o = 0; o < segs[i].length; o += piece_max)
      pieces.push_back({segs[i].path, segs[i].file_offset + o, segs[i].dst_offset + o,
                        std::min(piece_max, segs[i].length - o)});
  }
  if (pieces.empty()) return TCX_OK;
  std::stable_sort(pieces.begin(), pieces.end(), [](const Piece& a, const Piece& b) {
    const int c = std::strcmp(a.path, b.path);
    return c != 0 ? c < 0 : a.file_off < b.file_off;
  });
  std::vector<Window> windows;
  for (size_t i = 0; i < pieces.size();) {
    size_t j = i + 1;
    if (direct) {
      const uint64_t w0 = pieces[i].file_off & ~(kAlign - 1);
      while (j < pieces.size() && std::strcmp(pieces[j].path, pieces[i].path) == 0) {
        const uint64_t prev_end = pieces[j - 1].file_off + pieces[j - 1].len;
        const uint64_t end = pieces[j].file_off + pieces[j].len;
        if (pieces[j].file_off < prev_end || pieces[j].file_off - prev_end > kDirectGap || end - w0 > kDirectWindow)
          break;
        ++j;
      }
    }
    windows.push_back({i, j});
    i = j;
  }
  const int nt = std::max(1, std::min<int>(threads, static_cast<int>(windows.size())));
  std::atomic<uint64_t> next{0};
  std::atomic<int> status{TCX_OK};
  std::vector<std::string> errors(nt);
  auto* out = static_cast<uint8_t*>(dst);
  auto worker = [&](int t) {
    Fd f;
    uint8_t* bounce = nullptr;
    for (uint64_t k = next++; k < windows.size() && status.load() == TCX_OK; k = next++) {
      const Window& w = windows[k];
      const Piece& first = pieces[w.begin];
      if (!f.open_for(first.path, direct)) {
        errors[t] = std::string("open failed: ") + first.path + ": " + std::strerror(errno);
        status = TCX_NOT_FOUND;
        break;
      }
      if (!f.direct) {
        for (size_t i = w.begin; i < w.end; ++i) {
          uint64_t got = 0;
          if (!read_full(f.fd, out + pieces[i].dst_off, pieces[i].len, pieces[i].file_off, &got)) {
            errors[t] = std::string("short read while loading source: ") + pieces[i].path;
            status = TCX_DATA_LOSS;
            break;
          }
        }
        continue;
      }
      // Block-aligned window into the bounce buffer, then each piece to its place.
      const uint64_t w0 = first.file_off & ~(kAlign - 1);
      const uint64_t need = pieces[w.end - 1].file_off + pieces[w.end - 1].len;
      const uint64_t w1 = (need + kAlign - 1) & ~(kAlign - 1);
      if (bounce == nullptr && posix_memalign(reinterpret_cast<void**>(&bounce), kAlign, kDirectWindow + 2 * kAlign) != 0) {
        bounce = nullptr;
        errors[t] = "out of host memory for the direct-read buffer";
        status = TCX_RESOURCE_EXHAUSTED;
        break;
      }
      uint64_t got = 0;
      read_full(f.fd, bounce, w1 - w0, w0, &got);  // may stop at end of file
      if (got < need - w0) {
        errors[t] = std::string("short read while loading source: ") + first.path;
        status = TCX_DATA_LOSS;
        break;
      }
      for (size_t i = w.begin; i < w.end; ++i)
        std::memcpy(out + pieces[i].dst_off, bounce + (pieces[i].file_off - w0), pieces[i].len);
    }
    std::free(bounce);
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; ++t) pool.emplace_back(worker, t);
  worker(0);
  for (auto& th : pool) th.join();
  if (status != TCX_OK) {
    for (const auto& e : errors)
      if (!e.empty()) return set_error(status, e);
  }
  return status;
}

extern "C" tcx_status tcx_read_segments(const tcx_file_segment* segs, uint64_t n, void* dst, int threads) {
  return tcx_read_segments_ex(segs, n, dst, threads, 0);
}
