// Host-only planning of a collective load: which bytes each rank packs for each
// peer, which it copies locally, where received bytes go, and the view bytes
// no job writes. Pure C++ (no CUDA calls), so it is exercised on the CPU.
//
// Reference behaviour replaced: build_rank_tensor_slice / build_tensor_jobs
// (core/store/replica/collective_disk_loader.cc:834-1003) decide per tensor
// whether a rank receives the full tensor, a dim-0 slice or a dim-1 slice, and
// execute_{replicated,dim0,dim1}_tensor (:4237-4554) move those bytes from one
// root rank. Here every rank owns a leaf-aligned 1/N of the canonical byte
// space and each (rank, peer) pair exchanges exactly the bytes of the peer's
// view that lie in the rank's range, in a fixed order both sides derive from
// the same plan: the peer's jobs in order, each clipped to the range.
#include <algorithm>
#include <cstring>
#include <vector>

#include "tcx_internal.h"

namespace tcx {
namespace {

uint64_t job_total(const tcx_copy_job& j) { return j.rows * j.row_bytes; }

// Appends the parts of j whose source bytes lie in [lo, hi), in row order:
// a partial first row, a block of whole rows, a partial last row.
void clip_job(const tcx_copy_job& j, uint64_t lo, uint64_t hi, std::vector<tcx_copy_job>& out) {
  if (j.rows == 0 || j.row_bytes == 0 || lo >= hi) return;
  const uint64_t W = j.row_bytes;
  const uint64_t P = j.rows > 1 ? j.src_pitch : W;
  const uint64_t s0 = j.src_off;
  if (s0 >= hi) return;
  const uint64_t last_row_end = s0 + (j.rows - 1) * P + W;
  if (last_row_end <= lo) return;
  uint64_t k_first = 0;
  if (s0 + W <= lo) k_first = (lo - s0 - W) / P + 1;  // first row ending after lo
  uint64_t k_last = std::min<uint64_t>(j.rows - 1, (hi - 1 - s0) / P);  // last row starting before hi
  if (k_first > k_last) return;
  auto piece = [&](uint64_t k, uint64_t a, uint64_t b) {  // bytes [a, b) of row k (absolute source)
    const uint64_t sk = s0 + k * P;
    tcx_copy_job p;
    p.src_off = a;
    p.dst_off = j.dst_off + k * j.dst_pitch + (a - sk);
    p.src_pitch = P;
    p.dst_pitch = j.dst_pitch;
    p.row_bytes = b - a;
    p.rows = 1;
    out.push_back(p);
  };
  uint64_t k = k_first;
  {
    const uint64_t sk = s0 + k * P;
    const uint64_t a = std::max(sk, lo), b = std::min(sk + W, hi);
    if (a != sk || b != sk + W) {
      if (b > a) piece(k, a, b);
      ++k;
    }
  }
  if (k > k_last) return;
  uint64_t k_end = k_last;  // inclusive end of the whole-row block
  const uint64_t sl = s0 + k_last * P;
  const bool last_partial = sl + W > hi;
  if (last_partial) {
    if (k_last == k) {
      piece(k, sl, std::min(sl + W, hi));
      return;
    }
    k_end = k_last - 1;
  }
  if (k <= k_end) {
    tcx_copy_job b = j;
    b.src_off = s0 + k * P;
    b.dst_off = j.dst_off + k * j.dst_pitch;
    b.rows = k_end - k + 1;
    if (b.rows == 1) b.src_pitch = P;
    out.push_back(b);
  }
  if (last_partial) piece(k_last, sl, hi);
}

tcx_status validate_plan(const tcx_load_plan* plan, int world) {
  if (plan == nullptr) return set_error(TCX_INVALID_ARGUMENT, "plan is null");
  if (world < 1) return set_error(TCX_INVALID_ARGUMENT, "world must be >= 1");
  if (plan->total_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "total_bytes must be > 0");
  if (plan->leaf_bytes == 0 || plan->leaf_bytes > TCX_MAX_LEAF_BYTES)
    return set_error(TCX_INVALID_ARGUMENT, "leaf_bytes must be in [1, 64 MiB]");
  if (plan->stage_bounds == nullptr || plan->job_offsets == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "stage_bounds and job_offsets are required");
  const uint64_t* b = plan->stage_bounds;
  if (b[0] != 0 || b[world] != plan->total_bytes)
    return set_error(TCX_INVALID_ARGUMENT, "stage_bounds must start at 0 and end at total_bytes");
  for (int r = 0; r < world; ++r) {
    if (b[r + 1] < b[r]) return set_error(TCX_INVALID_ARGUMENT, "stage_bounds must be non-decreasing");
    if (r + 1 < world && b[r + 1] % plan->leaf_bytes != 0)
      return set_error(TCX_INVALID_ARGUMENT, "stage_bounds must be multiples of leaf_bytes");
  }
  const uint64_t n_jobs = plan->job_offsets[world];
  if (plan->job_offsets[0] != 0) return set_error(TCX_INVALID_ARGUMENT, "job_offsets[0] must be 0");
  if (n_jobs > 0 && plan->jobs == nullptr) return set_error(TCX_INVALID_ARGUMENT, "jobs is null");
  for (int r = 0; r < world; ++r)
    if (plan->job_offsets[r + 1] < plan->job_offsets[r])
      return set_error(TCX_INVALID_ARGUMENT, "job_offsets must be non-decreasing");
  for (uint64_t i = 0; i < n_jobs; ++i) {
    const tcx_copy_job& j = plan->jobs[i];
    if (j.rows == 0 || j.row_bytes == 0) continue;
    if (j.rows > 1 && (j.src_pitch < j.row_bytes || j.dst_pitch < j.row_bytes))
      return set_errorf(TCX_INVALID_ARGUMENT, "job %llu: pitches must be >= row_bytes",
                        static_cast<unsigned long long>(i));
    const uint64_t end = j.src_off + (j.rows - 1) * (j.rows > 1 ? j.src_pitch : 0) + j.row_bytes;
    if (end > plan->total_bytes || end < j.src_off)
      return set_errorf(TCX_INVALID_ARGUMENT, "job %llu reads past the canonical byte space",
                        static_cast<unsigned long long>(i));
  }
  return TCX_OK;
}

}  // namespace

tcx_status validate_load_plan(const tcx_load_plan* plan, int world) { return validate_plan(plan, world); }

// Pieces of `jobs` (one rank's view) whose sources lie in [lo, hi).
void clip_jobs(const tcx_copy_job* jobs, uint64_t n, uint64_t lo, uint64_t hi, std::vector<tcx_copy_job>& out) {
  for (uint64_t i = 0; i < n; ++i) clip_job(jobs[i], lo, hi, out);
}

bool pieces_contiguous(const std::vector<tcx_copy_job>& pieces) {
  uint64_t cursor = 0;
  bool first = true;
  for (const auto& p : pieces) {
    if (p.rows > 1 && p.dst_pitch != p.row_bytes) return false;
    if (!first && p.dst_off != cursor) return false;
    cursor = p.dst_off + job_total(p);
    first = false;
  }
  return true;
}

}  // namespace tcx

using namespace tcx;

extern "C" uint64_t tcx_plan_exchange_capacity(const tcx_load_plan* plan, int world) {
  if (plan == nullptr || plan->job_offsets == nullptr || world < 1) return 0;
  const uint64_t n = plan->job_offsets[world];
  uint64_t sparse_rows = 0;
  for (uint64_t i = 0; i < n; ++i)
    if (plan->jobs[i].rows > 1 && plan->jobs[i].dst_pitch != plan->jobs[i].row_bytes) sparse_rows += plan->jobs[i].rows;
  return 3 * n + sparse_rows + 2;
}

extern "C" tcx_status tcx_plan_exchange(const tcx_load_plan* plan, int world, int rank, tcx_exchange_plan* out) {
  tcx_status st = validate_plan(plan, world);
  if (st != TCX_OK) return st;
  if (rank < 0 || rank >= world) return set_error(TCX_INVALID_ARGUMENT, "rank out of range");
  if (out == nullptr || out->pack_jobs == nullptr || out->local_jobs == nullptr || out->scatter_jobs == nullptr ||
      out->send_offsets == nullptr || out->recv_offsets == nullptr || out->recv_view_off == nullptr ||
      out->recv_counts == nullptr ||
      out->direct == nullptr || out->gaps == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "exchange plan output arrays are required");
  const uint64_t* b = plan->stage_bounds;
  const uint64_t* jo = plan->job_offsets;
  const uint64_t lo = b[rank], hi = b[rank + 1];
  std::vector<tcx_copy_job> pieces;
  uint64_t n_pack = 0, n_local = 0, n_scatter = 0;

  // Sends: for every peer q, q's view bytes that lie in my staged range.
  out->send_offsets[0] = 0;
  for (int q = 0; q < world; ++q) {
    pieces.clear();
    clip_jobs(plan->jobs + jo[q], jo[q + 1] - jo[q], lo, hi, pieces);
    uint64_t pos = out->send_offsets[q];
    for (auto p : pieces) {
      p.src_off -= lo;
      if (q == rank) {
        out->local_jobs[n_local++] = p;
      } else {
        p.dst_off = pos;
        p.dst_pitch = p.row_bytes;
        pos += job_total(p);
        out->pack_jobs[n_pack++] = p;
      }
    }
    out->send_offsets[q + 1] = pos;
  }

  // Receives: my view bytes that lie in each peer's range.
  out->recv_offsets[0] = 0;
  for (int p = 0; p < world; ++p) {
    out->direct[p] = 0;
    out->recv_view_off[p] = 0;
    uint64_t off = out->recv_offsets[p];
    if (p != rank) {
      pieces.clear();
      clip_jobs(plan->jobs + jo[rank], jo[rank + 1] - jo[rank], b[p], b[p + 1], pieces);
      uint64_t bytes = 0;
      for (const auto& q : pieces) bytes += job_total(q);
      if (!pieces.empty() && pieces_contiguous(pieces)) {
        out->direct[p] = 1;
        out->recv_view_off[p] = pieces.front().dst_off;
      } else {
        uint64_t pos = off;
        for (const auto& q : pieces) {
          tcx_copy_job s = q;
          s.src_off = pos;
          s.src_pitch = q.row_bytes;
          pos += job_total(q);
          out->scatter_jobs[n_scatter++] = s;
        }
        off += bytes;
      }
      out->recv_counts[p] = bytes;
    } else {
      out->recv_counts[p] = 0;
    }
    out->recv_offsets[p + 1] = off;
  }

  // View bytes no job of this rank writes.
  std::vector<std::pair<uint64_t, uint64_t>> iv;
  for (uint64_t i = jo[rank]; i < jo[rank + 1]; ++i) {
    const tcx_copy_job& j = plan->jobs[i];
    if (j.rows == 0 || j.row_bytes == 0) continue;
    if (j.rows == 1 || j.dst_pitch == j.row_bytes) {
      iv.emplace_back(j.dst_off, j.dst_off + job_total(j));
    } else {
      for (uint64_t k = 0; k < j.rows; ++k) iv.emplace_back(j.dst_off + k * j.dst_pitch, j.dst_off + k * j.dst_pitch + j.row_bytes);
    }
  }
  std::sort(iv.begin(), iv.end());
  uint64_t cursor = 0, n_gaps = 0;
  for (const auto& [a, e] : iv) {
    if (a > cursor) {
      out->gaps[2 * n_gaps] = cursor;
      out->gaps[2 * n_gaps + 1] = a - cursor;
      ++n_gaps;
    }
    cursor = std::max(cursor, e);
  }
  if (plan->view_bytes > cursor) {
    out->gaps[2 * n_gaps] = cursor;
    out->gaps[2 * n_gaps + 1] = plan->view_bytes - cursor;
    ++n_gaps;
  }
  out->n_pack = n_pack;
  out->n_local = n_local;
  out->n_scatter = n_scatter;
  out->n_gaps = n_gaps;
  return TCX_OK;
}

extern "C" uint64_t tcx_plan_push_split_capacity(const tcx_load_plan* plan, int world) {
  if (plan == nullptr || plan->job_offsets == nullptr || world < 1) return 0;
  return 3 * plan->job_offsets[world] * static_cast<uint64_t>(world) + 2;
}

extern "C" tcx_status tcx_plan_push_split(const tcx_load_plan* plan, int world, int rank, uint64_t nccl_permille,
                                          tcx_copy_job* nccl_jobs, uint64_t* nccl_job_offsets, tcx_copy_job* ce_jobs,
                                          uint64_t* ce_offsets, uint64_t capacity) {
  tcx_status st = validate_plan(plan, world);
  if (st != TCX_OK) return st;
  if (rank < 0 || rank >= world) return set_error(TCX_INVALID_ARGUMENT, "rank out of range");
  if (nccl_jobs == nullptr || nccl_job_offsets == nullptr || ce_jobs == nullptr || ce_offsets == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "push split output arrays are required");
  const uint64_t share = std::min<uint64_t>(nccl_permille, 1000);
  const uint64_t* b = plan->stage_bounds;
  const uint64_t* jo = plan->job_offsets;
  const uint64_t lo = b[rank];
  std::vector<tcx_copy_job> pieces;
  uint64_t n_nccl = 0, n_ce = 0;
  for (int r = 0; r < world; ++r) {
    nccl_job_offsets[r] = n_nccl;
    ce_offsets[r] = n_ce;
    for (int p = 0; p < world; ++p) {
      if (p == r) continue;
      pieces.clear();
      clip_jobs(plan->jobs + jo[r], jo[r + 1] - jo[r], b[p], b[p + 1], pieces);
      uint64_t total = 0;
      for (const auto& j : pieces) total += job_total(j);
      const uint64_t want = (total * share + 999) / 1000;
      uint64_t acc = 0;
      for (auto j : pieces) {
        if (acc < want) {
          acc += job_total(j);
          if (n_nccl >= capacity) return set_error(TCX_INVALID_ARGUMENT, "push split capacity too small");
          nccl_jobs[n_nccl++] = j;
        } else if (p == rank) {
          j.src_off -= lo;
          if (n_ce >= capacity) return set_error(TCX_INVALID_ARGUMENT, "push split capacity too small");
          ce_jobs[n_ce++] = j;
        }
      }
    }
  }
  nccl_job_offsets[world] = n_nccl;
  ce_offsets[world] = n_ce;
  return TCX_OK;
}
