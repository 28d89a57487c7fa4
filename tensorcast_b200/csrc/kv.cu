// Paged KV-cache gather on sm_100a: pages scattered in a pool -> one contiguous
// buffer per sequence, laid out [plane][token][token_bytes] (plane = layer x K/V).
//
// There is no reference implementation of this step (the reference treats
// engine-owned KV as opaque byte artifacts); the layout follows the usual paged
// KV cache: pool page p of plane k at pool + (k * pool_pages + p) * page_bytes,
// page_tokens tokens of token_bytes each, a per-sequence page table of slots.
//
// kv_gather_kernel is a persistent grid over (sequence, plane, page) work items.
// Sequence s owns items [planes * page_offsets[s], planes * page_offsets[s+1]),
// so a binary search of page_offsets finds it; one CTA moves one page (up to
// page_tokens * token_bytes bytes) with 16-byte streaming loads and stores when
// everything is 16-byte aligned. Every index read from the tables is checked
// before it is used: a bad slot, a page past the sequence's tokens or an output
// past out_bytes skips the copy and records a code in *status.
#include <cuda_runtime.h>

#include "tcx_internal.h"

namespace tcx {
namespace {

constexpr int kKvThreads = 256;

struct KvArgs {
  const uint8_t* pool;
  uint8_t* out;
  const uint32_t* page_table;
  const uint64_t* page_offsets;
  const uint32_t* seq_tokens;
  const uint64_t* out_offsets;
  uint64_t n_seq, pool_pages, token_bytes, out_bytes, total_items;
  uint32_t planes, page_tokens;
  uint32_t* status;
};

__global__ void __launch_bounds__(kKvThreads) kv_gather_kernel(KvArgs a) {
  __shared__ uint64_t s_seq;
  const bool vec = ((reinterpret_cast<uintptr_t>(a.pool) | reinterpret_cast<uintptr_t>(a.out) | a.token_bytes) &
                    15u) == 0;
  for (uint64_t w = blockIdx.x; w < a.total_items; w += gridDim.x) {
    if (threadIdx.x == 0) {
      const uint64_t page = w / a.planes;  // global page index: page_offsets[s] <= page < page_offsets[s+1]
      uint64_t lo = 0, hi = a.n_seq;
      while (hi - lo > 1) {
        const uint64_t mid = (lo + hi) / 2;
        if (a.page_offsets[mid] <= page) lo = mid; else hi = mid;
      }
      s_seq = lo;
    }
    __syncthreads();
    const uint64_t s = s_seq;
    __syncthreads();
    const uint64_t p0 = a.page_offsets[s], pages = a.page_offsets[s + 1] - p0;
    const uint64_t local = w - static_cast<uint64_t>(a.planes) * p0;
    const uint64_t plane = local / pages, j = local % pages;
    const uint64_t tokens = a.seq_tokens[s];
    const uint32_t slot = a.page_table[p0 + j];
    const uint64_t first_tok = j * a.page_tokens;
    bool ok = true;
    if (slot >= a.pool_pages) {
      ok = false;
      if (threadIdx.x == 0) atomicCAS(a.status, 0u, 1u);
    } else if (first_tok >= tokens) {
      ok = false;
      if (threadIdx.x == 0) atomicCAS(a.status, 0u, 2u);
    }
    const uint64_t ntok = ok ? min(static_cast<uint64_t>(a.page_tokens), tokens - first_tok) : 0;
    const uint64_t bytes = ntok * a.token_bytes;
    const uint64_t dst_off = a.out_offsets[s] + (plane * tokens + first_tok) * a.token_bytes;
    if (ok && dst_off + bytes > a.out_bytes) {
      ok = false;
      if (threadIdx.x == 0) atomicCAS(a.status, 0u, 3u);
    }
    if (ok) {
      const uint8_t* src = a.pool + (plane * a.pool_pages + slot) * (a.page_tokens * a.token_bytes);
      uint8_t* dst = a.out + dst_off;
      if (vec && (dst_off & 15u) == 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        for (uint64_t k = threadIdx.x; k < bytes / 16; k += blockDim.x) __stcs(d4 + k, __ldcs(s4 + k));
      } else {
        for (uint64_t k = threadIdx.x; k < bytes; k += blockDim.x) dst[k] = src[k];
      }
    }
  }
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" tcx_status tcx_kv_gather(const void* d_pool, uint32_t planes, uint64_t pool_pages, uint32_t page_tokens,
                                    uint64_t token_bytes, const uint32_t* d_page_table, const uint64_t* d_page_offsets,
                                    const uint32_t* d_seq_tokens, const uint64_t* d_out_offsets, uint64_t n_seq,
                                    uint64_t total_pages, void* d_out, uint64_t out_bytes, uint32_t* d_status,
                                    void* stream) {
  if (n_seq == 0 || total_pages == 0) return TCX_OK;
  if (d_pool == nullptr || d_page_table == nullptr || d_page_offsets == nullptr || d_seq_tokens == nullptr ||
      d_out_offsets == nullptr || d_out == nullptr || d_status == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "null device pointer");
  if (planes == 0 || page_tokens == 0 || token_bytes == 0 || pool_pages == 0)
    return set_error(TCX_INVALID_ARGUMENT, "planes, page_tokens, token_bytes and pool_pages must be > 0");
  if (pool_pages > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "pool_pages exceeds 2^32");
  int dev = 0, sms = 148;
  TCX_CUDA_TRY(cudaGetDevice(&dev));
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  KvArgs a{static_cast<const uint8_t*>(d_pool), static_cast<uint8_t*>(d_out), d_page_table, d_page_offsets,
           d_seq_tokens, d_out_offsets, n_seq, pool_pages, token_bytes, out_bytes,
           static_cast<uint64_t>(planes) * total_pages, planes, page_tokens, d_status};
  const uint64_t grid = std::min<uint64_t>(a.total_items, static_cast<uint64_t>(sms) * 8);
  kv_gather_kernel<<<static_cast<unsigned>(grid), kKvThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  note_launches(1);
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}
