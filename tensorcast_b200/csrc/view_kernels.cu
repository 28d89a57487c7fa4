// View materialisation on sm_100a: batched strided byte copies and permutes.
//
// A view of a canonical byte space (view_planner.cc:358-668 in the reference)
// is a list of copies: an identity or dim-0 narrowed tensor is one contiguous
// row, a narrow along dim d > 0 is outer(d) rows of len*inner*esize bytes at a
// constant source pitch, and a transposed tensor is a full copy followed by a
// permute (view_transform_executor.cc:74-133 does permute().contiguous()).
// Every copy is a "copy job" (rows x row_bytes, source and destination pitch).
// The same jobs, clipped to a rank's staged byte range and re-based, pack the
// bytes a peer needs into a send buffer.
//
// copy_jobs_kernel is a persistent grid over (job, 32 KiB chunk) work items:
// item w is found by binary search over a device prefix of per-job chunk
// counts, so tensors of 8 KiB and 1 GiB share one launch with even load.
// Rows are moved as 16-byte vectors when every offset, pitch and length of the
// job is 16-byte aligned, otherwise byte by byte.
//
// 2-D transposes of 1- and 2-byte elements go through transpose2d_packed_kernel
// (element blocks transposed in registers into 32-bit words, a swizzled word
// tile, 16-byte global accesses on both sides), 4- and 8-byte elements through
// 64x64-element padded tiles; other permutations use a generic gather.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "tcx_internal.h"

namespace tcx {
namespace {

constexpr uint32_t kCopyChunk = 32 * 1024;  // bytes per work item
constexpr int kCopyThreads = 256;

__device__ __forceinline__ uint64_t job_bytes(const tcx_copy_job& j) { return j.rows * j.row_bytes; }

// prefix[k] = number of work items of jobs [0, k); prefix[n] = total.
__global__ void copy_prefix_kernel(const tcx_copy_job* __restrict__ jobs, uint64_t n, uint64_t* __restrict__ prefix) {
  // One CTA: block-wide scan in tiles of blockDim.x.
  __shared__ uint64_t tile[1024];
  __shared__ uint64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (uint64_t base = 0; base < n; base += blockDim.x) {
    const uint64_t k = base + threadIdx.x;
    uint64_t v = 0;
    if (k < n) v = (job_bytes(jobs[k]) + kCopyChunk - 1) / kCopyChunk;
    tile[threadIdx.x] = v;
    __syncthreads();
    for (uint32_t off = 1; off < blockDim.x; off <<= 1) {
      const uint64_t add = threadIdx.x >= off ? tile[threadIdx.x - off] : 0;
      __syncthreads();
      tile[threadIdx.x] += add;
      __syncthreads();
    }
    if (k < n) prefix[k + 1] = carry + tile[threadIdx.x];
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry += tile[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x == 0) prefix[0] = 0;
}

__device__ __forceinline__ uint64_t find_job(const uint64_t* prefix, uint64_t n, uint64_t w) {
  uint64_t lo = 0, hi = n;  // prefix[lo] <= w < prefix[hi]
  while (hi - lo > 1) {
    const uint64_t mid = (lo + hi) / 2;
    if (prefix[mid] <= w) lo = mid; else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(kCopyThreads) copy_jobs_kernel(const uint8_t* __restrict__ src,
                                                                 uint8_t* __restrict__ dst,
                                                                 const tcx_copy_job* __restrict__ jobs, uint64_t n,
                                                                 const uint64_t* __restrict__ prefix) {
  __shared__ uint64_t s_job;
  const uint64_t total = prefix[n];
  for (uint64_t w = blockIdx.x; w < total; w += gridDim.x) {
    if (threadIdx.x == 0) s_job = find_job(prefix, n, w);
    __syncthreads();
    const uint64_t ji = s_job;
    __syncthreads();
    if (ji >= n) continue;  // inconsistent prefix: never index past the job table
    const tcx_copy_job j = jobs[ji];
    const uint64_t bytes = j.rows * j.row_bytes;
    const uint64_t c0 = (w - prefix[ji]) * kCopyChunk;
    if (w < prefix[ji] || c0 >= bytes) continue;  // never copy outside the job
    const uint64_t c1 = min(c0 + kCopyChunk, bytes);
    const bool vec = ((j.src_off | j.dst_off | j.src_pitch | j.dst_pitch | j.row_bytes) & 15u) == 0 &&
                     ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0;
    if (vec) {
      const uint32_t upr = static_cast<uint32_t>(j.row_bytes >> 4);  // 16-byte units per row
      const uint64_t u0 = c0 >> 4;
      const uint64_t row0 = u0 / upr;
      const uint32_t col0 = static_cast<uint32_t>(u0 - row0 * upr);
      const uint32_t units = static_cast<uint32_t>((c1 - c0) >> 4);
      // Four 16-byte loads in flight per thread before their stores.
      constexpr int kBatch = 4;
      for (uint32_t base = threadIdx.x; base < units; base += blockDim.x * kBatch) {
        uint4 v[kBatch];
        uint64_t doff[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
          const uint32_t u = base + k * blockDim.x;
          if (u < units) {
            const uint32_t t = col0 + u;
            const uint32_t dr = t / upr;
            const uint32_t col = t - dr * upr;
            const uint64_t row = row0 + dr;
            v[k] = __ldcs(reinterpret_cast<const uint4*>(src + j.src_off + row * j.src_pitch) + col);
            doff[k] = j.dst_off + row * j.dst_pitch + 16ull * col;
          }
        }
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
          if (base + k * blockDim.x < units) __stcs(reinterpret_cast<uint4*>(dst + doff[k]), v[k]);
        }
      }
    } else {
      for (uint64_t b = c0 + threadIdx.x; b < c1; b += blockDim.x) {
        const uint64_t row = b / j.row_bytes;
        const uint64_t col = b - row * j.row_bytes;
        dst[j.dst_off + row * j.dst_pitch + col] = src[j.src_off + row * j.src_pitch + col];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Permutes.
// ---------------------------------------------------------------------------
constexpr int kTile = 64;  // elements per tile side

template <typename T>
struct VecOf {
  static constexpr int kPer = 16 / sizeof(T);  // elements per 16-byte vector
};

// dst[c][r] = src[r][c] for a [rows, cols] tensor; 64x64 tiles, 256 threads.
template <typename T>
__global__ void __launch_bounds__(256) transpose2d_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                          uint64_t rows, uint64_t cols, bool vec) {
  constexpr int V = VecOf<T>::kPer;
  __shared__ T tile[kTile][kTile + 16 / sizeof(T) + 1];
  const uint64_t tiles_c = (cols + kTile - 1) / kTile;
  const uint64_t tr = blockIdx.x / tiles_c, tc = blockIdx.x % tiles_c;
  const uint64_t r0 = tr * kTile, c0 = tc * kTile;
  const bool full = r0 + kTile <= rows && c0 + kTile <= cols;
  if (vec && full) {
    constexpr int VPR = kTile / V;  // vectors per tile row
    for (int k = threadIdx.x; k < kTile * VPR; k += blockDim.x) {
      const int r = k / VPR, cv = k % VPR;
      const uint4 v = *reinterpret_cast<const uint4*>(src + (r0 + r) * cols + c0 + cv * V);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int q = 0; q < V; ++q) tile[r][cv * V + q] = e[q];
    }
    __syncthreads();
    for (int k = threadIdx.x; k < kTile * VPR; k += blockDim.x) {
      const int c = k / VPR, rv = k % VPR;
      uint4 v;
      T* e = reinterpret_cast<T*>(&v);
#pragma unroll
      for (int q = 0; q < V; ++q) e[q] = tile[rv * V + q][c];
      *reinterpret_cast<uint4*>(dst + (c0 + c) * rows + r0 + rv * V) = v;
    }
  } else {
    for (int k = threadIdx.x; k < kTile * kTile; k += blockDim.x) {
      const int r = k / kTile, c = k % kTile;
      if (r0 + r < rows && c0 + c < cols) tile[r][c] = src[(r0 + r) * cols + c0 + c];
    }
    __syncthreads();
    for (int k = threadIdx.x; k < kTile * kTile; k += blockDim.x) {
      const int c = k / kTile, r = k % kTile;
      if (r0 + r < rows && c0 + c < cols) dst[(c0 + c) * rows + r0 + r] = tile[r][c];
    }
  }
}

// Packed-word transpose for 1- and 2-byte elements (P = 4 or 2 elements per
// 32-bit word). A tile is 32*P source rows by 32*P source columns: 32 row
// groups of P rows, each source row segment 128 bytes (8 chunks of 16 bytes).
// Phase 1: thread (group g, chunk q) loads the chunk from the P rows of its
// group (P 16-byte loads) and transposes them in registers with byte permutes
// into 4*P words, word j = the P elements of source column j, one per row, in
// row order, i.e. P consecutive elements of output row j. Words land in a
// shared tile W[column][group] whose group index is XOR-swizzled by 4*(chunk)
// so the 32 lanes of a store hit 32 distinct banks.
// Phase 2: each 16-byte output chunk (4 consecutive groups) is one swizzled,
// 16-byte-aligned shared load and one 16-byte global store; 8 lanes cover 128
// contiguous bytes of an output row.
// Full tiles only, and only when every row start is 16-byte aligned on both
// sides; edge tiles copy element by element.
template <int P>
struct PackedElem;
template <>
struct PackedElem<2> {
  using T = uint16_t;
};
template <>
struct PackedElem<4> {
  using T = uint8_t;
};

template <int P>
__device__ __forceinline__ void transpose_words(const uint32_t (&in)[P], uint32_t (&out)[P]);

template <>
__device__ __forceinline__ void transpose_words<2>(const uint32_t (&in)[2], uint32_t (&out)[2]) {
  out[0] = __byte_perm(in[0], in[1], 0x5410);  // low halves: element 0 of rows 0, 1
  out[1] = __byte_perm(in[0], in[1], 0x7632);  // high halves: element 1 of rows 0, 1
}

template <>
__device__ __forceinline__ void transpose_words<4>(const uint32_t (&in)[4], uint32_t (&out)[4]) {
  const uint32_t t0 = __byte_perm(in[0], in[1], 0x5140);  // (r0.b0, r1.b0, r0.b1, r1.b1)
  const uint32_t t1 = __byte_perm(in[2], in[3], 0x5140);  // (r2.b0, r3.b0, r2.b1, r3.b1)
  const uint32_t t2 = __byte_perm(in[0], in[1], 0x7362);  // (r0.b2, r1.b2, r0.b3, r1.b3)
  const uint32_t t3 = __byte_perm(in[2], in[3], 0x7362);  // (r2.b2, r3.b2, r2.b3, r3.b3)
  out[0] = __byte_perm(t0, t1, 0x5410);
  out[1] = __byte_perm(t0, t1, 0x7632);
  out[2] = __byte_perm(t2, t3, 0x5410);
  out[3] = __byte_perm(t2, t3, 0x7632);
}

template <int P, int G>
__global__ void __launch_bounds__(256) transpose2d_packed_kernel(const typename PackedElem<P>::T* __restrict__ src,
                                                                 typename PackedElem<P>::T* __restrict__ dst,
                                                                 uint64_t rows, uint64_t cols, bool vec) {
  using T = typename PackedElem<P>::T;
  constexpr int TR = 32 * P;      // source rows of one tile
  constexpr int R = TR * G;       // a CTA takes G tiles stacked along the rows
  constexpr int C = 32 * P;       // source columns of a tile
  constexpr int CPQ = 4 * P;      // columns per 16-byte chunk
  __shared__ __align__(16) uint32_t W[G][C][32];
  const uint64_t tiles_c = (cols + C - 1) / C;
  const uint64_t tr = blockIdx.x / tiles_c, tc = blockIdx.x % tiles_c;
  const uint64_t r0 = tr * R, c0 = tc * C;
  if (vec && r0 + R <= rows && c0 + C <= cols) {
    const int q = threadIdx.x & 7, g = threadIdx.x >> 3;
    uint4 v[G][P];  // every load of the CTA's tiles in flight before the first shared store
#pragma unroll
    for (int t = 0; t < G; ++t)
#pragma unroll
      for (int k = 0; k < P; ++k)
        v[t][k] = *reinterpret_cast<const uint4*>(src + (r0 + t * TR + P * g + k) * cols + c0 + q * CPQ);
    const int phys = g ^ (4 * q);
#pragma unroll
    for (int t = 0; t < G; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t in[P], out[P];
#pragma unroll
        for (int k = 0; k < P; ++k) in[k] = reinterpret_cast<const uint32_t*>(&v[t][k])[i];
        transpose_words<P>(in, out);
#pragma unroll
        for (int k = 0; k < P; ++k) W[t][q * CPQ + i * P + k][phys] = out[k];
      }
    __syncthreads();
    // item m: output row j, tile t, chunk c; 8*G consecutive lanes cover G*128
    // contiguous bytes of one output row.
#pragma unroll
    for (int m = threadIdx.x; m < G * C * 8; m += 256) {
      const int c = m & 7, t = (m >> 3) % G, j = (m >> 3) / G;
      const uint4 o = *reinterpret_cast<const uint4*>(&W[t][j][4 * (c ^ ((j / CPQ) & 7))]);
      *reinterpret_cast<uint4*>(dst + (c0 + j) * rows + r0 + t * TR + c * CPQ) = o;
    }
  } else {
    const uint64_t nr = rows - r0 < static_cast<uint64_t>(R) ? rows - r0 : R;
    const uint64_t nc = cols - c0 < static_cast<uint64_t>(C) ? cols - c0 : C;
    for (uint64_t k = threadIdx.x; k < nr * nc; k += blockDim.x) {
      const uint64_t j = k / nr, r = k % nr;
      dst[(c0 + j) * rows + r0 + r] = src[(r0 + r) * cols + c0 + j];
    }
  }
}

struct PermuteParams {
  uint32_t ndim;
  uint64_t out_shape[TCX_MAX_DIMS];
  uint64_t in_stride_of_out_dim[TCX_MAX_DIMS];  // source element stride of each output dimension
};

// Generic permute: one thread per output element.
template <typename T>
__global__ void permute_generic_kernel(const T* __restrict__ src, T* __restrict__ dst, uint64_t numel,
                                       PermuteParams pp) {
  for (uint64_t o = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; o < numel;
       o += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    uint64_t rem = o, in = 0;
    for (int d = static_cast<int>(pp.ndim) - 1; d >= 0; --d) {
      const uint64_t idx = rem % pp.out_shape[d];
      rem /= pp.out_shape[d];
      in += idx * pp.in_stride_of_out_dim[d];
    }
    dst[o] = src[in];
  }
}

template <typename T>
tcx_status launch_permute_t(const uint8_t* src, uint8_t* dst, const tcx_permute_job& pj, cudaStream_t stream) {
  uint64_t numel = 1;
  for (uint32_t d = 0; d < pj.ndim; ++d) numel *= static_cast<uint64_t>(pj.shape[d]);
  if (numel == 0) return TCX_OK;
  const T* s = reinterpret_cast<const T*>(src + pj.src_off);
  T* o = reinterpret_cast<T*>(dst + pj.dst_off);
  if (pj.ndim == 2 && pj.perm[0] == 1 && pj.perm[1] == 0) {
    const uint64_t rows = pj.shape[0], cols = pj.shape[1];
    const bool vec = ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(o)) & 15u) == 0 &&
                     (rows * sizeof(T)) % 16 == 0 && (cols * sizeof(T)) % 16 == 0;
    if constexpr (sizeof(T) <= 2) {
      // 16 KiB of loads in flight per CTA: two 64x64 tiles of 2-byte elements, one 128x128 of 1-byte.
      constexpr int P = 4 / sizeof(T), G = P == 2 ? 2 : 1, E = 32 * P;
      const uint64_t tiles = ((rows + E * G - 1) / (E * G)) * ((cols + E - 1) / E);
      if (tiles > 0x7fffffffull) return set_error(TCX_INVALID_ARGUMENT, "tensor too large to permute");
      transpose2d_packed_kernel<P, G><<<static_cast<unsigned>(tiles), 256, 0, stream>>>(s, o, rows, cols, vec);
    } else {
      const uint64_t tiles = ((rows + kTile - 1) / kTile) * ((cols + kTile - 1) / kTile);
      if (tiles > 0x7fffffffull) return set_error(TCX_INVALID_ARGUMENT, "tensor too large to permute");
      transpose2d_kernel<T><<<static_cast<unsigned>(tiles), 256, 0, stream>>>(s, o, rows, cols, vec);
    }
    note_launches(1);
  } else {
    PermuteParams pp{};
    pp.ndim = pj.ndim;
    uint64_t in_stride[TCX_MAX_DIMS];
    uint64_t acc = 1;
    for (int d = static_cast<int>(pj.ndim) - 1; d >= 0; --d) {
      in_stride[d] = acc;
      acc *= static_cast<uint64_t>(pj.shape[d]);
    }
    for (uint32_t d = 0; d < pj.ndim; ++d) {
      pp.out_shape[d] = static_cast<uint64_t>(pj.shape[pj.perm[d]]);
      pp.in_stride_of_out_dim[d] = in_stride[pj.perm[d]];
    }
    const unsigned grid = static_cast<unsigned>(std::min<uint64_t>((numel + 255) / 256, sm_count() * 16ull));
    permute_generic_kernel<T><<<grid, 256, 0, stream>>>(s, o, numel, pp);
    note_launches(1);
  }
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

}  // namespace

// SM count of the current device (cached per thread).
int sm_count() {
  static thread_local int dev_cached = -1, sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev != dev_cached) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    dev_cached = dev;
  }
  return sms;
}

tcx_status launch_copy_jobs(const void* d_src, void* d_dst, const tcx_copy_job* d_jobs, uint64_t n_jobs,
                            uint64_t* d_prefix, cudaStream_t stream, uint32_t max_ctas) {
  if (n_jobs == 0) return TCX_OK;
  copy_prefix_kernel<<<1, 1024, 0, stream>>>(d_jobs, n_jobs, d_prefix);
  note_launches(1);
  TCX_CUDA_TRY(cudaGetLastError());
  unsigned grid = static_cast<unsigned>(sm_count()) * 8u;
  if (max_ctas) grid = std::min<unsigned>(grid, max_ctas);
  copy_jobs_kernel<<<grid, kCopyThreads, 0, stream>>>(static_cast<const uint8_t*>(d_src),
                                                      static_cast<uint8_t*>(d_dst), d_jobs, n_jobs, d_prefix);
  note_launches(1);
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

tcx_status check_permute(const tcx_permute_job& pj) {
  if (pj.ndim == 0 || pj.ndim > TCX_MAX_DIMS) return set_error(TCX_INVALID_ARGUMENT, "permute ndim out of range");
  bool seen[TCX_MAX_DIMS] = {};
  for (uint32_t d = 0; d < pj.ndim; ++d) {
    if (pj.shape[d] < 0) return set_error(TCX_INVALID_ARGUMENT, "negative permute extent");
    if (pj.perm[d] < 0 || static_cast<uint32_t>(pj.perm[d]) >= pj.ndim || seen[pj.perm[d]])
      return set_error(TCX_INVALID_ARGUMENT, "perm is not a permutation");
    seen[pj.perm[d]] = true;
  }
  if (pj.esize != 1 && pj.esize != 2 && pj.esize != 4 && pj.esize != 8)
    return set_error(TCX_INVALID_ARGUMENT, "permute element size must be 1, 2, 4 or 8");
  return TCX_OK;
}

tcx_status launch_permute(const void* d_src, void* d_dst, const tcx_permute_job& pj, cudaStream_t stream) {
  tcx_status st = check_permute(pj);
  if (st != TCX_OK) return st;
  const auto* s = static_cast<const uint8_t*>(d_src);
  auto* d = static_cast<uint8_t*>(d_dst);
  switch (pj.esize) {
    case 1: return launch_permute_t<uint8_t>(s, d, pj, stream);
    case 2: return launch_permute_t<uint16_t>(s, d, pj, stream);
    case 4: return launch_permute_t<uint32_t>(s, d, pj, stream);
    default: return launch_permute_t<uint64_t>(s, d, pj, stream);
  }
}

}  // namespace tcx

using namespace tcx;

extern "C" uint64_t tcx_copy_jobs_scratch_bytes(uint64_t n_jobs) { return ((n_jobs + 1) * 8 + 255) & ~255ull; }

extern "C" tcx_status tcx_copy_jobs(const void* d_src, void* d_dst, const tcx_copy_job* d_jobs, uint64_t n_jobs,
                                    void* d_scratch, uint64_t scratch_bytes, void* stream) {
  if (n_jobs == 0) return TCX_OK;
  if (d_src == nullptr || d_dst == nullptr || d_jobs == nullptr || d_scratch == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "null pointer");
  if (scratch_bytes < tcx_copy_jobs_scratch_bytes(n_jobs))
    return set_error(TCX_INVALID_ARGUMENT, "copy-job scratch too small");
  if ((reinterpret_cast<uintptr_t>(d_scratch) & 7u) != 0 || (reinterpret_cast<uintptr_t>(d_jobs) & 7u) != 0)
    return set_error(TCX_INVALID_ARGUMENT, "jobs and scratch must be 8-byte aligned");
  return launch_copy_jobs(d_src, d_dst, d_jobs, n_jobs, static_cast<uint64_t*>(d_scratch),
                          static_cast<cudaStream_t>(stream));
}

extern "C" tcx_status tcx_permute(const void* d_src, void* d_dst, const tcx_permute_job* job, void* stream) {
  if (d_src == nullptr || d_dst == nullptr || job == nullptr) return set_error(TCX_INVALID_ARGUMENT, "null pointer");
  return launch_permute(d_src, d_dst, *job, static_cast<cudaStream_t>(stream));
}
