// Content hashing on sm_100a: per-leaf SHA-256, the Merkle reduction and the
// data-multihash entry point of the C ABI.
//
// Reference behaviour followed (core/common/artifact_hash_gpu.cc, artifact_hash_cpu.cc):
//   * leaves [i*L, min((i+1)*L, T)), 32-byte big-endian digests (kernel :384-411);
//   * pairwise Merkle tree, odd node promoted unchanged (:198-233 of the CPU file);
//   * argument checks and messages of compute_data_multihash_from_gpu (:903-957);
//   * leaf policy determine_leaf_chunk_size (artifact_hash_cpu.cc:269-303).
//
// Kernel design. SHA-256 is serial inside a leaf, so the unit of parallelism is
// the leaf ("chain"). Two kernels:
//   * sha256_leaf_kernel: one thread owns one chain and keeps the state, the
//     16-word message window and the next block in registers. Best when there
//     are enough chains to fill every SM sub-partition (SMSP) several times.
//   * sha256_leaf_ws_kernel (warp-specialised): a consumer warp runs only the
//     64 compression rounds of 32 chains while a producer warp on another SMSP
//     loads the blocks, expands the message schedule and adds the round
//     constants, handing K[t]+W[t] over through a double-buffered shared-memory
//     ring guarded by named barriers. With few chains (large leaves) the chain's
//     own instruction stream is the limit, and this removes ~40% of it.
// Both take a pass window [seg_off, seg_off+seg_len) inside every leaf and a
// per-chain state array, so a leaf can be hashed in several passes as its bytes
// arrive (streamed loads); a single pass with seg_off = 0 covers the whole leaf.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "sha256_device.cuh"
#include "tcx_internal.h"

namespace tcx {
namespace {

constexpr int kLeafThreads = 64;       // threads (= leaves) per CTA of the leaf kernel
constexpr int kMerkleThreads = 256;    // threads per CTA of a Merkle level
constexpr uint32_t kFinishMax = 2048;  // levels at or below this size finish in one CTA
constexpr int kFinishThreads = 1024;

// ---------------------------------------------------------------------------
// Leaf geometry. Uniform: leaf i covers [i*leaf, min((i+1)*leaf, total)).
// Table: leaf i covers [off[i], off[i] + len[i]) (segmented inputs such as
// per-sequence buffers, or a chosen subset of leaves).
// ---------------------------------------------------------------------------
struct LeafGeom {
  uint64_t total;
  uint64_t leaf;
  const uint64_t* off;  // table mode when non-null
  const uint32_t* len;
  uint64_t pitch;       // > 0: the pass's bytes of leaf i are at src + i * pitch (a slab buffer)
};

// Per-chain quantities of one pass. A pass covers [seg_off, seg_off + seg_len) of
// every leaf (seg_off and, unless it reaches the leaf end, seg_len are multiples
// of 64). The chain is finalised in the pass that reaches its end.
struct LeafPass {
  uint64_t start;     // byte offset of the leaf in the source
  uint64_t leaf_len;  // bytes of this leaf
  uint64_t begin;     // first byte of the pass inside the leaf
  uint64_t data;      // offset of that byte in the source buffer
  uint64_t nfull;     // full 64-byte blocks of leaf data in this pass
  uint32_t nb;        // blocks compressed in this pass (data + padding)
  bool active;        // the pass touches this leaf
  bool finalize;      // the pass reaches the leaf end: pad and emit the digest
};

__device__ __forceinline__ LeafPass leaf_pass(uint32_t i, uint32_t n_leaves, const LeafGeom& g, uint64_t seg_off,
                                              uint64_t seg_len) {
  LeafPass p{};
  if (i >= n_leaves) return p;
  if (g.off != nullptr) {
    p.start = g.off[i];
    p.leaf_len = g.len[i];
  } else {
    p.start = static_cast<uint64_t>(i) * g.leaf;
    p.leaf_len = min(g.leaf, g.total - p.start);
  }
  if (p.leaf_len == 0) return p;
  if (seg_off >= p.leaf_len) return p;
  p.active = true;
  p.begin = seg_off;
  p.data = g.pitch ? static_cast<uint64_t>(i) * g.pitch : p.start + seg_off;
  const uint64_t room = p.leaf_len - seg_off;
  p.finalize = seg_len >= room;
  const uint64_t bytes = p.finalize ? room : seg_len;
  p.nfull = bytes >> 6;
  p.nb = static_cast<uint32_t>(p.nfull) + (p.finalize ? ((p.leaf_len & 63u) < 56u ? 1u : 2u) : 0u);
  return p;
}

__device__ __forceinline__ void load_or_init_state(uint32_t s[8], const LeafPass& p, const uint32_t* states,
                                                   uint32_t i) {
  if (p.begin == 0 || states == nullptr) {
    dev::init_state(s);
  } else {
    const uint4* st = reinterpret_cast<const uint4*>(states + 8ull * i);
    const uint4 x = st[0], y = st[1];
    s[0] = x.x; s[1] = x.y; s[2] = x.z; s[3] = x.w;
    s[4] = y.x; s[5] = y.y; s[6] = y.z; s[7] = y.w;
  }
}

__device__ __forceinline__ void save_state(const uint32_t s[8], uint32_t* states, uint32_t i) {
  uint4* st = reinterpret_cast<uint4*>(states + 8ull * i);
  st[0] = make_uint4(s[0], s[1], s[2], s[3]);
  st[1] = make_uint4(s[4], s[5], s[6], s[7]);
}

// ---------------------------------------------------------------------------
// Plain leaf kernel: one thread per chain.
// kVec: every leaf start is 16-byte aligned (16-aligned base, L % 16 == 0).
// Otherwise each leaf start has a fixed misalignment s = addr & 3 and a block is
// assembled from 17 aligned words with funnel shifts. Every word read lies in the
// same aligned 4-byte word as at least one byte of the leaf, so no read can leave
// the pages of the buffer.
// ---------------------------------------------------------------------------
template <bool kVec>
__global__ void __launch_bounds__(kLeafThreads) sha256_leaf_kernel(const uint8_t* __restrict__ src, LeafGeom geom,
                                                                   uint32_t n_leaves, uint64_t seg_off,
                                                                   uint64_t seg_len, uint32_t* __restrict__ states,
                                                                   uint8_t* __restrict__ digests) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  const LeafPass ps = leaf_pass(i, n_leaves, geom, seg_off, seg_len);
  if (!ps.active) return;
  const uint8_t* p = src + ps.data;
  const uint64_t nfull = ps.nfull;

  uint32_t s[8];
  load_or_init_state(s, ps, states, i);
  uint32_t w[16];

  if constexpr (kVec) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    uint4 v0, v1, v2, v3;
    if (nfull > 0) {
      v0 = dev::ldg_stream(q + 0);
      v1 = dev::ldg_stream(q + 1);
      v2 = dev::ldg_stream(q + 2);
      v3 = dev::ldg_stream(q + 3);
    }
    for (uint64_t b = 0; b < nfull; ++b) {
      dev::words_from_vec(w, v0, v1, v2, v3);
      if (b + 1 < nfull) {
        const uint4* nq = q + 4 * (b + 1);
        v0 = dev::ldg_stream(nq + 0);
        v1 = dev::ldg_stream(nq + 1);
        v2 = dev::ldg_stream(nq + 2);
        v3 = dev::ldg_stream(nq + 3);
      }
      dev::compress(s, w);
    }
  } else {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(p);
    const uint32_t shift = static_cast<uint32_t>(addr & 3u) * 8u;
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(addr & ~static_cast<uintptr_t>(3));
    for (uint64_t b = 0; b < nfull; ++b) {
      const uint32_t* bw = wp + 16 * b;
      uint32_t lo = __ldg(bw);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        // The 17th word is only needed (and only read) when the block is misaligned.
        const uint32_t hi = (shift != 0 || k < 15) ? __ldg(bw + k + 1) : 0u;
        w[k] = dev::bswap32(shift ? __funnelshift_r(lo, hi, shift) : lo);
        lo = hi;
      }
      dev::compress(s, w);
    }
  }
  if (ps.finalize) {
    dev::finish(s, p + (nfull << 6), static_cast<uint32_t>(ps.leaf_len & 63u), ps.leaf_len);
    dev::store_digest(digests + 32ull * i, s);
  } else {
    save_state(s, states, i);
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised leaf kernel (16-byte aligned leaves only).
// CTA = P consumer warps (warps 0..P-1) + P producer warps (warps P..2P-1);
// producer warp P+c feeds consumer warp c, lane j <-> chain j.
// Shared ring per pair: kWsStages stages x kWsBlocks blocks x 64 words x 32 lanes,
// laid out [stage][block][t/4][lane][t%4] so that each lane moves 16 bytes per
// access and a warp touches 512 contiguous bytes (no bank conflicts).
// ---------------------------------------------------------------------------
constexpr int kWsStages = 2;
constexpr int kWsBlockWords = 64 * 32;
// Layouts (pairs per CTA, blocks per stage), by chains n:
//  * <2, 4> while the grid is one wave (n <= 64 per SM): warps 0-3 of the CTA sit
//    on SMSPs 0-3, so each consumer has an SMSP to itself; 4 blocks per stage
//    (128 KiB of ring) measured 1.7% faster per block than 2 on the 3830-chain
//    Llama-3-8B load (fewer ring hand-offs);
//  * <4, 2> for n <= 96 per SM: one CTA per SM whose four consumers and four
//    producers share the four SMSPs one each, instead of a second <2, *> CTA
//    stacking two consumers on SMSPs 0 and 1. Measured on B200 (4 MiB leaves):
//    10240 chains 102.6 ms against 109.1 ms for <2, 2>; at 17920 chains it lost
//    (136.8 against 125.6 ms), so it stops at 96 chains per SM;
//  * <2, 2> beyond that (64 KiB, three CTAs per SM).
constexpr size_t ws_smem_bytes(int pairs, int blocks) {
  return static_cast<size_t>(pairs) * kWsStages * blocks * kWsBlockWords * 4;
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Message words of block b of a pass: data (b < nfull), the padded tail, or the
// length-only block; zero for blocks past the chain's end.
__device__ __forceinline__ void ws_tail_words(uint32_t w[16], const LeafPass& ps, const uint8_t* p, uint32_t b) {
  const uint32_t rem = static_cast<uint32_t>(ps.leaf_len & 63u);
  const uint64_t bits = ps.leaf_len * 8ull;
  const bool tail = ps.finalize && b == ps.nfull;
  const bool len_only = ps.finalize && rem >= 56 && b == ps.nfull + 1;
  const uint8_t* t = p + (ps.nfull << 6);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t pos = 4u * k + j;
      uint32_t byte = 0;
      if (tail) {
        if (pos < rem) {
          byte = t[pos];
        } else if (pos == rem) {
          byte = 0x80u;
        }
      }
      word |= byte << (24 - 8 * j);
    }
    w[k] = word;
  }
  if ((tail && rem < 56) || len_only) {
    w[14] = static_cast<uint32_t>(bits >> 32);
    w[15] = static_cast<uint32_t>(bits);
  }
}

__device__ __forceinline__ void ws_produce_block(uint4* dst, uint32_t w[16], uint32_t lane) {
  // K[t] + W[t] for the 64 rounds, four rounds per 16-byte store.
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    uint32_t kw[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = 4 * q + r;
      if (t >= 16) {
        w[t & 15] += dev::small_sigma1(w[(t - 2) & 15]) + w[(t - 7) & 15] + dev::small_sigma0(w[(t - 15) & 15]);
      }
      kw[r] = dev::kRoundK[t] + w[t & 15];
    }
    dst[q * 32 + lane] = make_uint4(kw[0], kw[1], kw[2], kw[3]);
  }
}

// 64 rounds of one block from K[t]+W[t] in shared memory (16 bytes per lane per
// four rounds). Measured on B200, plain adds here beat moving the off-recurrence
// adds to the FMA pipe, so the compiler's schedule is kept.
__device__ __forceinline__ void ws_consume_block(uint32_t s[8], const uint4* src, uint32_t lane, bool keep) {
  uint32_t a = s[0], b = s[1], c = s[2], d = s[3], e = s[4], f = s[5], g = s[6], h = s[7];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const uint4 kw4 = src[q * 32 + lane];
    const uint32_t kw[4] = {kw4.x, kw4.y, kw4.z, kw4.w};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t t1 = h + kw[r] + dev::big_sigma1(e) + dev::choose(e, f, g);
      const uint32_t t2 = dev::big_sigma0(a) + dev::majority(a, b, c);
      h = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
  }
  if (keep) {
    s[0] += a; s[1] += b; s[2] += c; s[3] += d;
    s[4] += e; s[5] += f; s[6] += g; s[7] += h;
  }
}

template <int kWsPairs, int kWsBlocks>
__global__ void __launch_bounds__(64 * kWsPairs, 1) sha256_leaf_ws_kernel(const uint8_t* __restrict__ src,
                                                                          LeafGeom geom, uint32_t n_leaves,
                                                                          uint64_t seg_off, uint64_t seg_len,
                                                                          uint32_t* __restrict__ states,
                                                                          uint8_t* __restrict__ digests) {
  static_assert(kWsPairs * 2 * kWsStages <= 16, "named barriers 0..15");
  constexpr int kWsStageWords = kWsBlocks * kWsBlockWords;
  extern __shared__ uint4 ws_smem[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const bool producer = warp >= kWsPairs;
  const uint32_t pair = producer ? warp - kWsPairs : warp;
  const uint32_t i = blockIdx.x * (32u * kWsPairs) + pair * 32u + lane;
  const LeafPass ps = leaf_pass(i, n_leaves, geom, seg_off, seg_len);
  const uint32_t max_nb = __reduce_max_sync(0xffffffffu, ps.active ? ps.nb : 0u);
  const uint32_t n_stages = (max_nb + kWsBlocks - 1) / kWsBlocks;
  uint4* ring = ws_smem + static_cast<size_t>(pair) * kWsStages * (kWsStageWords / 4);
  // Named barriers pair*4 + {0, 1} (stage full) and + {2, 3} (stage empty); the
  // kernel never uses barrier 0 otherwise (no __syncthreads).
  const uint32_t bar_full = pair * 2u * kWsStages;
  const uint32_t bar_empty = bar_full + kWsStages;

  if (producer) {
    const uint8_t* p = src + (ps.active ? ps.data : 0ull);
    const uint4* q = reinterpret_cast<const uint4*>(p);
    uint4 cur[4], nxt[4];
    if (ps.active && ps.nfull > 0) {
#pragma unroll
      for (int k = 0; k < 4; ++k) cur[k] = dev::ldg_stream(q + k);
    }
    if (ps.active && ps.nfull > 1) {
#pragma unroll
      for (int k = 0; k < 4; ++k) nxt[k] = dev::ldg_stream(q + 4 + k);
    }
    uint32_t b = 0;
    for (uint32_t st = 0; st < n_stages; ++st) {
      const uint32_t slot = st % kWsStages;
      named_bar_sync(bar_empty + slot, 64);
      uint4* stage = ring + static_cast<size_t>(slot) * (kWsStageWords / 4);
#pragma unroll 1
      for (int blk = 0; blk < kWsBlocks; ++blk, ++b) {
        if (b >= max_nb) break;
        uint32_t w[16];
        if (ps.active && b < ps.nfull) {
          dev::words_from_vec(w, cur[0], cur[1], cur[2], cur[3]);
#pragma unroll
          for (int k = 0; k < 4; ++k) cur[k] = nxt[k];
          if (b + 2 < ps.nfull) {
            const uint4* nq = q + 4ull * (b + 2);
#pragma unroll
            for (int k = 0; k < 4; ++k) nxt[k] = dev::ldg_stream(nq + k);
          }
        } else {
          ws_tail_words(w, ps, p, b);
        }
        ws_produce_block(stage + blk * (kWsBlockWords / 4), w, lane);
      }
      named_bar_arrive(bar_full + slot, 64);
    }
    // Match the consumer's trailing releases so every barrier generation completes.
    for (uint32_t st = n_stages; st < n_stages + kWsStages; ++st) named_bar_sync(bar_empty + st % kWsStages, 64);
  } else {
    uint32_t s[8];
    load_or_init_state(s, ps, states, i);
    for (int k = 0; k < kWsStages; ++k) named_bar_arrive(bar_empty + k, 64);
    uint32_t b = 0;
    for (uint32_t st = 0; st < n_stages; ++st) {
      const uint32_t slot = st % kWsStages;
      named_bar_sync(bar_full + slot, 64);
      const uint4* stage = ring + static_cast<size_t>(slot) * (kWsStageWords / 4);
#pragma unroll 1
      for (int blk = 0; blk < kWsBlocks; ++blk, ++b) {
        if (b >= max_nb) break;
        ws_consume_block(s, stage + blk * (kWsBlockWords / 4), lane, ps.active && b < ps.nb);
      }
      named_bar_arrive(bar_empty + slot, 64);
    }
    if (ps.active) {
      if (ps.finalize) {
        dev::store_digest(digests + 32ull * i, s);
      } else {
        save_state(s, states, i);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Register-only compression throughput probe: n chains x `blocks` compressions
// whose message words are derived from the running state (so nothing can be
// hoisted), no memory traffic except the final state. Measures the SHA-256
// compute bound (and, with one warp, the per-block chain latency) of this GPU.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kLeafThreads) sha256_probe_kernel(uint32_t n, uint32_t blocks, uint32_t* out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t s[8], w[16];
  dev::init_state(s);
  s[0] ^= i;
  for (uint32_t b = 0; b < blocks; ++b) {
#pragma unroll
    for (int k = 0; k < 16; ++k) w[k] = s[k & 7] + static_cast<uint32_t>(k) + b;
    dev::compress(s, w);
  }
  uint4* o = reinterpret_cast<uint4*>(out + 8ull * i);
  o[0] = make_uint4(s[0], s[1], s[2], s[3]);
  o[1] = make_uint4(s[4], s[5], s[6], s[7]);
}

// ---------------------------------------------------------------------------
// Merkle reduction. node = SHA-256(left || right): one data block plus the
// constant padding block of a 64-byte message.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void hash_pair(const uint8_t* pair64, uint8_t* out32) {
  const uint4* q = reinterpret_cast<const uint4*>(pair64);
  uint32_t s[8], w[16];
  dev::init_state(s);
  dev::words_from_vec(w, q[0], q[1], q[2], q[3]);
  dev::compress(s, w);
#pragma unroll
  for (int k = 0; k < 16; ++k) w[k] = 0;
  w[0] = 0x80000000u;
  w[15] = 512u;
  dev::compress(s, w);
  dev::store_digest(out32, s);
}

// One level: dst[j] = H(src[2j] || src[2j+1]); an odd last node is copied.
__global__ void __launch_bounds__(kMerkleThreads) merkle_level_kernel(const uint8_t* __restrict__ src, uint32_t m,
                                                                      uint8_t* __restrict__ dst) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t pairs = m / 2;
  if (j < pairs) {
    hash_pair(src + 64ull * j, dst + 32ull * j);
  } else if (j == pairs && (m & 1u)) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src + 32ull * (m - 1));
    uint4* d4 = reinterpret_cast<uint4*>(dst + 32ull * j);
    d4[0] = s4[0];
    d4[1] = s4[1];
  }
}

// Remaining levels (m <= kFinishMax) inside one CTA, in shared memory; writes the root.
__global__ void __launch_bounds__(kFinishThreads) merkle_finish_kernel(const uint8_t* __restrict__ src, uint32_t m,
                                                                       uint8_t* __restrict__ root) {
  extern __shared__ uint4 smem4[];
  uint8_t* nodes = reinterpret_cast<uint8_t*>(smem4);
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  for (uint32_t k = threadIdx.x; k < 2 * m; k += blockDim.x) smem4[k] = s4[k];
  __syncthreads();
  while (m > 1) {
    const uint32_t pairs = m / 2;
    const uint32_t j = threadIdx.x;  // pairs <= kFinishMax / 2 == blockDim.x
    uint32_t s[8];
    uint4 keep0 = make_uint4(0, 0, 0, 0), keep1 = keep0;
    if (j < pairs) {
      const uint4* q = reinterpret_cast<const uint4*>(nodes + 64u * j);
      uint32_t w[16];
      dev::init_state(s);
      dev::words_from_vec(w, q[0], q[1], q[2], q[3]);
      dev::compress(s, w);
#pragma unroll
      for (int k = 0; k < 16; ++k) w[k] = 0;
      w[0] = 0x80000000u;
      w[15] = 512u;
      dev::compress(s, w);
    } else if (j == pairs && (m & 1u)) {
      keep0 = smem4[2 * (m - 1)];
      keep1 = smem4[2 * (m - 1) + 1];
    }
    __syncthreads();  // every read of this level precedes every write
    if (j < pairs) {
      dev::store_digest(nodes + 32u * j, s);
    } else if (j == pairs && (m & 1u)) {
      smem4[2 * j] = keep0;
      smem4[2 * j + 1] = keep1;
    }
    __syncthreads();
    m = pairs + (m & 1u);
  }
  if (threadIdx.x < 2) reinterpret_cast<uint4*>(root)[threadIdx.x] = smem4[threadIdx.x];
}

// Per-segment roots: CTA s reduces the digests of segment s (at most
// kFinishMax leaves) in shared memory and writes its root to roots + 32*s.
__global__ void __launch_bounds__(kFinishThreads) merkle_segments_kernel(const uint8_t* __restrict__ digests,
                                                                         const uint64_t* __restrict__ seg_first,
                                                                         uint8_t* __restrict__ roots) {
  extern __shared__ uint4 seg4[];
  const uint64_t first = seg_first[blockIdx.x];
  uint32_t m = static_cast<uint32_t>(seg_first[blockIdx.x + 1] - first);
  if (m == 0 || m > kFinishMax) return;  // empty segments are rejected on the host; big ones reduced separately
  uint8_t* nodes = reinterpret_cast<uint8_t*>(seg4);
  const uint4* s4 = reinterpret_cast<const uint4*>(digests + 32ull * first);
  for (uint32_t k = threadIdx.x; k < 2 * m; k += blockDim.x) seg4[k] = s4[k];
  __syncthreads();
  while (m > 1) {
    const uint32_t pairs = m / 2;
    const uint32_t j = threadIdx.x;
    uint32_t st[8];
    uint4 keep0 = make_uint4(0, 0, 0, 0), keep1 = keep0;
    if (j < pairs) {
      const uint4* q = reinterpret_cast<const uint4*>(nodes + 64u * j);
      uint32_t w[16];
      dev::init_state(st);
      dev::words_from_vec(w, q[0], q[1], q[2], q[3]);
      dev::compress(st, w);
#pragma unroll
      for (int k = 0; k < 16; ++k) w[k] = 0;
      w[0] = 0x80000000u;
      w[15] = 512u;
      dev::compress(st, w);
    } else if (j == pairs && (m & 1u)) {
      keep0 = seg4[2 * (m - 1)];
      keep1 = seg4[2 * (m - 1) + 1];
    }
    __syncthreads();
    if (j < pairs) {
      dev::store_digest(nodes + 32u * j, st);
    } else if (j == pairs && (m & 1u)) {
      seg4[2 * j] = keep0;
      seg4[2 * j + 1] = keep1;
    }
    __syncthreads();
    m = pairs + (m & 1u);
  }
  if (threadIdx.x < 2) reinterpret_cast<uint4*>(roots + 32ull * blockIdx.x)[threadIdx.x] = seg4[threadIdx.x];
}

// ---------------------------------------------------------------------------
// Host helpers.
// ---------------------------------------------------------------------------
uint64_t div_up(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

uint64_t leaf_policy(uint64_t total, uint64_t requested) {
  uint64_t bounded = requested == 0 ? TCX_DEFAULT_LEAF_BYTES : requested;
  bounded = std::min<uint64_t>(bounded, TCX_MAX_LEAF_BYTES);
  bounded = std::max<uint64_t>(bounded, 64);
  bounded -= bounded % 64;
  if (bounded == 0) bounded = 64;
  if (requested != TCX_DEFAULT_LEAF_BYTES) return bounded;
  uint64_t adjusted = bounded;
  while (adjusted > TCX_MIN_ADAPTIVE_LEAF_BYTES && div_up(total, adjusted) < TCX_TARGET_LEAF_COUNT) {
    uint64_t candidate = adjusted / 2;
    candidate -= candidate % 64;
    if (candidate < TCX_MIN_ADAPTIVE_LEAF_BYTES) break;
    adjusted = candidate;
  }
  if (adjusted < TCX_MIN_ADAPTIVE_LEAF_BYTES) adjusted = TCX_MIN_ADAPTIVE_LEAF_BYTES;
  return adjusted == 0 ? 64 : adjusted;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Chains up to which the warp-specialised kernel is chosen. Measured on B200: the
// warp-specialised kernel is ahead up to ~65k chains (per-chain latency matters
// while chains are scarce), the one-thread-per-chain kernel above ~100k chains
// (ALU throughput matters once every SMSP holds two or more chain warps).
static constexpr uint32_t kWsMaxChains = 98304u;

static int hash_kernel_choice() {
  // TCX_HASH_KERNEL=plain|ws|auto (default auto) selects the leaf kernel.
  const char* v = std::getenv("TCX_HASH_KERNEL");
  if (v == nullptr) return 0;
  if (std::strcmp(v, "plain") == 0) return 1;
  if (std::strcmp(v, "ws") == 0) return 2;
  return 0;
}

static tcx_status launch_leaf_kernels(const uint8_t* src, const LeafGeom& geom, uint32_t n, bool vec,
                                      uint64_t seg_off, uint64_t seg_len, uint32_t* states, uint8_t* out,
                                      cudaStream_t stream) {
  const int choice = hash_kernel_choice();
  const bool ws = vec && (choice == 2 || (choice == 0 && n <= kWsMaxChains));
  if (ws) {
    static thread_local int configured_device = -1;
    int dev = 0;
    TCX_CUDA_TRY(cudaGetDevice(&dev));
    if (configured_device != dev) {
      TCX_CUDA_TRY(cudaFuncSetAttribute(sha256_leaf_ws_kernel<2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(ws_smem_bytes(2, 2))));
      TCX_CUDA_TRY(cudaFuncSetAttribute(sha256_leaf_ws_kernel<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(ws_smem_bytes(2, 4))));
      TCX_CUDA_TRY(cudaFuncSetAttribute(sha256_leaf_ws_kernel<4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(ws_smem_bytes(4, 2))));
      configured_device = dev;
    }
    const uint64_t sms = static_cast<uint64_t>(sm_count());
    int layout = n <= sms * 64 ? 0 : (n <= sms * 96 ? 1 : 2);
    // TCX_WS_LAYOUT=0|1|2 forces a layout (measurement knob).
    if (const char* v = std::getenv("TCX_WS_LAYOUT")) layout = std::atoi(v) % 3;
    if (layout == 0) {
      const dim3 grid(static_cast<unsigned>(div_up(n, 64u)));
      sha256_leaf_ws_kernel<2, 4><<<grid, 128, ws_smem_bytes(2, 4), stream>>>(src, geom, n, seg_off, seg_len, states,
                                                                              out);
    } else if (layout == 1) {
      const dim3 grid(static_cast<unsigned>(div_up(n, 128u)));
      sha256_leaf_ws_kernel<4, 2><<<grid, 256, ws_smem_bytes(4, 2), stream>>>(src, geom, n, seg_off, seg_len, states,
                                                                              out);
    } else {
      const dim3 grid(static_cast<unsigned>(div_up(n, 64u)));
      sha256_leaf_ws_kernel<2, 2><<<grid, 128, ws_smem_bytes(2, 2), stream>>>(src, geom, n, seg_off, seg_len, states,
                                                                              out);
    }
    note_launches(1);
  } else if (vec) {
    const dim3 grid(static_cast<unsigned>(div_up(n, kLeafThreads)));
    sha256_leaf_kernel<true><<<grid, kLeafThreads, 0, stream>>>(src, geom, n, seg_off, seg_len, states, out);
    note_launches(1);
  } else {
    const dim3 grid(static_cast<unsigned>(div_up(n, kLeafThreads)));
    sha256_leaf_kernel<false><<<grid, kLeafThreads, 0, stream>>>(src, geom, n, seg_off, seg_len, states, out);
    note_launches(1);
  }
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

tcx_status launch_leaf_pass(const void* d_src, uint64_t total, uint64_t leaf, uint32_t n, uint64_t seg_off,
                            uint64_t seg_len, uint32_t* states, void* d_digests, cudaStream_t stream) {
  const LeafGeom geom{total, leaf, nullptr, nullptr, 0};
  const bool vec = aligned16(d_src) && leaf % 16 == 0;
  return launch_leaf_kernels(static_cast<const uint8_t*>(d_src), geom, n, vec, seg_off, seg_len, states,
                             static_cast<uint8_t*>(d_digests), stream);
}

tcx_status launch_leaf_pass_pitched(const void* d_src, uint64_t pitch, uint64_t total, uint64_t leaf, uint32_t n,
                                    uint64_t seg_off, uint64_t seg_len, uint32_t* states, void* d_digests,
                                    cudaStream_t stream) {
  if (pitch == 0 || pitch < std::min(seg_len, leaf))
    return set_error(TCX_INVALID_ARGUMENT, "slab pitch is smaller than the pass");
  const LeafGeom geom{total, leaf, nullptr, nullptr, pitch};
  const bool vec = aligned16(d_src) && pitch % 16 == 0;
  return launch_leaf_kernels(static_cast<const uint8_t*>(d_src), geom, n, vec, seg_off, seg_len, states,
                             static_cast<uint8_t*>(d_digests), stream);
}

tcx_status launch_leaf_table(const void* d_src, const uint64_t* d_off, const uint32_t* d_len, uint32_t n,
                             bool offsets_aligned16, void* d_digests, cudaStream_t stream) {
  const LeafGeom geom{0, 0, d_off, d_len, 0};
  const bool vec = aligned16(d_src) && offsets_aligned16;
  return launch_leaf_kernels(static_cast<const uint8_t*>(d_src), geom, n, vec, 0, ~0ull, nullptr,
                             static_cast<uint8_t*>(d_digests), stream);
}

tcx_status launch_leaves(const void* d_src, uint64_t total, uint64_t leaf, uint32_t n, void* d_digests,
                         cudaStream_t stream) {
  return launch_leaf_pass(d_src, total, leaf, n, 0, ~0ull, nullptr, d_digests, stream);
}

uint64_t merkle_scratch_bytes(uint64_t n) {
  // Two ping-pong level buffers; the largest levels are ceil(n/2) and ceil(n/4) nodes.
  const uint64_t a = div_up(n, 2), b = div_up(n, 4);
  return ((a + b + 2) * 32 + 255) & ~255ull;
}

tcx_status launch_merkle(const uint8_t* digests, uint64_t n, uint8_t* scratch, uint8_t* root, cudaStream_t stream) {
  const uint64_t a_nodes = div_up(n, 2);
  uint8_t* buf[2] = {scratch, scratch + ((a_nodes * 32 + 255) & ~255ull)};
  const uint8_t* cur = digests;
  uint64_t m = n;
  int which = 0;
  while (m > kFinishMax) {
    const uint64_t next = div_up(m, 2);
    const unsigned grid = static_cast<unsigned>(div_up(next, kMerkleThreads));
    merkle_level_kernel<<<grid, kMerkleThreads, 0, stream>>>(cur, static_cast<uint32_t>(m), buf[which]);
    note_launches(1);
    TCX_CUDA_TRY(cudaGetLastError());
    cur = buf[which];
    which ^= 1;
    m = next;
  }
  const size_t smem = static_cast<size_t>(m) * 32;
  if (smem > 48 * 1024) {
    // The attribute is per device; setting it is a cheap host-side call.
    TCX_CUDA_TRY(cudaFuncSetAttribute(merkle_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kFinishMax * 32)));
  }
  merkle_finish_kernel<<<1, kFinishThreads, smem, stream>>>(cur, static_cast<uint32_t>(m), root);
  note_launches(1);
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

void encode_multihash(const uint8_t digest[32], char out[57]) {
  static const char kAlphabet[] = "abcdefghijklmnopqrstuvwxyz234567";
  uint8_t mh[34];
  mh[0] = 0x12;
  mh[1] = 0x20;
  std::memcpy(mh + 2, digest, 32);
  char tmp[64];
  size_t pos = 0;
  for (size_t i = 0; i < sizeof mh;) {
    const size_t take = std::min<size_t>(5, sizeof mh - i);
    uint64_t acc = 0;
    for (size_t j = 0; j < take; ++j) acc = (acc << 8) | mh[i + j];
    acc <<= (5 - take) * 8;
    for (int sh = 35; sh >= 0; sh -= 5) tmp[pos++] = kAlphabet[(acc >> sh) & 31u];
    i += take;
  }
  out[0] = 'b';
  std::memcpy(out + 1, tmp, 55);  // ceil(34 * 8 / 5) = 55 significant characters
  out[56] = '\0';
}

// Loads every hashing kernel on the current device (a lazily loaded module
// allocates device memory at its first launch otherwise).
tcx_status preload_hash_kernels() {
  cudaFuncAttributes attr;
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_kernel<true>));
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_kernel<false>));
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_ws_kernel<2, 2>));
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_ws_kernel<2, 4>));
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, sha256_leaf_ws_kernel<4, 2>));
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, merkle_level_kernel));
  TCX_CUDA_TRY(cudaFuncGetAttributes(&attr, merkle_finish_kernel));
  TCX_CUDA_TRY(cudaFuncSetAttribute(merkle_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kFinishMax * 32)));
  return TCX_OK;
}

namespace {

// Per-device resources of tcx_multihash_from_gpu, created once and grown on demand.
struct DeviceHashContext {
  std::mutex mu;
  bool ready = false;
  cudaStream_t stream = nullptr;
  uint8_t* digests = nullptr;
  uint64_t digests_cap = 0;
  uint8_t* scratch = nullptr;
  uint64_t scratch_cap = 0;
  uint8_t* d_root = nullptr;
  uint8_t* h_root = nullptr;  // pinned
  cudaEvent_t queued = nullptr;  // marks prior work on the legacy default stream
};

constexpr int kMaxDevices = 64;
DeviceHashContext g_ctx[kMaxDevices];

// Caller holds ctx.mu and has made the device current.
tcx_status ensure_context(DeviceHashContext& ctx, uint64_t n_leaves) {
  if (!ctx.ready) {
    TCX_CUDA_TRY(cudaStreamCreateWithFlags(&ctx.stream, cudaStreamNonBlocking));
    TCX_CUDA_TRY(cudaEventCreateWithFlags(&ctx.queued, cudaEventDisableTiming));
    TCX_CUDA_TRY(cudaMalloc(&ctx.d_root, 256));
    TCX_CUDA_TRY(cudaMallocHost(&ctx.h_root, 256));
    tcx_status st = preload_hash_kernels();
    if (st != TCX_OK) return st;
    ctx.ready = true;
  }
  const uint64_t need_d = std::max<uint64_t>(n_leaves, 1) * 32;
  if (need_d > ctx.digests_cap) {
    if (ctx.digests) TCX_CUDA_TRY(cudaFree(ctx.digests));
    ctx.digests = nullptr;
    ctx.digests_cap = 0;
    const uint64_t cap = std::max<uint64_t>(need_d, 4096 * 32);
    TCX_CUDA_TRY(cudaMalloc(&ctx.digests, cap));
    ctx.digests_cap = cap;
  }
  const uint64_t need_s = merkle_scratch_bytes(n_leaves);
  if (need_s > ctx.scratch_cap) {
    if (ctx.scratch) TCX_CUDA_TRY(cudaFree(ctx.scratch));
    ctx.scratch = nullptr;
    ctx.scratch_cap = 0;
    const uint64_t cap = std::max<uint64_t>(need_s, merkle_scratch_bytes(4096));
    TCX_CUDA_TRY(cudaMalloc(&ctx.scratch, cap));
    ctx.scratch_cap = cap;
  }
  return TCX_OK;
}

tcx_status fallback_disabled(tcx_status st) {
  if (st == TCX_OK) return st;
  const std::string msg = tcx_last_error();
  return set_error(st, "GPU hashing unavailable; CPU fallback disabled: " + msg);
}

}  // namespace
}  // namespace tcx

using namespace tcx;

extern "C" tcx_status tcx_leaf_policy(uint64_t total_bytes, uint64_t requested_leaf_bytes, uint64_t* leaf_bytes_out) {
  if (leaf_bytes_out == nullptr) return set_error(TCX_INVALID_ARGUMENT, "leaf_bytes_out is null");
  *leaf_bytes_out = leaf_policy(total_bytes, requested_leaf_bytes);
  return TCX_OK;
}

namespace tcx {
namespace {
tcx_status check_leaf_args(const void* d_src, uint64_t total_bytes, uint64_t leaf_bytes, void* d_digests,
                           uint64_t digest_capacity) {
  if (d_src == nullptr) return set_error(TCX_INVALID_ARGUMENT, "GPU pointer is null");
  if (total_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "Cannot hash empty GPU buffer");
  if (total_bytes > TCX_MAX_HASH_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "GPU buffer too large for hashing: %llu bytes",
                      static_cast<unsigned long long>(total_bytes));
  if (leaf_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "leaf_chunk_bytes must be > 0");
  if (leaf_bytes > TCX_MAX_LEAF_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "Chunk size too large: %llu (max: %llu)",
                      static_cast<unsigned long long>(leaf_bytes), static_cast<unsigned long long>(TCX_MAX_LEAF_BYTES));
  const uint64_t n = div_up(total_bytes, leaf_bytes);
  if (n > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");
  if (d_digests == nullptr) return set_error(TCX_INVALID_ARGUMENT, "digest buffer is null");
  if (!aligned16(d_digests)) return set_error(TCX_INVALID_ARGUMENT, "digest buffer must be 16-byte aligned");
  if (digest_capacity < n)
    return set_errorf(TCX_INVALID_ARGUMENT, "digest buffer holds %llu digests, %llu needed",
                      static_cast<unsigned long long>(digest_capacity), static_cast<unsigned long long>(n));
  return TCX_OK;
}
}  // namespace
}  // namespace tcx

extern "C" tcx_status tcx_sha256_leaves(const void* d_src, uint64_t total_bytes, uint64_t leaf_bytes,
                                        void* d_digests, uint64_t digest_capacity, void* stream) {
  tcx_status st = check_leaf_args(d_src, total_bytes, leaf_bytes, d_digests, digest_capacity);
  if (st != TCX_OK) return st;
  const uint64_t n = div_up(total_bytes, leaf_bytes);
  return launch_leaves(d_src, total_bytes, leaf_bytes, static_cast<uint32_t>(n), d_digests,
                       static_cast<cudaStream_t>(stream));
}

extern "C" tcx_status tcx_sha256_leaves_pass(const void* d_src, uint64_t total_bytes, uint64_t leaf_bytes,
                                             uint64_t seg_off, uint64_t seg_len, void* d_states, void* d_digests,
                                             uint64_t digest_capacity, void* stream) {
  if (seg_off % 64 != 0 || seg_len % 64 != 0 || seg_len == 0)
    return set_error(TCX_INVALID_ARGUMENT, "seg_off and seg_len must be non-zero multiples of 64");
  if (d_states == nullptr || !aligned16(d_states))
    return set_error(TCX_INVALID_ARGUMENT, "state buffer must be non-null and 16-byte aligned");
  // Same argument checks as the single-pass entry point.
  tcx_status st = check_leaf_args(d_src, total_bytes, leaf_bytes, d_digests, digest_capacity);
  if (st != TCX_OK) return st;
  const uint64_t n = div_up(total_bytes, leaf_bytes);
  return launch_leaf_pass(d_src, total_bytes, leaf_bytes, static_cast<uint32_t>(n), seg_off, seg_len,
                          static_cast<uint32_t*>(d_states), d_digests, static_cast<cudaStream_t>(stream));
}

extern "C" tcx_status tcx_sha256_compute_probe(uint32_t n_chains, uint32_t blocks, void* d_out, void* stream) {
  if (n_chains == 0 || d_out == nullptr || !aligned16(d_out))
    return set_error(TCX_INVALID_ARGUMENT, "n_chains > 0 and a 16-byte aligned output are required");
  const dim3 grid(static_cast<unsigned>(div_up(n_chains, kLeafThreads)));
  sha256_probe_kernel<<<grid, kLeafThreads, 0, static_cast<cudaStream_t>(stream)>>>(n_chains, blocks,
                                                                                   static_cast<uint32_t*>(d_out));
  note_launches(1);
  TCX_CUDA_TRY(cudaGetLastError());
  return TCX_OK;
}

extern "C" uint64_t tcx_merkle_scratch_bytes(uint64_t n_leaves) { return merkle_scratch_bytes(n_leaves); }

extern "C" tcx_status tcx_merkle_root(const void* d_digests, uint64_t n_leaves, void* d_scratch, uint64_t scratch_bytes,
                                      void* d_root, void* stream) {
  if (d_digests == nullptr || d_root == nullptr) return set_error(TCX_INVALID_ARGUMENT, "null device pointer");
  if (n_leaves == 0) return set_error(TCX_INVALID_ARGUMENT, "Leaf digests must not be empty");
  if (n_leaves > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");
  if (!aligned16(d_digests) || !aligned16(d_root)) return set_error(TCX_INVALID_ARGUMENT, "digests and root must be 16-byte aligned");
  if (n_leaves > kFinishMax) {
    if (d_scratch == nullptr || !aligned16(d_scratch) || scratch_bytes < merkle_scratch_bytes(n_leaves))
      return set_errorf(TCX_INVALID_ARGUMENT, "Merkle scratch must be 16-byte aligned and hold %llu bytes",
                        static_cast<unsigned long long>(merkle_scratch_bytes(n_leaves)));
  }
  return launch_merkle(static_cast<const uint8_t*>(d_digests), n_leaves, static_cast<uint8_t*>(d_scratch),
                       static_cast<uint8_t*>(d_root), static_cast<cudaStream_t>(stream));
}

extern "C" tcx_status tcx_multihash_encode(const uint8_t* digest32, char* out, size_t out_capacity) {
  if (digest32 == nullptr || out == nullptr) return set_error(TCX_INVALID_ARGUMENT, "null pointer");
  if (out_capacity < TCX_MULTIHASH_CHARS + 1) return set_error(TCX_INVALID_ARGUMENT, "output buffer needs 57 bytes");
  encode_multihash(digest32, out);
  return TCX_OK;
}

extern "C" tcx_status tcx_multihash_from_gpu(const void* d_src, uint64_t total_bytes, int device_id,
                                             uint64_t leaf_chunk_bytes, char* out, size_t out_capacity) {
  // Argument checks in the order of artifact_hash_gpu.cc:907-927.
  if (d_src == nullptr) return set_error(TCX_INVALID_ARGUMENT, "GPU pointer is null");
  if (total_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "Cannot hash empty GPU buffer");
  if (total_bytes > TCX_MAX_HASH_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "GPU buffer too large for hashing: %llu bytes",
                      static_cast<unsigned long long>(total_bytes));
  if (leaf_chunk_bytes == 0) return set_error(TCX_INVALID_ARGUMENT, "leaf_chunk_bytes must be > 0");
  if (leaf_chunk_bytes > TCX_MAX_LEAF_BYTES)
    return set_errorf(TCX_INVALID_ARGUMENT, "Chunk size too large: %llu (max: %llu)",
                      static_cast<unsigned long long>(leaf_chunk_bytes),
                      static_cast<unsigned long long>(TCX_MAX_LEAF_BYTES));
  if (out == nullptr || out_capacity < TCX_MULTIHASH_CHARS + 1)
    return set_error(TCX_INVALID_ARGUMENT, "output buffer needs 57 bytes");
  if (device_id < 0 || device_id >= kMaxDevices)
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: invalid device ordinal", device_id);
  if (cudaError_t e = cudaSetDevice(device_id); e != cudaSuccess)
    return set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: %s", device_id, cuda_msg(e).c_str());

  const uint64_t leaf = leaf_policy(total_bytes, leaf_chunk_bytes);
  const uint64_t n = div_up(total_bytes, leaf);
  if (n > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");

  DeviceHashContext& ctx = g_ctx[device_id];
  std::lock_guard<std::mutex> lock(ctx.mu);
  tcx_status st = ensure_context(ctx, n);
  if (st == TCX_OK) {
    // The hash runs on the library's own stream; it first waits for the work already
    // queued on the legacy default stream (which orders every blocking stream), so a
    // buffer just written there is complete before it is hashed.
    cudaError_t e = cudaEventRecord(ctx.queued, cudaStreamLegacy);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx.stream, ctx.queued, 0);
    if (e != cudaSuccess) st = set_error(TCX_INTERNAL, "stream ordering failed: " + cuda_msg(e));
  }
  if (st == TCX_OK) st = launch_leaves(d_src, total_bytes, leaf, static_cast<uint32_t>(n), ctx.digests, ctx.stream);
  if (st == TCX_OK) st = launch_merkle(ctx.digests, n, ctx.scratch, ctx.d_root, ctx.stream);
  if (st == TCX_OK) {
    cudaError_t e = cudaMemcpyAsync(ctx.h_root, ctx.d_root, 32, cudaMemcpyDeviceToHost, ctx.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx.stream);
    if (e != cudaSuccess) st = set_error(TCX_INTERNAL, "digest readback failed: " + cuda_msg(e));
  }
  if (st != TCX_OK) return fallback_disabled(st);
  encode_multihash(ctx.h_root, out);
  return TCX_OK;
}

extern "C" tcx_status tcx_prewarm_device(int device_id) {
  if (device_id < 0) return set_error(TCX_INVALID_ARGUMENT, "device_id must be >= 0");
  int count = 0;
  TCX_CUDA_TRY(cudaGetDeviceCount(&count));
  if (device_id >= count || device_id >= kMaxDevices)
    return set_errorf(TCX_INVALID_ARGUMENT, "device_id %d out of range for visible GPU count %d", device_id, count);
  int prior = -1;
  const bool have_prior = cudaGetDevice(&prior) == cudaSuccess;
  tcx_status st = TCX_OK;
  if (cudaError_t e = cudaSetDevice(device_id); e != cudaSuccess) {
    st = set_errorf(TCX_INTERNAL, "Failed to set CUDA device %d: %s", device_id, cuda_msg(e).c_str());
  } else {
    DeviceHashContext& ctx = g_ctx[device_id];
    std::lock_guard<std::mutex> lock(ctx.mu);
    st = ensure_context(ctx, TCX_TARGET_LEAF_COUNT);
  }
  if (have_prior && prior != device_id) cudaSetDevice(prior);
  return st;
}

extern "C" tcx_status tcx_prewarm_visible_devices(void) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return TCX_OK;
  if (e != cudaSuccess) return set_error(TCX_INTERNAL, "cudaGetDeviceCount failed: " + cuda_msg(e));
  for (int d = 0; d < count; ++d) {
    tcx_status st = tcx_prewarm_device(d);
    if (st != TCX_OK) {
      const std::string msg = tcx_last_error();
      return set_errorf(st, "GPU hash prewarm failed for device %d: %s", d, msg.c_str());
    }
  }
  return TCX_OK;
}

extern "C" tcx_status tcx_sha256_leaf_table(const void* d_src, const uint64_t* d_leaf_offsets,
                                            const uint32_t* d_leaf_lengths, uint64_t n_leaves, int offsets_aligned16,
                                            void* d_digests, void* stream) {
  if (n_leaves == 0) return set_error(TCX_INVALID_ARGUMENT, "Leaf digests must not be empty");
  if (n_leaves > 0xffffffffull) return set_error(TCX_INVALID_ARGUMENT, "Leaf count exceeds supported range");
  if (d_src == nullptr || d_leaf_offsets == nullptr || d_leaf_lengths == nullptr || d_digests == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "null device pointer");
  if (!aligned16(d_digests)) return set_error(TCX_INVALID_ARGUMENT, "digest buffer must be 16-byte aligned");
  return launch_leaf_table(d_src, d_leaf_offsets, d_leaf_lengths, static_cast<uint32_t>(n_leaves),
                           offsets_aligned16 != 0, d_digests, static_cast<cudaStream_t>(stream));
}

extern "C" uint64_t tcx_merkle_segments_scratch_bytes(const uint64_t* seg_first, uint64_t n_segments) {
  uint64_t need = 256;
  for (uint64_t s = 0; s < n_segments; ++s) {
    const uint64_t m = seg_first[s + 1] - seg_first[s];
    if (m > kFinishMax) need = std::max(need, merkle_scratch_bytes(m));
  }
  return need;
}

extern "C" tcx_status tcx_merkle_roots_segmented(const void* d_digests, const uint64_t* seg_first,
                                                 const uint64_t* d_seg_first, uint64_t n_segments, void* d_scratch,
                                                 uint64_t scratch_bytes, void* d_roots, void* stream) {
  if (n_segments == 0) return TCX_OK;
  if (d_digests == nullptr || seg_first == nullptr || d_seg_first == nullptr || d_roots == nullptr)
    return set_error(TCX_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(d_digests) || !aligned16(d_roots))
    return set_error(TCX_INVALID_ARGUMENT, "digests and roots must be 16-byte aligned");
  if (n_segments > 0x7fffffffull) return set_error(TCX_INVALID_ARGUMENT, "too many segments");
  for (uint64_t s = 0; s < n_segments; ++s) {
    if (seg_first[s + 1] <= seg_first[s]) return set_errorf(TCX_INVALID_ARGUMENT, "segment %llu has no leaves",
                                                             static_cast<unsigned long long>(s));
  }
  if (scratch_bytes < tcx_merkle_segments_scratch_bytes(seg_first, n_segments) ||
      (d_scratch != nullptr && !aligned16(d_scratch)))
    return set_error(TCX_INVALID_ARGUMENT, "segment Merkle scratch too small or misaligned");
  const auto st = static_cast<cudaStream_t>(stream);
  TCX_CUDA_TRY(cudaFuncSetAttribute(merkle_segments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kFinishMax * 32)));
  merkle_segments_kernel<<<static_cast<unsigned>(n_segments), kFinishThreads, kFinishMax * 32, st>>>(
      static_cast<const uint8_t*>(d_digests), d_seg_first, static_cast<uint8_t*>(d_roots));
  note_launches(1);
  TCX_CUDA_TRY(cudaGetLastError());
  for (uint64_t s = 0; s < n_segments; ++s) {
    const uint64_t m = seg_first[s + 1] - seg_first[s];
    if (m <= kFinishMax) continue;
    tcx_status rc = launch_merkle(static_cast<const uint8_t*>(d_digests) + 32 * seg_first[s], m,
                                  static_cast<uint8_t*>(d_scratch), static_cast<uint8_t*>(d_roots) + 32 * s, st);
    if (rc != TCX_OK) return rc;
  }
  return TCX_OK;
}
