"""Paged KV-cache gather + per-sequence content hash (the paged-KV benchmark).

No reference implementation exists for this step (the reference keeps engine-owned
KV as opaque byte artifacts); it combines the same leaf hash / Merkle tree /
multihash as the artifact path (2 MiB leaves) with an on-device gather:

* pool: ``planes`` planes (layers x {K, V}), each ``pool_pages`` pages of
  ``page_tokens`` tokens x ``token_bytes`` (8 kv heads x 128 x bf16 = 2048 B);
* a sequence's pages are listed in its page table (slots of the pool);
* ``gather_and_hash`` writes every sequence contiguously as [plane][token][...]
  (tcx_kv_gather), hashes each sequence's bytes in its own 2 MiB leaves
  (tcx_sha256_leaf_table) and reduces one Merkle root per sequence
  (tcx_merkle_roots_segmented).

``workload`` builds the seeded benchmark workload: sequence lengths drawn from
``default_rng(seed).integers(64, 4097)`` in order while their pages fit in the
pool, page slots from ``default_rng(seed).permutation(pool_pages)``, sequences
dealt round-robin to ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _native
from .hashing import multibase_multihash_sha256

PAGE_TOKENS = 16
TOKEN_BYTES = 8 * 128 * 2  # 8 kv heads x head_dim 128 x bf16
KV_LEAF = 2 << 20


@dataclass
class KvWorkload:
    planes: int
    pool_pages: int
    page_tokens: int
    token_bytes: int
    seq_tokens: np.ndarray  # uint32 [n_seq]
    page_offsets: np.ndarray  # uint64 [n_seq + 1]
    page_table: np.ndarray  # uint32 [total_pages]

    @property
    def n_seq(self) -> int:
        return int(self.seq_tokens.size)

    def seq_bytes(self) -> np.ndarray:
        return self.seq_tokens.astype(np.uint64) * np.uint64(self.planes * self.token_bytes)

    def shard(self, world: int, rank: int, local_pool: bool = False) -> "KvWorkload":
        """Sequences rank, rank + world, ... With local_pool the rank's pool holds only its own
        pages, each at the rank of its global slot among the rank's slots (the random order of
        the global placement is kept, the pool shrinks to the rank's pages)."""
        idx = np.arange(rank, self.n_seq, world)
        pages = [self.page_table[self.page_offsets[i]:self.page_offsets[i + 1]] for i in idx]
        offs = np.zeros(idx.size + 1, np.uint64)
        offs[1:] = np.cumsum([p.size for p in pages]) if pages else []
        table = np.concatenate(pages).astype(np.uint32) if pages else np.zeros(0, np.uint32)
        pool_pages = self.pool_pages
        if local_pool and table.size:
            order = np.argsort(table, kind="stable")
            local = np.empty_like(table)
            local[order] = np.arange(table.size, dtype=np.uint32)
            table, pool_pages = local, int(table.size)
        return KvWorkload(self.planes, pool_pages, self.page_tokens, self.token_bytes,
                          self.seq_tokens[idx].copy(), offs, table)


def workload(seed: int = 3, planes: int = 64, pool_pages: int = 65536, max_seqs: int = 4096,
             min_tokens: int = 64, max_tokens: int = 4096, page_tokens: int = PAGE_TOKENS,
             token_bytes: int = TOKEN_BYTES) -> KvWorkload:
    rng = np.random.default_rng(seed)
    lens = rng.integers(min_tokens, max_tokens + 1, size=max_seqs)
    used, keep = 0, []
    for n in lens:
        p = -(-int(n) // page_tokens)
        if used + p > pool_pages:
            break
        keep.append(int(n))
        used += p
    slots = np.random.default_rng(seed).permutation(pool_pages).astype(np.uint32)
    seq_tokens = np.array(keep, np.uint32)
    pages = -(-seq_tokens.astype(np.int64) // page_tokens)
    offs = np.zeros(len(keep) + 1, np.uint64)
    offs[1:] = np.cumsum(pages)
    return KvWorkload(planes, pool_pages, page_tokens, token_bytes, seq_tokens, offs, slots[: int(offs[-1])].copy())


def make_pool(w: KvWorkload, seed: int = 3, device="cuda") -> torch.Tensor:
    """Seeded pool bytes (bf16 ~N(0,1) per plane) as a flat uint8 device tensor."""
    per_plane = w.pool_pages * w.page_tokens * w.token_bytes
    pool = torch.empty(w.planes * per_plane, dtype=torch.uint8, device=device)
    g = torch.Generator(device=device)
    for k in range(w.planes):
        g.manual_seed((seed << 32) | k)
        v = torch.randn(per_plane // 2, generator=g, dtype=torch.float32, device=device).to(torch.bfloat16)
        pool[k * per_plane:(k + 1) * per_plane].copy_(v.view(torch.uint8))
    return pool


@dataclass
class KvPlan:
    out_offsets: np.ndarray  # uint64 [n_seq]
    out_bytes: int
    leaf_offsets: np.ndarray  # uint64 [n_leaves]
    leaf_lengths: np.ndarray  # uint32 [n_leaves]
    seg_first: np.ndarray  # uint64 [n_seq + 1]


def plan(w: KvWorkload, leaf: int = KV_LEAF, align: int = 256) -> KvPlan:
    sb = w.seq_bytes()
    out_offsets = np.zeros(w.n_seq, np.uint64)
    cur = 0
    for i, b in enumerate(sb):
        out_offsets[i] = cur
        cur += -(-int(b) // align) * align
    lo, ll, first = [], [], [0]
    for i, b in enumerate(sb):
        n = -(-int(b) // leaf)
        starts = int(out_offsets[i]) + leaf * np.arange(n, dtype=np.uint64)
        lens = np.minimum(np.uint64(leaf), np.uint64(b) - leaf * np.arange(n, dtype=np.uint64))
        lo.append(starts)
        ll.append(lens.astype(np.uint32))
        first.append(first[-1] + n)
    return KvPlan(out_offsets, max(cur, 1), np.concatenate(lo).astype(np.uint64) if lo else np.zeros(0, np.uint64),
                  np.concatenate(ll) if ll else np.zeros(0, np.uint32), np.array(first, np.uint64))


class KvGatherHash:
    """Device-resident tables for one workload shard; ``run`` gathers and hashes."""

    def __init__(self, w: KvWorkload, leaf: int = KV_LEAF, device="cuda", out: torch.Tensor | None = None):
        self.w, self.leaf = w, leaf
        self.p = plan(w, leaf)
        d = torch.device(device)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(d)  # noqa: E731
        self.page_table = t(w.page_table.view(np.int32))
        self.page_offsets = t(w.page_offsets.view(np.int64))
        self.seq_tokens = t(w.seq_tokens.view(np.int32))
        self.out_offsets = t(self.p.out_offsets.view(np.int64))
        self.leaf_off = t(self.p.leaf_offsets.view(np.int64))
        self.leaf_len = t(self.p.leaf_lengths.view(np.int32))
        self.seg_first_dev = t(self.p.seg_first.view(np.int64))
        if out is not None and out.numel() < self.p.out_bytes:
            raise ValueError("output buffer too small for the workload")
        self.out = out[: self.p.out_bytes] if out is not None else torch.empty(self.p.out_bytes, dtype=torch.uint8,
                                                                                device=d)
        n = max(len(self.p.leaf_lengths), 1)
        self.digests = torch.empty((n, 32), dtype=torch.uint8, device=d)
        self.roots = torch.empty((max(w.n_seq, 1), 32), dtype=torch.uint8, device=d)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        L = _native.lib()
        sf = self.p.seg_first
        self.seg_scratch_bytes = int(L.tcx_merkle_segments_scratch_bytes(sf.ctypes.data, w.n_seq)) if w.n_seq else 0
        self.seg_scratch = torch.empty(max(self.seg_scratch_bytes, 256), dtype=torch.uint8, device=d)
        self.aligned16 = bool((self.p.leaf_offsets % 16 == 0).all())

    @property
    def gathered_bytes(self) -> int:
        return int(self.w.seq_bytes().sum())

    def run(self, pool: torch.Tensor, stream=None) -> None:
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        w, p = self.w, self.p
        if w.n_seq == 0:
            return
        _native.call("tcx_kv_gather", pool.data_ptr(), w.planes, w.pool_pages, w.page_tokens, w.token_bytes,
                     self.page_table.data_ptr(), self.page_offsets.data_ptr(), self.seq_tokens.data_ptr(),
                     self.out_offsets.data_ptr(), w.n_seq, int(w.page_offsets[-1]), self.out.data_ptr(),
                     p.out_bytes, self.status.data_ptr(), s)
        _native.call("tcx_sha256_leaf_table", self.out.data_ptr(), self.leaf_off.data_ptr(), self.leaf_len.data_ptr(),
                     len(p.leaf_lengths), int(self.aligned16), self.digests.data_ptr(), s)
        _native.call("tcx_merkle_roots_segmented", self.digests.data_ptr(), p.seg_first.ctypes.data,
                     self.seg_first_dev.data_ptr(), w.n_seq, self.seg_scratch.data_ptr(), self.seg_scratch_bytes,
                     self.roots.data_ptr(), s)

    def check_status(self) -> None:
        code = int(self.status.item())
        if code:
            raise _native.TcxError(_native.DATA_LOSS,
                                   {1: "page slot outside the pool", 2: "page past the sequence's tokens",
                                    3: "output past the buffer"}.get(code, f"kv gather status {code}"))

    def multihashes(self) -> list[str]:
        return [multibase_multihash_sha256(bytes(r)) for r in self.roots[: self.w.n_seq].cpu().numpy()]

    def sequence(self, i: int) -> torch.Tensor:
        o, b = int(self.p.out_offsets[i]), int(self.w.seq_bytes()[i])
        return self.out[o:o + b]
