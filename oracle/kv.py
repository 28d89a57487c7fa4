"""CPU oracle for the paged KV gather + per-sequence hash. TEST INFRASTRUCTURE ONLY.

There is no reference implementation of this step; the oracle is a numpy gather
(pages -> [plane][token][token_bytes] per sequence) plus the reference's tree hash
(oracle.leaf_digests / tree_root / multihash, artifact_hash_cpu.cc:198-254) at the
given leaf size.
"""
from __future__ import annotations

import numpy as np

from . import oracle


def gather_sequence(pool: np.ndarray, planes: int, pool_pages: int, page_tokens: int, token_bytes: int,
                    slots: np.ndarray, tokens: int) -> np.ndarray:
    page_bytes = page_tokens * token_bytes
    P = pool.reshape(planes, pool_pages, page_bytes)
    parts = []
    for k in range(planes):
        seq = P[k, slots.astype(np.int64)].reshape(-1)[: tokens * token_bytes]
        parts.append(seq)
    return np.concatenate(parts)


def sequence_multihash(seq_bytes: np.ndarray, leaf: int) -> str:
    d = oracle.leaf_digests(seq_bytes, leaf, openssl=True, threads=8)
    return oracle.multihash(oracle.tree_root(d))
