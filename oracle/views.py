"""CPU view oracle. TEST INFRASTRUCTURE ONLY (imported by tests/, smoke() and bench.py's checks).

Materialises a view of a canonical byte space with numpy, independently of the
product planner (tensorcast_b200/views.py) and its copy jobs: every tensor is read
as an array of its element width, narrowed with numpy slicing and permuted with
``np.transpose(...)`` + ``ascontiguousarray``.

Restates, byte for byte:
* the canonical byte space (canonical_index.cc:155-221): names sorted bytewise, each start
  aligned to 8 bytes, pad bytes zero;
* the view layout of compute_bidirectional_internal (view_planner.cc:358-668): subset
  order (first occurrence) or sorted order, 8-byte aligned starts with zero pads, a narrow
  keeps the slice, a transpose is ``permute(perm).contiguous()``
  (view_transform_executor.cc:116-131);
* the fused narrow + transpose extension (no reference result): narrow, then permute.
"""
from __future__ import annotations

import numpy as np

_UINT = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}


def canonical_bytes(tensors: dict) -> tuple[np.ndarray, dict]:
    """tensors: name -> (raw bytes as uint8 array, shape, esize). Returns (canonical bytes,
    name -> (offset, shape, esize))."""
    names = sorted(tensors, key=lambda s: s.encode("utf-8"))
    offsets, cursor = {}, 0
    for n in names:
        if cursor % 8:
            cursor += 8 - cursor % 8
        offsets[n] = cursor
        cursor += tensors[n][0].size
    out = np.zeros(cursor, np.uint8)
    meta = {}
    for n in names:
        raw, shape, es = tensors[n]
        out[offsets[n]:offsets[n] + raw.size] = raw
        meta[n] = (offsets[n], tuple(shape), es)
    return out, meta


def materialize_view(canon: np.ndarray, meta: dict, slices=None, transpose=None, subset=None) -> np.ndarray:
    """meta: name -> (offset, shape, esize). slices: name -> (dim, start, length).
    transpose: name -> list of (d0, d1). Returns the view bytes."""
    slices, transpose = slices or {}, transpose or {}
    order = list(dict.fromkeys(subset)) if subset else sorted(meta, key=lambda s: s.encode("utf-8"))
    parts, cursor = [], 0
    for n in order:
        off, shape, es = meta[n]
        numel = int(np.prod(shape, dtype=np.int64)) if shape else 1
        arr = canon[off:off + numel * es].view(_UINT[es]).reshape(shape)
        if n in slices:
            d, s, ln = slices[n]
            idx = [slice(None)] * len(shape)
            idx[d] = slice(s, s + ln)
            arr = arr[tuple(idx)]
        if n in transpose:
            perm = list(range(arr.ndim))
            for a, b in transpose[n]:
                perm[a], perm[b] = perm[b], perm[a]
            arr = np.transpose(arr, perm)
        data = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        pad = (8 - cursor % 8) % 8
        if pad:
            parts.append(np.zeros(pad, np.uint8))
            cursor += pad
        parts.append(data)
        cursor += data.size
    return np.concatenate(parts) if parts else np.zeros(0, np.uint8)


def tp_slices(meta: dict, world: int, rank: int) -> dict:
    """The Llama tensor-parallel sharding of the benchmark loads: q/k/v/gate/up, embed and
    lm_head split along dim 0, o_proj/down_proj along dim 1, everything else whole."""
    out = {}
    for n, (_, shape, _) in meta.items():
        if any(k in n for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "embed_tokens", "lm_head")):
            d = 0
        elif any(k in n for k in ("o_proj", "down_proj")):
            d = 1
        else:
            continue
        ext = shape[d]
        if ext % world:
            raise ValueError(f"{n}: dim {d} ({ext}) is not divisible by {world}")
        ln = ext // world
        out[n] = (d, rank * ln, ln)
    return out
