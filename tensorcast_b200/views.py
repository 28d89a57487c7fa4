"""View specs and the view planner: which canonical bytes a view holds and where.

Mirrors the reference (same rules, same error messages):

* ``NarrowOp`` / ``TransposeOp`` / ``ViewSpec``  -> contracts/view/view_spec.h:12-51
* ``normalize_slices``      -> validate_narrow (tensorcast/api/_view_ops.py:193-248):
                               slice or (dim, slice), step 1, one narrow per tensor; a full
                               slice is no op
* ``normalize_transpose``   -> validate_transpose (tensorcast/api/_view_ops.py:251+)
* ``plan_view``             -> compute_bidirectional_internal (view_planner.cc:358-668) with
                               validate_ops (:42-72): names in subset order (first occurrence)
                               or sorted, each tensor start 8-byte aligned, a narrow along d
                               becomes prod(shape[:d]) rows of length*inner*esize bytes, a
                               transpose composes into a permutation applied after the copy
                               (execute_transform, view_transform_executor.cc:74-133)

A narrow and a transpose on the same tensor are rejected as in the reference unless
``allow_fused=True``; then the narrowed block is permuted (an extension with no reference
result, checked against numpy ``narrow(...).permute(...)``).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .artifact import CANONICAL_ALIGN, CanonicalIndex

JOB_DTYPE = np.dtype([("src_off", "<u8"), ("dst_off", "<u8"), ("src_pitch", "<u8"), ("dst_pitch", "<u8"),
                      ("row_bytes", "<u8"), ("rows", "<u8")])
MAX_DIMS = 8


@dataclass(frozen=True)
class NarrowOp:
    dim: int
    start: int
    length: int


@dataclass(frozen=True)
class TransposeOp:
    dim0: int
    dim1: int


@dataclass
class ViewSpec:
    tensors: dict = field(default_factory=dict)  # name -> list of ops

    def is_empty(self) -> bool:
        return not any(self.tensors.values())


def normalize_slice(name: str, shape, spec):
    """validate_narrow: returns NarrowOp or None (full range)."""
    if isinstance(spec, (list, tuple)) and len(spec) == 1 and not isinstance(spec[0], int):
        spec = spec[0]
    if isinstance(spec, slice):
        dim, sl = 0, spec
    elif isinstance(spec, tuple) and len(spec) == 2 and isinstance(spec[0], int) and isinstance(spec[1], slice):
        dim, sl = spec
    else:
        raise ValueError("Slice spec must be a slice object or (dim, slice) tuple")
    nd = len(shape)
    if dim < 0 or dim >= nd:
        raise ValueError(f"Slice dim {dim} out of range for tensor '{name}' (ndim={nd})")
    step = 1 if sl.step is None else sl.step
    if step != 1:
        raise ValueError(f"Slice step must be 1 for tensor '{name}'")
    extent = shape[dim]
    start = 0 if sl.start is None else int(sl.start)
    stop = extent if sl.stop is None else int(sl.stop)
    if start < 0:
        start += extent
    if stop < 0:
        stop += extent
    if start < 0 or start >= extent:
        raise ValueError(f"Slice start {start} out of range for tensor '{name}'")
    if stop <= start:
        raise ValueError(f"Slice stop {stop} must be greater than start {start} for tensor '{name}'")
    length = stop - start
    if start + length > extent:
        raise ValueError(f"Slice range [{start}, {stop}) exceeds dimension {extent} for tensor '{name}'")
    if start == 0 and length == extent:
        return None
    return NarrowOp(int(dim), int(start), int(length))


def normalize_transpose(name: str, shape, ops) -> list:
    nd = len(shape)
    if not ops:
        raise ValueError(f"Transpose spec for '{name}' must be a non-empty sequence")
    out = []
    for d0, d1 in ops:
        if d0 < 0:
            d0 += nd
        if d1 < 0:
            d1 += nd
        if not (0 <= d0 < nd and 0 <= d1 < nd):
            raise ValueError(f"Transpose dims out of range for tensor '{name}'")
        if d0 == d1:
            raise ValueError(f"Transpose dims must differ for tensor '{name}'")
        out.append(TransposeOp(int(d0), int(d1)))
    return out


def build_view_spec(index: CanonicalIndex, slices=None, transpose=None) -> ViewSpec:
    spec = ViewSpec()
    for name, s in (slices or {}).items():
        if name not in index.entries:
            raise ValueError(f"ViewSpec references unknown tensor: {name}")
        op = normalize_slice(name, index.entries[name].shape, s)
        if op is not None:
            spec.tensors.setdefault(name, []).append(op)
    for name, t in (transpose or {}).items():
        if name not in index.entries:
            raise ValueError(f"ViewSpec references unknown tensor: {name}")
        spec.tensors.setdefault(name, []).extend(normalize_transpose(name, index.entries[name].shape, t))
    return spec


@dataclass
class ViewTensor:
    name: str
    offset: int  # byte offset in the view buffer
    nbytes: int
    shape: tuple
    dtype: str


@dataclass
class ViewPlan:
    tensors: list  # ViewTensor in view order
    view_bytes: int
    jobs: np.ndarray  # JOB_DTYPE copy jobs (src in the canonical space, dst in the view)
    permutes: list  # dicts: dst_off, esize, shape, perm (in place over the view)
    is_identity: bool


def _validate_ops(ops, allow_fused: bool) -> None:
    mode, seen_narrow = None, False
    for op in ops:
        if isinstance(op, NarrowOp):
            if mode == "t" and not allow_fused:
                raise ValueError("mixing transpose and narrow in the same tensor is not supported")
            if seen_narrow:
                raise ValueError("multiple narrow ops per tensor are not supported")
            seen_narrow, mode = True, "n"
        elif isinstance(op, TransposeOp):
            if mode == "n" and not allow_fused:
                raise ValueError("mixing transpose and narrow in the same tensor is not supported")
            if op.dim0 == op.dim1:
                raise ValueError("transpose dims must be different")
            mode = "t"
        else:
            raise ValueError("unsupported view operation kind")


def plan_view(index: CanonicalIndex, spec: ViewSpec | None = None, subset=None, allow_fused: bool = False) -> ViewPlan:
    spec = spec or ViewSpec()
    for name, ops in spec.tensors.items():
        if name not in index.entries:
            raise ValueError(f"ViewSpec references unknown tensor: {name}")
        _validate_ops(ops, allow_fused)
    subset = list(subset) if subset else []
    for name in subset:
        if name not in index.entries:
            raise ValueError(f"View subset references unknown tensor: {name}")
    if subset:
        order = list(dict.fromkeys(subset))
    else:
        order = list(index.entries)
    jobs, permutes, tensors = [], [], []
    cursor, has_transform = 0, False
    for name in order:
        e = index.entries[name]
        if cursor % CANONICAL_ALIGN:
            cursor += CANONICAL_ALIGN - cursor % CANONICAL_ALIGN
        es = e.esize
        shape = list(e.shape)
        ops = spec.tensors.get(name, [])
        narrow = next((o for o in ops if isinstance(o, NarrowOp)), None)
        perm = list(range(len(shape)))
        for o in ops:
            if isinstance(o, TransposeOp):
                if not (0 <= o.dim0 < len(perm) and 0 <= o.dim1 < len(perm)):
                    raise ValueError(f"transpose dims out of range for tensor {name}")
                perm[o.dim0], perm[o.dim1] = perm[o.dim1], perm[o.dim0]
        dst = cursor
        nbytes = e.size
        view_shape = tuple(shape)
        if narrow is not None:
            d = narrow.dim
            if narrow.length == 0:
                raise ValueError(f"narrow length must be > 0 for tensor {name}")
            if d < 0 or d >= len(shape):
                raise ValueError(f"narrow dim out of range for tensor {name}")
            extent = shape[d]
            start = narrow.start + extent if narrow.start < 0 else narrow.start
            if start < 0 or start >= extent:
                raise ValueError(f"narrow start out of range for tensor {name}")
            if start + narrow.length > extent:
                raise ValueError(f"narrow length exceeds dimension for tensor {name}")
            if not (start == 0 and narrow.length == extent):
                has_transform = True
                inner = int(np.prod(shape[d + 1:], dtype=np.int64)) if d + 1 < len(shape) else 1
                outer = int(np.prod(shape[:d], dtype=np.int64)) if d > 0 else 1
                row = narrow.length * inner * es
                jobs.append((e.offset + start * inner * es, dst, extent * inner * es, row, row, max(outer, 1)))
                shape[d] = narrow.length
                view_shape = tuple(shape)
                nbytes = row * max(outer, 1)
                narrow = "applied"
        if narrow != "applied":
            jobs.append((e.offset, dst, e.size, e.size, e.size, 1))
        if perm != list(range(len(perm))):
            has_transform = True
            if len(shape) > MAX_DIMS:
                raise ValueError(f"tensor {name} has more than {MAX_DIMS} dimensions")
            permutes.append({"dst_off": dst, "esize": es, "shape": tuple(shape), "perm": tuple(perm)})
            view_shape = tuple(shape[p] for p in perm)
        tensors.append(ViewTensor(name, dst, nbytes, view_shape, e.dtype))
        cursor = dst + nbytes
    job_arr = np.array(jobs, dtype=JOB_DTYPE) if jobs else np.zeros(0, JOB_DTYPE)
    return ViewPlan(tensors, cursor, job_arr, permutes, is_identity=not has_transform and not subset)


def permute_array(permutes: list) -> np.ndarray:
    """Permute descriptors as the tcx_permute_job C struct layout (for the C ABI)."""
    dt = np.dtype([("src_off", "<u8"), ("dst_off", "<u8"), ("esize", "<u4"), ("ndim", "<u4"),
                   ("shape", "<i8", (MAX_DIMS,)), ("perm", "<i4", (MAX_DIMS,))])
    arr = np.zeros(len(permutes), dt)
    for i, p in enumerate(permutes):
        arr[i]["src_off"] = p["dst_off"]
        arr[i]["dst_off"] = p["dst_off"]
        arr[i]["esize"] = p["esize"]
        arr[i]["ndim"] = len(p["shape"])
        arr[i]["shape"][: len(p["shape"])] = p["shape"]
        arr[i]["perm"][: len(p["perm"])] = p["perm"]
    return arr
