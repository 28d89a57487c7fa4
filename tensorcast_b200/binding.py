"""Loads into caller-owned CUDA tensors: the reference's ``Artifact.bind_into``.

Mirrors the SDK surface of tensorcast/api/store/mapped_binding.py (``Range``,
``CopyPlanEntry``, ``copy_plan_to_json`` / ``copy_plan_from_json``,
``normalize_copy_plan``, ``validate_copy_plan``; same JSON format, checks, messages and
status codes) and turns a binding into copy jobs whose destinations are the targets'
own device addresses, so the collective load writes every byte straight into the
caller's tensors (``TCX_LOAD_TARGETS``): no view buffer, no second copy.

A copy-plan entry moves a slice of one checkpoint tensor (a range on dim 0 or 1, or the
whole tensor) into a slice of one target along the same dim. A dim-0 slice of a
contiguous tensor is one contiguous byte run; a dim-1 slice is ``shape[0]`` rows at the
tensor's row pitch — one strided copy job (the reference's rect2d). Several entries into
one target concatenate along their dim (the reference's concat jobs, e.g. a fused QKV
weight built from q, k and v).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Mapping, Sequence

import numpy as np

from .views import JOB_DTYPE

_COPY_PLAN_VERSION = 1


class BindingError(RuntimeError):
    def __init__(self, message: str, status_code: str = "INVALID_ARGUMENT", retryable: bool = False):
        super().__init__(message)
        self.status_code = status_code
        self.retryable = retryable


def _err(msg: str, code: str = "INVALID_ARGUMENT") -> BindingError:
    # api.ArtifactError is a subclass of RuntimeError with the same fields; raise the
    # SDK's error type when it is importable so callers catch one class.
    try:
        from .api import ArtifactError
        return ArtifactError(msg, code)
    except ImportError:  # pragma: no cover
        return BindingError(msg, code)


@dataclass(frozen=True, slots=True)
class Range:
    dim: int
    start: int
    end: int

    @property
    def length(self) -> int:
        return int(self.end) - int(self.start)


@dataclass(frozen=True, slots=True)
class CopyPlanEntry:
    ckpt_name: str
    ckpt_range: Range | None
    dst_name: str
    dst_range: Range | None


CopyPlan = Sequence[CopyPlanEntry]


def _range_to_dict(r: Range | None):
    return None if r is None else {"dim": int(r.dim), "start": int(r.start), "end": int(r.end)}


def _range_from_dict(d) -> Range | None:
    if d is None:
        return None
    if isinstance(d, Range):
        return d
    if not isinstance(d, Mapping):
        raise _err("copy plan ranges must be objects with dim, start and end")
    try:
        return Range(dim=int(d["dim"]), start=int(d["start"]), end=int(d["end"]))
    except (KeyError, TypeError, ValueError) as exc:
        raise _err(f"invalid copy plan range {d!r}") from exc


def _entry_from_dict(d: Mapping) -> CopyPlanEntry:
    return CopyPlanEntry(ckpt_name=str(d.get("ckpt_name", "")), ckpt_range=_range_from_dict(d.get("ckpt_range")),
                         dst_name=str(d.get("dst_name", "")), dst_range=_range_from_dict(d.get("dst_range")))


def copy_plan_to_json(plan: CopyPlan) -> str:
    entries = [{"ckpt_name": e.ckpt_name, "ckpt_range": _range_to_dict(e.ckpt_range), "dst_name": e.dst_name,
                "dst_range": _range_to_dict(e.dst_range)} for e in plan]
    return json.dumps({"version": _COPY_PLAN_VERSION, "entries": entries}, sort_keys=True, separators=(",", ":"))


def copy_plan_from_json(data: str) -> tuple[CopyPlanEntry, ...]:
    try:
        payload = json.loads(data)
    except json.JSONDecodeError as exc:
        raise _err(f"Invalid copy plan JSON: {exc}") from exc
    if not isinstance(payload, dict):
        raise _err("Copy plan JSON must be an object")
    version = int(payload.get("version", 0))
    if version != _COPY_PLAN_VERSION:
        raise _err(f"Unsupported copy plan version {version}")
    entries = payload.get("entries")
    if not isinstance(entries, list) or not entries:
        raise _err("Copy plan JSON requires a non-empty entries list")
    out = []
    for e in entries:
        if not isinstance(e, dict):
            raise _err("Copy plan entries must be objects")
        out.append(_entry_from_dict(e))
    return tuple(out)


def normalize_copy_plan(plan) -> tuple[CopyPlanEntry, ...]:
    if not isinstance(plan, Sequence) or isinstance(plan, (str, bytes)) or not plan:
        raise _err("mapping must be a non-empty sequence of CopyPlanEntry objects")
    out = []
    for e in plan:
        if isinstance(e, CopyPlanEntry):
            out.append(e)
        elif isinstance(e, Mapping):
            out.append(_entry_from_dict(e))
        elif isinstance(e, tuple) and len(e) == 4:
            out.append(CopyPlanEntry(str(e[0]), _range_from_dict(e[1]), str(e[2]), _range_from_dict(e[3])))
        else:
            raise _err("mapping entries must be CopyPlanEntry objects or dicts")
    return tuple(out)


def _compact_stride(shape) -> tuple:
    st, acc = [0] * len(shape), 1
    for i in range(len(shape) - 1, -1, -1):
        st[i] = acc
        acc *= int(shape[i])
    return tuple(st)


def _resolve_dim(a: Range | None, b: Range | None):
    if a is not None and b is not None:
        if a.dim != b.dim:
            raise _err(f"mapping range dims differ ({a.dim} vs {b.dim})")
        return int(a.dim)
    if a is not None:
        return int(a.dim)
    if b is not None:
        return int(b.dim)
    return None


def _interval(dim, shape, rng: Range | None) -> tuple[int, int]:
    if not shape:
        return (0, 1)
    if dim is None:
        dim = int(rng.dim) if rng is not None else 0
    if dim < 0 or dim >= len(shape):
        raise _err(f"Slice dim {dim} out of range for shape {tuple(shape)}")
    if rng is None:
        return (0, int(shape[dim]))
    return (int(rng.start), int(rng.end))


def _count(shape, dim, start, end) -> int:
    if not shape:
        return 1
    dim = 0 if dim is None else dim
    c = int(end) - int(start)
    for i, s in enumerate(shape):
        if i != dim:
            c *= int(s)
    return c


def _check_range(idx, name, shape, rng: Range | None, narrow: Range | None, role: str) -> None:
    if not shape:
        if rng is not None:
            raise _err(f"mapping entry {idx} {role} range set for scalar '{name}'")
        return
    if rng is None:
        if narrow is not None:
            raise _err(f"mapping entry {idx} {role} range required for view-narrowed tensor '{name}'")
        return
    dim = int(rng.dim)
    if dim not in (0, 1):
        raise _err(f"mapping entry {idx} {role} dim must be 0 or 1")
    if dim >= len(shape):
        raise _err(f"mapping entry {idx} {role} dim {dim} out of range for '{name}'")
    if rng.start < 0 or rng.end <= rng.start:
        raise _err(f"mapping entry {idx} {role} range must have start < end")
    if rng.end > shape[dim]:
        raise _err(f"mapping entry {idx} {role} range exceeds shape for '{name}'")
    if narrow is not None:
        if dim != narrow.dim:
            raise _err(f"mapping entry {idx} {role} dim {dim} does not match view narrow dim {narrow.dim} for '{name}'")
        if rng.start < narrow.start or rng.end > narrow.end:
            raise _err(f"mapping entry {idx} {role} range outside view bounds for '{name}' "
                       f"({narrow.start}:{narrow.end})")


def validate_copy_plan(*, plan: CopyPlan, canonical_index, target_tensors, view_narrows=None,
                       require_full_coverage: bool = True) -> None:
    """validate_copy_plan (mapped_binding.py:287-426): names, contiguity, dtypes, ranges,
    element counts, one slice dim per target, no overlaps and (optionally) full coverage."""
    if not plan:
        raise _err("mapping must include at least one entry")
    if {e.dst_name for e in plan} != {str(n) for n in target_tensors}:
        raise _err("mapping dst_name set must match target_tensors", "FAILED_PRECONDITION")
    entries = canonical_index.entries
    slices: dict[str, list] = {}
    dims: dict[str, int] = {}
    for idx, e in enumerate(plan):
        if not e.ckpt_name:
            raise _err(f"mapping entry {idx} missing ckpt_name")
        if not e.dst_name:
            raise _err(f"mapping entry {idx} missing dst_name")
        src = entries.get(e.ckpt_name)
        if src is None:
            raise _err(f"mapping entry {idx} references unknown source '{e.ckpt_name}'")
        if tuple(src.stride) != _compact_stride(src.shape):
            raise _err(f"mapping source '{e.ckpt_name}' must be contiguous", "FAILED_PRECONDITION")
        dst = target_tensors.get(e.dst_name)
        if dst is None:
            raise _err(f"mapping entry {idx} references unknown target '{e.dst_name}'")
        if not dst.is_contiguous():
            raise _err(f"mapping target '{e.dst_name}' must be contiguous", "FAILED_PRECONDITION")
        if int(dst.storage_offset()) != 0:
            raise _err(f"mapping target '{e.dst_name}' must have storage_offset=0", "FAILED_PRECONDITION")
        if str(dst.dtype) != src.dtype:
            raise _err(f"mapping entry {idx} dtype mismatch: {e.ckpt_name}({src.dtype}) -> {e.dst_name}({dst.dtype})")
        narrow = (view_narrows or {}).get(e.ckpt_name)
        _check_range(idx, e.ckpt_name, tuple(src.shape), e.ckpt_range, narrow, "source")
        dshape = tuple(int(v) for v in dst.shape)
        _check_range(idx, e.dst_name, dshape, e.dst_range, None, "target")
        dim = _resolve_dim(e.ckpt_range, e.dst_range)
        if dim is not None:
            prev = dims.get(e.dst_name)
            if prev is None:
                dims[e.dst_name] = dim
            elif prev != dim:
                raise _err(f"mapping target '{e.dst_name}' mixes slice dims {prev} and {dim}")
        a, b = _interval(dim, dshape, e.dst_range)
        slices.setdefault(e.dst_name, []).append((a, b, idx))
        sshape = tuple(src.shape)
        if sshape:
            s0, s1 = _interval(dim, sshape, e.ckpt_range)
            if narrow is not None:
                s0, s1 = s0 - narrow.start, s1 - narrow.start
            scount = _count(sshape, dim, s0, s1)
        else:
            scount = 1
        dcount = _count(dshape, dim, a, b) if dshape else 1
        if scount != dcount:
            raise _err(f"mapping entry {idx} element count mismatch ({scount} != {dcount})")
    for name, t in target_tensors.items():
        iv = sorted(slices.get(name, ()))
        if not iv:
            raise _err(f"mapping missing target '{name}'")
        shape = tuple(int(v) for v in t.shape)
        if not shape:
            if len(iv) != 1:
                raise _err(f"mapping target '{name}' must have a single entry for scalar")
            continue
        dim = dims.get(name, 0)
        cursor = 0
        for a, b, idx in iv:
            if a < cursor:
                raise _err(f"mapping entry {idx} overlaps prior slice for '{name}'")
            if require_full_coverage and a != cursor:
                raise _err(f"mapping target '{name}' has gaps before entry {idx}")
            cursor = b
        if require_full_coverage and cursor != shape[dim]:
            raise _err(f"mapping target '{name}' does not cover full dim {dim}")


def _side(shape, esize: int, base_off: int, dim, rng: Range | None):
    """(offset, rows, row_bytes, pitch) of a slice of a contiguous tensor."""
    shape = tuple(int(v) for v in shape)
    if not shape or dim is None or rng is None:
        n = esize
        for s in shape:
            n *= s
        return base_off, 1, n, n
    inner = esize
    for s in shape[dim + 1:]:
        inner *= s
    if dim == 0:
        return base_off + rng.start * inner, 1, rng.length * inner, rng.length * inner
    outer = shape[0]
    return base_off + rng.start * inner, outer, rng.length * inner, shape[1] * inner


def mapped_copy_jobs(plan: CopyPlan, canonical_index, target_tensors, base_ptr: int) -> np.ndarray:
    """One copy job per plan entry: canonical source slice -> target slice, destinations as
    device addresses relative to base_ptr (entries validated by validate_copy_plan)."""
    jobs = []
    for idx, e in enumerate(plan):
        src = canonical_index.entries[e.ckpt_name]
        es = src.esize
        dim = _resolve_dim(e.ckpt_range, e.dst_range)
        src_rng = e.ckpt_range if e.ckpt_range is not None or dim is None else \
            Range(dim, 0, int(src.shape[dim]))
        dst = target_tensors[e.dst_name]
        dst_rng = e.dst_range if e.dst_range is not None or dim is None else Range(dim, 0, int(dst.shape[dim]))
        so, sr, sb, sp = _side(src.shape, es, src.offset, dim, src_rng)
        do, dr, db, dp = _side(dst.shape, es, dst.data_ptr() - base_ptr, dim, dst_rng)
        if sr * sb != dr * db:
            raise _err(f"mapping entry {idx} element count mismatch ({sr * sb // es} != {dr * db // es})")
        if (sr, sb) != (dr, db):
            contiguous = (sr == 1 or sp == sb) and (dr == 1 or dp == db)
            if not contiguous:
                raise _err(f"mapping entry {idx}: source and target slices have different row layouts "
                           f"({sr} x {sb} B vs {dr} x {db} B)")
            sr, sb, sp, dr, db, dp = 1, sr * sb, sr * sb, 1, dr * db, dr * db
        jobs.append((so, do, sp if sr > 1 else sb, dp if dr > 1 else db, sb, sr))
    return np.array(jobs, dtype=JOB_DTYPE) if jobs else np.zeros(0, JOB_DTYPE)


def target_ranges(target_tensors) -> tuple[int, list, int]:
    """(base address, sorted (offset, length) ranges relative to it, view bytes) of targets."""
    base = min(t.data_ptr() for t in target_tensors.values())
    ranges = sorted((t.data_ptr() - base, t.numel() * t.element_size()) for t in target_tensors.values())
    for (a0, l0), (a1, _) in zip(ranges, ranges[1:]):
        if a1 < a0 + l0:
            raise _err("bind_into targets must not overlap")
    return base, ranges, max(a + n for a, n in ranges)


def view_target_jobs(plan, target_tensors, base: int):
    """A view plan's copy jobs and permutes re-addressed from the view buffer to the target
    tensor of each view tensor (same shape and dtype, contiguous)."""
    delta = {}
    for t in plan.tensors:
        tgt = target_tensors[t.name]
        if tuple(tgt.shape) != tuple(t.shape) or str(tgt.dtype) != t.dtype:
            raise _err(f"bind_into target '{t.name}' must be {t.dtype}{list(t.shape)}, got "
                       f"{tgt.dtype}{list(tgt.shape)}", "FAILED_PRECONDITION")
        if not tgt.is_contiguous():
            raise _err(f"bind_into target '{t.name}' must be contiguous", "FAILED_PRECONDITION")
        if t.nbytes:  # an empty tensor has no jobs and may share its offset with the next
            delta[t.offset] = tgt.data_ptr() - base - t.offset
    starts = sorted(delta)

    def moved(off: int) -> int:
        i = int(np.searchsorted(starts, off, side="right")) - 1
        return off + delta[starts[i]]

    jobs = plan.jobs.copy()
    for j in jobs:
        j["dst_off"] = moved(int(j["dst_off"]))
    permutes = [dict(p, dst_off=moved(int(p["dst_off"]))) for p in plan.permutes]
    return jobs, permutes
