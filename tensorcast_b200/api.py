"""The reference's Python realization surface, over the native collective loader.

Same names, arguments and error behaviour as the TensorCast SDK for this path:

* ``from_disk(path, *, key=None, verify_checksums=True, show_progress=None)``
  (tensorcast/api/store/__init__.py:4548-4560, method :3294-3388)
* ``Artifact.subset(names)`` / ``Artifact.view(*, slices=None, transpose=None)`` /
  ``Artifact.tensor_dict(*, device, options=None, ctx=None)``
  (tensorcast/api/store/artifact.py:1779, 1765-1776, 1509-1520)
* ``Artifact.bind_into(target_tensors, *, mapping=None, packing=..., options=None, ctx=None)``
  (tensorcast/api/store/artifact.py:1889-2110): the load writes straight into caller-owned
  CUDA tensors, optionally through a copy plan (``binding.py``)
* ``CallContext(collective=CollectiveLoadGroup(group_id, world_size, rank))``
  (tensorcast/api/context.py:13-18)

Instead of a gRPC call into a daemon, ``tensor_dict`` runs the load in-process: each
rank stages its leaf-aligned 1/N of the canonical bytes (read from the files inside the
load), the ranks exchange the bytes of each other's views over NVLink, and every rank
returns its tensors as views of one device buffer. Ranks are either one process per GPU
joined by torch.distributed, or -- the reference daemon's model -- threads of one
process that call with the same ``CollectiveLoadGroup.group_id`` (one thread per GPU).

Verification follows verification_stage.cc:55-141: the data multihash of the loaded
bytes is always computed on the GPU (leaf size from the adaptive policy of
compute_data_multihash_from_gpu, unless ``leaf_chunk_bytes`` is given); when an
``artifact_descriptor.json`` next to the artifact holds a data multihash, a mismatch
raises ``ArtifactError`` with status DATA_LOSS ("ARTIFACT_ID_MISMATCH").
"""
from __future__ import annotations

import json
import os
import threading
import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _native
from .artifact import build_canonical_index, build_source_index, canonical_segments, pad_ranges, safetensors_files
from .hashing import DEFAULT_LEAF_CHUNK_BYTES, determine_leaf_chunk_size
from .loader import Group, read_segments, stage_bounds
from .views import JOB_DTYPE, build_view_spec, plan_view

_TORCH_DTYPES = {
    "torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16, "torch.float32": torch.float32,
    "torch.float": torch.float32, "torch.float64": torch.float64, "torch.double": torch.float64,
    "torch.int8": torch.int8, "torch.uint8": torch.uint8, "torch.int16": torch.int16, "torch.int32": torch.int32,
    "torch.int64": torch.int64, "torch.bool": torch.bool, "torch.float8_e4m3fn": torch.float8_e4m3fn,
    "torch.float8_e5m2": torch.float8_e5m2,
}


class ArtifactError(RuntimeError):
    def __init__(self, message: str, status_code: str = "INTERNAL", retryable: bool = False):
        super().__init__(message)
        self.status_code = status_code
        self.retryable = retryable


@dataclass(frozen=True)
class CollectiveLoadGroup:
    """Explicit collective load contract for a single materialization call."""

    group_id: str
    world_size: int
    rank: int


@dataclass(frozen=True)
class CallContext:
    collective: CollectiveLoadGroup | None = None


@dataclass(frozen=True)
class GetArtifactOptions:
    export_policy: str | None = None
    direct_io: bool = False  # stage with O_DIRECT reads (cold block devices); buffered where refused


_GROUPS: dict = {}


def _process_model(world: int, rank: int) -> bool:
    """True when torch.distributed holds this group's ranks (one process per GPU);
    otherwise the ranks are threads of this process that find each other by group id
    (the reference daemon's model)."""
    import torch.distributed as dist
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() == world and \
        dist.get_rank() == rank


def _reader_threads(world: int, rank: int) -> int:
    """Host reader threads for this rank's file staging: the CPUs this process may run on,
    shared with the other ranks of this host (the rank threads of this process, or
    LOCAL_WORLD_SIZE processes), at least 2 and at most 32 per rank."""
    cpus = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 4)
    if world <= 1:
        sharing = 1
    elif _process_model(world, rank):
        sharing = max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1") or 1))
    else:
        sharing = world  # rank threads of this process
    return max(2, min(32, cpus // sharing))


_GROUPS_LOCK = threading.Lock()


def _group_for(device_index: int, world: int, rank: int, group_id: str) -> Group:
    key = (device_index, world, rank, group_id)
    with _GROUPS_LOCK:
        g = _GROUPS.get(key)
    if g is None:
        if world == 1:
            g = Group(1, 0, device_index)
        elif _process_model(world, rank):
            g = Group.from_torch_distributed(device_index)
        elif group_id:
            g = Group.join(group_id, world, rank, device_index)
        else:
            raise ArtifactError("a collective load needs torch.distributed initialised with the group's ranks, or a "
                                "group_id shared by the rank threads of this process", "FAILED_PRECONDITION")
        with _GROUPS_LOCK:
            _GROUPS[key] = g
    return g


_RDV = threading.Condition()
_RDV_TABLE: dict = {}


def _gather_in_process(group_id: str, world: int, rank: int, payload: bytes, timeout_s: float = 120.0) -> list:
    """All-gather of one bytes object per rank among the rank threads of this process
    that share group_id; repeated calls with the same id form successive rounds."""
    deadline = time.monotonic() + timeout_s
    with _RDV:
        while True:
            e = _RDV_TABLE.get(group_id)
            if e is None:
                e = _RDV_TABLE[group_id] = {"world": world, "items": [None] * world, "n": 0, "taken": 0}
            if e["world"] != world:
                raise ArtifactError(f"group {group_id} gathered with world sizes {e['world']} and {world}",
                                    "INVALID_ARGUMENT")
            if e["items"][rank] is None:
                break
            if not _RDV.wait(deadline - time.monotonic()):  # an earlier round still being read
                raise ArtifactError(f"group {group_id}: rank {rank} timed out waiting for the previous round",
                                    "DEADLINE_EXCEEDED")
        e["items"][rank] = payload
        e["n"] += 1
        _RDV.notify_all()
        while e["n"] < world:
            if not _RDV.wait(deadline - time.monotonic()) and e["n"] < world:
                # withdraw this rank's item so that a later round starts clean
                e["items"][rank] = None
                e["n"] -= 1
                if e["n"] == 0:
                    del _RDV_TABLE[group_id]
                _RDV.notify_all()
                raise ArtifactError(f"group {group_id}: rank {rank} timed out waiting for {world - e['n'] - 1} "
                                    "rank(s)", "DEADLINE_EXCEEDED")
        out = list(e["items"])
        e["taken"] += 1
        if e["taken"] == world:
            del _RDV_TABLE[group_id]
            _RDV.notify_all()
    return out


def gather_rank_jobs(jobs: np.ndarray, world: int, rank: int | None = None, group_id: str | None = None) -> list:
    """Every rank's view copy jobs (all ranks call it): one all_gather of the job bytes
    over torch.distributed, or, for rank threads of one process, through group_id."""
    if world == 1:
        return [jobs]
    if rank is None or _process_model(world, rank):
        import torch.distributed as dist
        out = [None] * world
        dist.all_gather_object(out, jobs.tobytes())
    else:
        out = _gather_in_process(group_id, world, rank, jobs.tobytes())
    return [np.frombuffer(b, dtype=JOB_DTYPE).copy() for b in out]


def _read_descriptor(path: str):
    d = path if os.path.isdir(path) else os.path.dirname(path)
    p = os.path.join(d, "artifact_descriptor.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f)


class Artifact:
    """A lazy handle on a safetensors artifact (optionally a subset / view of it)."""

    def __init__(self, path: str, index, *, subset=None, spec=None, verify_checksums=True, leaf_chunk_bytes=None,
                 key=None):
        self.path, self.index, self.key = path, index, key
        self._subset, self._spec = subset, spec
        self._slices, self._transpose = {}, {}
        self.verify_checksums = verify_checksums
        self.leaf_chunk_bytes = leaf_chunk_bytes
        self.data_multihash: str | None = None

    def _derive(self, subset=None, slices=None, transpose=None) -> "Artifact":
        a = Artifact(self.path, self.index, subset=self._subset if subset is None else subset,
                     verify_checksums=self.verify_checksums, leaf_chunk_bytes=self.leaf_chunk_bytes, key=self.key)
        a._slices = dict(self._slices, **(slices or {}))
        a._transpose = dict(self._transpose, **(transpose or {}))
        a._spec = build_view_spec(self.index, a._slices, a._transpose)
        return a

    def subset(self, names) -> "Artifact":
        names = [str(n) for n in names]
        for n in names:
            if n not in self.index.entries:
                raise ValueError(f"View subset references unknown tensor: {n}")
        return self._derive(subset=names)

    def view(self, *, slices=None, transpose=None) -> "Artifact":
        return self._derive(slices=slices, transpose=transpose)

    def describe(self) -> str:
        return (f"Artifact({self.path}: {len(self.index.entries)} tensors, {self.index.total_bytes} bytes, "
                f"subset={len(self._subset) if self._subset else 'all'}, view_ops={len(self._spec.tensors) if self._spec else 0})")

    @property
    def canonical_index_json(self) -> str:
        return self.index.to_json()

    def _context(self, device, ctx):
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ArtifactError("this build materialises on CUDA devices only", "UNIMPLEMENTED")
        dev_index = dev.index if dev.index is not None else torch.cuda.current_device()
        coll = ctx.collective if ctx is not None else None
        world, rank = (coll.world_size, coll.rank) if coll is not None else (1, 0)
        if world < 1 or not (0 <= rank < world):
            raise ArtifactError("invalid collective group (world_size, rank)", "INVALID_ARGUMENT")
        return dev, dev_index, coll, world, rank

    def _load(self, dev, dev_index, coll, world, rank, jobs, permutes, view_bytes, d_view=None, alias=False,
              target_ranges=None, options: GetArtifactOptions | None = None) -> dict:
        """Stages this rank's leaf-aligned range from the files, then one tcx_group_load
        (hash + exchange + view) into d_view (None: the staged buffer, for an identity view)."""
        T = self.index.total_bytes
        L = self.leaf_chunk_bytes or determine_leaf_chunk_size(T, DEFAULT_LEAF_CHUNK_BYTES)
        rank_jobs = gather_rank_jobs(jobs, world, rank, coll.group_id if coll else None)
        bounds = stage_bounds(T, L, world)
        lo, hi = bounds[rank], bounds[rank + 1]
        with torch.cuda.device(dev_index):
            # Buffered reads stream through the group's reader threads and pinned
            # buffers inside the load (reads, copies and hashing overlap); O_DIRECT
            # reads go through aligned windows into a pinned copy of the range first.
            h_stage, files = None, canonical_segments(self.index, lo, hi)
            if options and options.direct_io:
                h_stage = torch.empty(max(hi - lo, 1), dtype=torch.uint8, pin_memory=True)
                read_segments(files, h_stage.data_ptr(), threads=min(16, os.cpu_count() or 4), direct=True)
                for off, ln in pad_ranges(self.index, lo, hi):
                    h_stage[off:off + ln].zero_()
                files = None
            d_stage = torch.empty(max(hi - lo, 1), dtype=torch.uint8, device=dev)
            if alias:
                d_view = d_stage
            elif d_view is None:
                d_view = torch.empty(max(view_bytes, 1), dtype=torch.uint8, device=dev)
            expected = None
            desc = _read_descriptor(self.path) if self.verify_checksums else None
            if desc and desc.get("data_multihash") and not self.leaf_chunk_bytes:
                expected = _root_of_multihash(desc["data_multihash"])
            group = _group_for(dev_index, world, rank, coll.group_id if coll else "")
            try:
                res = group.load(T, L, bounds, rank_jobs, d_stage=d_stage, d_view=d_view, h_stage=h_stage,
                                 files=files, permutes=permutes, view_bytes=view_bytes, expected_root=expected,
                                 target_ranges=target_ranges, read_threads=_reader_threads(world, rank))
            except _native.TcxError as e:
                code = {15: "DATA_LOSS", 3: "INVALID_ARGUMENT", 4: "DEADLINE_EXCEEDED",
                        5: "NOT_FOUND"}.get(e.code, "INTERNAL")
                raise ArtifactError(str(e), code) from e
        self.data_multihash = res["multihash"]
        res["d_view"] = d_view
        return res

    def tensor_dict(self, *, device, options: GetArtifactOptions | None = None,
                    ctx: CallContext | None = None) -> dict:
        dev, dev_index, coll, world, rank = self._context(device, ctx)
        plan = plan_view(self.index, self._spec, self._subset)
        res = self._load(dev, dev_index, coll, world, rank, plan.jobs, plan.permutes, plan.view_bytes,
                         alias=world == 1 and plan.is_identity, options=options)
        d_view = res["d_view"]
        out = {}
        for t in plan.tensors:
            dt = _TORCH_DTYPES[t.dtype]
            out[t.name] = d_view[t.offset:t.offset + t.nbytes].view(dt).view(t.shape)
        return out

    def bind_into(self, target_tensors, *, mapping=None, packing: str = "byte_space",
                  options: GetArtifactOptions | None = None, ctx: CallContext | None = None) -> "Binding":
        """Fills caller-owned CUDA tensors straight from the load (artifact.py:1889-2110).

        Without ``mapping`` the targets are the artifact's (sub)view tensors by name, with
        the same shapes and dtypes. With ``mapping`` (a copy plan, ``binding.CopyPlanEntry``)
        each entry copies a checkpoint-tensor slice into a target slice; entries into one
        target concatenate (mapped_binding.py:287-426 validation). Bytes land in the
        targets through the load's own copy kernels (TCX_LOAD_TARGETS)."""
        from . import binding as _b
        if not isinstance(target_tensors, dict) and not hasattr(target_tensors, "items"):
            raise ArtifactError("bind_into target_tensors must be a non-empty mapping", "INVALID_ARGUMENT")
        if not target_tensors:
            raise ArtifactError("bind_into target_tensors must be a non-empty mapping", "INVALID_ARGUMENT")
        if str(packing).strip().lower() not in {"append", "plan", "byte_space"}:
            raise ArtifactError("packing must be 'append', 'plan', or 'byte_space'", "INVALID_ARGUMENT")
        for name, t in target_tensors.items():
            if not isinstance(t, torch.Tensor):
                raise ArtifactError(f"bind_into target '{name}' must be a torch.Tensor", "INVALID_ARGUMENT")
            if not t.is_cuda:
                raise ArtifactError(f"bind_into target '{name}' must be CUDA", "FAILED_PRECONDITION")
        devices = {t.device.index for t in target_tensors.values()}
        if len(devices) != 1:
            raise ArtifactError("bind_into targets must share the same CUDA device", "FAILED_PRECONDITION")
        device = next(iter(target_tensors.values())).device
        dev, dev_index, coll, world, rank = self._context(device, ctx)
        base, ranges, view_bytes = _b.target_ranges(target_tensors)
        if mapping is not None:
            plan_entries = _b.normalize_copy_plan(mapping)
            narrows = {}
            for name, ops in (self._spec.tensors.items() if self._spec else ()):
                for op in ops:
                    if hasattr(op, "length"):
                        narrows[name] = _b.Range(op.dim, op.start, op.start + op.length)
                    else:
                        raise ArtifactError("mapping over a transposed view is not supported", "UNIMPLEMENTED")
            _b.validate_copy_plan(plan=plan_entries, canonical_index=self.index, target_tensors=target_tensors,
                                  view_narrows=narrows, require_full_coverage=True)
            jobs = _b.mapped_copy_jobs(plan_entries, self.index, target_tensors, base)
            permutes = []
        else:
            plan = plan_view(self.index, self._spec, self._subset)
            if set(map(str, target_tensors)) != {t.name for t in plan.tensors}:
                raise ArtifactError("bind_into target tensors must cover the artifact selection", "FAILED_PRECONDITION")
            jobs, permutes = _b.view_target_jobs(plan, target_tensors, base)
        self._load(dev, dev_index, coll, world, rank, jobs, permutes, view_bytes, d_view=base,
                   target_ranges=ranges, options=options)
        return Binding(dict(target_tensors), self.data_multihash)


@dataclass
class Binding:
    """The filled targets of a bind_into call and the verified data multihash."""
    tensors: dict
    data_multihash: str | None

    def tensor_dict(self) -> dict:
        return self.tensors


def _root_of_multihash(mh: str) -> bytes:
    import base64
    if not mh.startswith("b"):
        raise ArtifactError(f"unsupported multibase prefix in {mh!r}", "INVALID_ARGUMENT")
    body = mh[1:].upper()
    raw = base64.b32decode(body + "=" * ((8 - len(body) % 8) % 8))
    if raw[:2] != b"\x12\x20" or len(raw) != 34:
        raise ArtifactError("descriptor data_multihash is not a sha2-256 multihash", "INVALID_ARGUMENT")
    return raw[2:]


def from_disk(path, *, key: str | None = None, verify_checksums: bool = True, show_progress=None,
              leaf_chunk_bytes: int | None = None) -> Artifact:
    """A lazy artifact over one safetensors file or a directory of them."""
    path = os.fspath(path)
    if not os.path.exists(path):
        raise ArtifactError(f"path does not exist: {path}", "NOT_FOUND")
    index = build_canonical_index(build_source_index(safetensors_files(path)))
    return Artifact(path, index, verify_checksums=verify_checksums, leaf_chunk_bytes=leaf_chunk_bytes, key=key)
