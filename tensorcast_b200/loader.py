"""Collective load: Python face of tcx_group_* (include/tcx.h).

A ``Group`` is one rank of an N-rank load: one process per GPU (``from_torch_distributed``)
or one thread per GPU in one process (``join``, the reference daemon's model). Ranks agree on a
leaf-aligned split of the canonical byte space (``stage_bounds``); each stages its
part, hashes the leaves it staged, and the native engine exchanges exactly the bytes
each peer's view needs (NCCL grouped send/recv). All ranks end with their view and
the Merkle root of the whole artifact.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import _native
from .views import JOB_DTYPE, permute_array


VIEW_HASH = 1  # TCX_LOAD_VIEW_HASH
PEER_PUSH = 2  # TCX_LOAD_PEER_PUSH
TARGETS = 4  # TCX_LOAD_TARGETS
ALLGATHER = 8  # TCX_LOAD_ALLGATHER


def stage_bounds(total: int, leaf: int, world: int) -> list[int]:
    """Leaf-aligned split of [0, total) into `world` contiguous ranges (rank r stages
    leaves [r*n//world, (r+1)*n//world))."""
    n = (total + leaf - 1) // leaf
    b = [min(total, ((r * n) // world) * leaf) for r in range(world)] + [total]
    b[0] = 0
    return b


def _jobs_concat(rank_jobs: list) -> tuple[np.ndarray, np.ndarray]:
    arrs = [np.ascontiguousarray(j, dtype=JOB_DTYPE) for j in rank_jobs]
    offs = np.zeros(len(arrs) + 1, np.uint64)
    for i, a in enumerate(arrs):
        offs[i + 1] = offs[i] + a.size
    jobs = np.concatenate(arrs) if arrs and offs[-1] > 0 else np.zeros(1, JOB_DTYPE)
    return jobs, offs


class _Plan:
    """A tcx_load_plan with its arrays kept alive."""

    def __init__(self, total, leaf, bounds, rank_jobs, permutes=(), view_bytes=0, slab_bytes=0, window_bytes=0,
                 flags=0, target_ranges=None, push_nccl_share=0.0):
        self.bounds = np.ascontiguousarray(bounds, dtype=np.uint64)
        self.targets = None if target_ranges is None else np.ascontiguousarray(target_ranges, dtype=np.uint64).ravel()
        self.jobs, self.job_offsets = _jobs_concat(rank_jobs)
        self.perms = permute_array(list(permutes)) if permutes else None
        self.c = _native.LoadPlan(
            total_bytes=int(total), leaf_bytes=int(leaf), stage_bounds=self.bounds.ctypes.data,
            jobs=self.jobs.ctypes.data, job_offsets=self.job_offsets.ctypes.data,
            permutes=self.perms.ctypes.data if self.perms is not None else None,
            n_permutes=0 if self.perms is None else len(self.perms), view_bytes=int(view_bytes),
            slab_bytes=int(slab_bytes), window_bytes=int(window_bytes), flags=int(flags),
            target_ranges=None if self.targets is None else self.targets.ctypes.data,
            n_targets=0 if self.targets is None else len(self.targets) // 2,
            push_nccl_permille=int(round(max(0.0, min(1.0, push_nccl_share)) * 1000)))


def plan_exchange(total, leaf, bounds, rank_jobs, rank, view_bytes=0) -> dict:
    """Host-only exchange schedule of `rank` (tcx_plan_exchange), as numpy arrays."""
    world = len(bounds) - 1
    plan = _Plan(total, leaf, bounds, rank_jobs, view_bytes=view_bytes)
    L = _native.lib()
    cap = int(L.tcx_plan_exchange_capacity(ctypes.byref(plan.c), world))
    out = {k: np.zeros(cap, JOB_DTYPE) for k in ("pack", "local", "scatter")}
    for k, n in (("send_offsets", world + 1), ("recv_offsets", world + 1), ("recv_counts", world),
                 ("recv_view_off", world)):
        out[k] = np.zeros(n, np.uint64)
    out["direct"] = np.zeros(world, np.uint8)
    out["gaps"] = np.zeros(2 * cap, np.uint64)
    xp = _native.ExchangePlan(out["pack"].ctypes.data, 0, out["local"].ctypes.data, 0, out["scatter"].ctypes.data, 0,
                              out["send_offsets"].ctypes.data, out["recv_offsets"].ctypes.data,
                              out["recv_counts"].ctypes.data, out["recv_view_off"].ctypes.data,
                              out["direct"].ctypes.data, out["gaps"].ctypes.data, 0)
    _native.call("tcx_plan_exchange", ctypes.byref(plan.c), world, rank, ctypes.byref(xp))
    out["pack"] = out["pack"][: xp.n_pack].copy()
    out["local"] = out["local"][: xp.n_local].copy()
    out["scatter"] = out["scatter"][: xp.n_scatter].copy()
    out["gaps"] = out["gaps"][: 2 * xp.n_gaps].reshape(-1, 2).copy()
    return out


def plan_push_split(total, leaf, bounds, rank_jobs, rank, nccl_share: float) -> dict:
    """Host-only split of a push exchange (tcx_plan_push_split): {"nccl": every receiver's
    NCCL pieces (list of job arrays), "ce": this rank's copy-engine pieces per receiver}."""
    world = len(bounds) - 1
    plan = _Plan(total, leaf, bounds, rank_jobs)
    L = _native.lib()
    cap = int(L.tcx_plan_push_split_capacity(ctypes.byref(plan.c), world))
    nj, ce = np.zeros(cap, JOB_DTYPE), np.zeros(cap, JOB_DTYPE)
    noff, coff = np.zeros(world + 1, np.uint64), np.zeros(world + 1, np.uint64)
    _native.call("tcx_plan_push_split", ctypes.byref(plan.c), world, rank, int(round(nccl_share * 1000)),
                 nj.ctypes.data, noff.ctypes.data, ce.ctypes.data, coff.ctypes.data, cap)
    return {"nccl": [nj[int(noff[r]):int(noff[r + 1])].copy() for r in range(world)],
            "ce": [ce[int(coff[r]):int(coff[r + 1])].copy() for r in range(world)]}


READ_DIRECT = 1  # TCX_READ_DIRECT


def read_segments(segments, dst_ptr: int, threads: int = 8, direct: bool = False) -> None:
    """Parallel preads of (path, file_offset, dst_offset, length) segments into dst_ptr, in
    source order; direct: O_DIRECT through aligned windows (cold reads past the page cache)."""
    if not segments:
        return
    arr = (_native.FileSegment * len(segments))()
    keep = []
    for i, (path, foff, doff, ln) in enumerate(segments):
        p = os.fsencode(path)
        keep.append(p)
        arr[i] = _native.FileSegment(p, foff, doff, ln)
    _native.call("tcx_read_segments_ex", arr, len(segments), dst_ptr, int(threads), READ_DIRECT if direct else 0)


def bind_device_cpus(device: int) -> int:
    """Binds the calling thread (and threads it starts later) to the CPUs local to `device`;
    returns how many. Call before allocating pinned staging buffers."""
    n = ctypes.c_int(0)
    _native.call("tcx_bind_device_cpus", int(device), ctypes.byref(n))
    return n.value


class FileMapping:
    """A read-only mapping of a file range, page-locked for direct H2D (tcx_host_map_file)."""

    def __init__(self, path: str, offset: int, length: int, register: bool = True):
        self._h = ctypes.c_void_p()
        ptr = ctypes.c_void_p()
        _native.call("tcx_host_map_file", os.fsencode(path), int(offset), int(length), int(register),
                     ctypes.byref(ptr), ctypes.byref(self._h))
        self.ptr, self.length = int(ptr.value), int(length)

    def data_ptr(self) -> int:
        return self.ptr

    def close(self) -> None:
        if self._h:
            _native.call("tcx_host_unmap_file", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Group:
    """One rank of a collective load (tcx_group)."""

    def __init__(self, world: int = 1, rank: int = 0, device: int = 0, unique_id: bytes | None = None,
                 timeout_ms: int = 120_000):
        self.world, self.rank, self.device = world, rank, device
        self._h = ctypes.c_void_p()
        uid = None
        if world > 1:
            if unique_id is None or len(unique_id) != 128:
                raise ValueError("a 128-byte NCCL unique id is required for world > 1")
            uid = ctypes.create_string_buffer(bytes(unique_id), 128)
        _native.call("tcx_group_create", uid, world, rank, device, int(timeout_ms), ctypes.byref(self._h))

    @classmethod
    def join(cls, group_id: str, world: int, rank: int, device: int, timeout_ms: int = 120_000) -> "Group":
        """Joins rank `rank` of group `group_id` from a thread of this process (tcx_group_join):
        the rank threads of one process find each other by the id, no launcher or store needed."""
        g = cls.__new__(cls)
        g.world, g.rank, g.device = world, rank, device
        g._h = ctypes.c_void_p()
        _native.call("tcx_group_join", str(group_id).encode(), int(world), int(rank), int(device), int(timeout_ms),
                     ctypes.byref(g._h))
        return g

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _native.call("tcx_group_unique_id", buf)
        return buf.raw

    @classmethod
    def from_torch_distributed(cls, device: int, timeout_ms: int = 120_000) -> "Group":
        """Builds the group over the ranks of the default torch.distributed process group
        (the unique id travels through it)."""
        import torch.distributed as dist
        world, rank = dist.get_world_size(), dist.get_rank()
        obj = [cls.unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(obj, src=0)
        return cls(world, rank, device, obj[0] if world > 1 else None, timeout_ms)

    def load(self, total, leaf, bounds, rank_jobs, *, d_stage, d_view, h_stage=None, files=None, permutes=(),
             view_bytes=None, expected_root: bytes | None = None, slab_bytes: int = 0, window_bytes: int = 0,
             view_hash: bool = False, peer_push: bool = False, target_ranges=None, all_gather: bool = False,
             read_threads: int = 0, ring_slots: int = 0, slot_bytes: int = 0, push_nccl_share: float = 0.0) -> dict:
        """Runs one load; returns the result fields as a dict. h_stage None and files None:
        device-resident (d_stage already holds this rank's range).

        files: this rank's staged range as (path, file_offset, stage_offset, length) segments
        (stage offsets relative to bounds[rank]; uncovered bytes are zero): the range is read
        inside the call by the group's reader threads, overlapped with the copies to the device
        and the hash (tcx_group_load_files). Leaves of at least 128 KiB are read in pieces (up to 256 KiB
        of a few consecutive leaves per 4 MiB copy, each reader with two pinned buffers); shorter
        leaves in slabs through a ring of ring_slots pinned slots of about slot_bytes each.

        peer_push: exchange by copying into the peers' views over NVLink (d_view must be a
        cudaMalloc allocation, e.g. a torch CUDA tensor); push_nccl_share (0..1): that share of
        every peer pair's bytes goes over NCCL send/recv beside the copy engines; all_gather: a windowed
        all-gather of every rank's staged bytes instead (every rank sees every byte); else the
        NCCL send/recv shard exchange.
        target_ranges: (offset, length) pairs of separate target tensors (TCX_LOAD_TARGETS):
        d_view is then the lowest target's address and view offsets are relative to it."""
        if view_bytes is None:
            view_bytes = d_view.numel() * d_view.element_size() if isinstance(d_view, torch.Tensor) else 0
        plan = _Plan(total, leaf, bounds, rank_jobs, permutes, view_bytes, slab_bytes, window_bytes,
                     flags=(VIEW_HASH if view_hash else 0) | (PEER_PUSH if peer_push else 0) |
                     (TARGETS if target_ranges is not None else 0) | (ALLGATHER if all_gather else 0),
                     target_ranges=target_ranges, push_nccl_share=push_nccl_share)
        res = _native.LoadResult()
        exp = None
        if expected_root is not None:
            if len(expected_root) != 32:
                raise ValueError("expected_root must be 32 bytes")
            exp = ctypes.create_string_buffer(bytes(expected_root), 32)
        ptr = lambda x: None if x is None else (x.data_ptr() if hasattr(x, "data_ptr") else int(x))  # noqa: E731
        stream = torch.cuda.current_stream().cuda_stream
        if files is not None:
            if h_stage is not None:
                raise ValueError("give either h_stage or files")
            segs = (_native.FileSegment * max(len(files), 1))()
            keep = []
            for i, (path, foff, doff, ln) in enumerate(files):
                p = os.fsencode(path)
                keep.append(p)
                segs[i] = _native.FileSegment(p, int(foff), int(doff), int(ln))
            fs = _native.FileStage(segs, len(files), int(read_threads), int(ring_slots), int(slot_bytes))
            _native.call("tcx_group_load_files", self._h, ctypes.byref(plan.c), ctypes.byref(fs), ptr(d_stage),
                         ptr(d_view), exp, ctypes.byref(res), stream)
        else:
            _native.call("tcx_group_load", self._h, ctypes.byref(plan.c), ptr(h_stage), ptr(d_stage), ptr(d_view),
                         exp, ctypes.byref(res), stream)
        return {"root": bytes(res.root), "multihash": res.multihash.decode(), "leaves": res.leaves,
                "h2d_bytes": res.h2d_bytes, "peer_send_bytes": res.peer_send_bytes,
                "peer_recv_bytes": res.peer_recv_bytes, "h2d_ms": res.h2d_ms, "hash_ms": res.hash_ms,
                "exchange_ms": res.exchange_ms, "total_ms": res.total_ms,
                "view_multihash": res.view_multihash.decode(), "view_leaf_bytes": res.view_leaf_bytes,
                "stage_read_ms": res.stage_read_ms, "transfer_ms": res.transfer_ms}

    def close(self) -> None:
        if self._h:
            _native.lib().tcx_group_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
