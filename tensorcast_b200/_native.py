"""ctypes binding of libtcx.so (the C ABI declared in include/tcx.h).

The library is built in-tree (tensorcast_b200/_lib/libtcx.so). There is no CPU
fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH, build_native

_lock = threading.Lock()
_lib = None

OK = 0
INVALID_ARGUMENT = 3
DEADLINE_EXCEEDED = 4
NOT_FOUND = 5
RESOURCE_EXHAUSTED = 8
FAILED_PRECONDITION = 9
UNIMPLEMENTED = 12
INTERNAL = 13
DATA_LOSS = 15

_CODE_NAMES = {0: "OK", 1: "CANCELLED", 2: "UNKNOWN", 3: "INVALID_ARGUMENT", 4: "DEADLINE_EXCEEDED",
               5: "NOT_FOUND", 8: "RESOURCE_EXHAUSTED", 9: "FAILED_PRECONDITION", 11: "OUT_OF_RANGE",
               12: "UNIMPLEMENTED", 13: "INTERNAL", 14: "UNAVAILABLE", 15: "DATA_LOSS"}


class TcxError(RuntimeError):
    """A libtcx call failed; ``code`` is the absl status code number."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_CODE_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class TcxInvalidArgument(TcxError, ValueError):
    pass


def _raise(code: int) -> None:
    msg = _lib.tcx_last_error().decode("utf-8", "replace")
    if code == INVALID_ARGUMENT:
        raise TcxInvalidArgument(code, msg)
    raise TcxError(code, msg)


_c = ctypes


class CopyJob(ctypes.Structure):
    _fields_ = [("src_off", _c.c_uint64), ("dst_off", _c.c_uint64), ("src_pitch", _c.c_uint64),
                ("dst_pitch", _c.c_uint64), ("row_bytes", _c.c_uint64), ("rows", _c.c_uint64)]


MAX_DIMS = 8


class PermuteJob(ctypes.Structure):
    _fields_ = [("src_off", _c.c_uint64), ("dst_off", _c.c_uint64), ("esize", _c.c_uint32), ("ndim", _c.c_uint32),
                ("shape", _c.c_int64 * MAX_DIMS), ("perm", _c.c_int32 * MAX_DIMS)]


class FileSegment(ctypes.Structure):
    _fields_ = [("path", _c.c_char_p), ("file_offset", _c.c_uint64), ("dst_offset", _c.c_uint64),
                ("length", _c.c_uint64)]


class LoadPlan(ctypes.Structure):
    _fields_ = [("total_bytes", _c.c_uint64), ("leaf_bytes", _c.c_uint64), ("stage_bounds", _c.c_void_p),
                ("jobs", _c.c_void_p), ("job_offsets", _c.c_void_p), ("permutes", _c.c_void_p),
                ("n_permutes", _c.c_uint64), ("view_bytes", _c.c_uint64), ("slab_bytes", _c.c_uint64),
                ("window_bytes", _c.c_uint64), ("flags", _c.c_uint64), ("target_ranges", _c.c_void_p),
                ("n_targets", _c.c_uint64), ("push_nccl_permille", _c.c_uint64)]


class ExchangePlan(ctypes.Structure):
    _fields_ = [("pack_jobs", _c.c_void_p), ("n_pack", _c.c_uint64), ("local_jobs", _c.c_void_p),
                ("n_local", _c.c_uint64), ("scatter_jobs", _c.c_void_p), ("n_scatter", _c.c_uint64),
                ("send_offsets", _c.c_void_p), ("recv_offsets", _c.c_void_p), ("recv_counts", _c.c_void_p),
                ("recv_view_off", _c.c_void_p), ("direct", _c.c_void_p), ("gaps", _c.c_void_p),
                ("n_gaps", _c.c_uint64)]


class LoadResult(ctypes.Structure):
    _fields_ = [("root", _c.c_uint8 * 32), ("multihash", _c.c_char * 64), ("leaves", _c.c_uint64),
                ("h2d_bytes", _c.c_uint64), ("peer_send_bytes", _c.c_uint64), ("peer_recv_bytes", _c.c_uint64),
                ("h2d_ms", _c.c_float), ("hash_ms", _c.c_float), ("exchange_ms", _c.c_float),
                ("total_ms", _c.c_float), ("view_multihash", _c.c_char * 64), ("view_leaf_bytes", _c.c_uint64),
                ("stage_read_ms", _c.c_float), ("transfer_ms", _c.c_float)]


class FileStage(ctypes.Structure):
    _fields_ = [("segments", _c.POINTER(FileSegment)), ("n_segments", _c.c_uint64), ("read_threads", _c.c_int),
                ("ring_slots", _c.c_int), ("slot_bytes", _c.c_uint64)]


# Every function exported by include/tcx.h with (restype, argtypes).
_SIGNATURES = {
    "tcx_last_error": (_c.c_char_p, []),
    "tcx_version": (_c.c_char_p, []),
    "tcx_kernel_launch_count": (_c.c_uint64, []),
    "tcx_sha256_compute_probe": (_c.c_int, [_c.c_uint32, _c.c_uint32, _c.c_void_p, _c.c_void_p]),
    "tcx_leaf_policy": (_c.c_int, [_c.c_uint64, _c.c_uint64, _c.POINTER(_c.c_uint64)]),
    "tcx_sha256_leaves": (_c.c_int, [_c.c_void_p, _c.c_uint64, _c.c_uint64, _c.c_void_p, _c.c_uint64, _c.c_void_p]),
    "tcx_sha256_leaves_pass": (_c.c_int, [_c.c_void_p, _c.c_uint64, _c.c_uint64, _c.c_uint64, _c.c_uint64,
                                          _c.c_void_p, _c.c_void_p, _c.c_uint64, _c.c_void_p]),
    "tcx_merkle_scratch_bytes": (_c.c_uint64, [_c.c_uint64]),
    "tcx_sha256_leaf_table": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_uint64, _c.c_int, _c.c_void_p,
                                         _c.c_void_p]),
    "tcx_merkle_segments_scratch_bytes": (_c.c_uint64, [_c.c_void_p, _c.c_uint64]),
    "tcx_merkle_roots_segmented": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_uint64, _c.c_void_p,
                                              _c.c_uint64, _c.c_void_p, _c.c_void_p]),
    "tcx_kv_gather": (_c.c_int, [_c.c_void_p, _c.c_uint32, _c.c_uint64, _c.c_uint32, _c.c_uint64, _c.c_void_p,
                                 _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_uint64, _c.c_uint64, _c.c_void_p,
                                 _c.c_uint64, _c.c_void_p, _c.c_void_p]),
    "tcx_merkle_root": (_c.c_int, [_c.c_void_p, _c.c_uint64, _c.c_void_p, _c.c_uint64, _c.c_void_p, _c.c_void_p]),
    "tcx_multihash_encode": (_c.c_int, [_c.c_void_p, _c.c_char_p, _c.c_size_t]),
    "tcx_multihash_from_gpu": (_c.c_int, [_c.c_void_p, _c.c_uint64, _c.c_int, _c.c_uint64, _c.c_char_p, _c.c_size_t]),
    "tcx_multihash_from_gpu_noalloc": (_c.c_int, [_c.c_void_p, _c.c_uint64, _c.c_int, _c.c_uint64, _c.c_char_p,
                                                  _c.c_size_t, _c.c_void_p]),
    "tcx_prewarm_device": (_c.c_int, [_c.c_int]),
    "tcx_prewarm_visible_devices": (_c.c_int, []),
    "tcx_copy_jobs_scratch_bytes": (_c.c_uint64, [_c.c_uint64]),
    "tcx_copy_jobs": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_uint64, _c.c_void_p, _c.c_uint64,
                                 _c.c_void_p]),
    "tcx_permute": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.POINTER(PermuteJob), _c.c_void_p]),
    "tcx_plan_exchange_capacity": (_c.c_uint64, [_c.POINTER(LoadPlan), _c.c_int]),
    "tcx_plan_exchange": (_c.c_int, [_c.POINTER(LoadPlan), _c.c_int, _c.c_int, _c.POINTER(ExchangePlan)]),
    "tcx_plan_push_split_capacity": (_c.c_uint64, [_c.POINTER(LoadPlan), _c.c_int]),
    "tcx_plan_push_split": (_c.c_int, [_c.POINTER(LoadPlan), _c.c_int, _c.c_int, _c.c_uint64, _c.c_void_p,
                                       _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_uint64]),
    "tcx_read_segments": (_c.c_int, [_c.POINTER(FileSegment), _c.c_uint64, _c.c_void_p, _c.c_int]),
    "tcx_read_segments_ex": (_c.c_int, [_c.POINTER(FileSegment), _c.c_uint64, _c.c_void_p, _c.c_int, _c.c_uint64]),
    "tcx_multihash_from_file_segments": (_c.c_int, [_c.POINTER(FileSegment), _c.c_uint64, _c.c_uint64, _c.c_uint64,
                                                    _c.c_int, _c.c_uint64, _c.c_int, _c.c_int, _c.c_uint64, _c.c_void_p,
                                                    _c.c_void_p, _c.c_void_p, _c.c_char_p, _c.c_uint64]),
    "tcx_file_hash_release": (_c.c_int, [_c.c_int]),
    "tcx_host_map_file": (_c.c_int, [_c.c_char_p, _c.c_uint64, _c.c_uint64, _c.c_int, _c.POINTER(_c.c_void_p),
                                     _c.POINTER(_c.c_void_p)]),
    "tcx_host_unmap_file": (_c.c_int, [_c.c_void_p]),
    "tcx_bind_device_cpus": (_c.c_int, [_c.c_int, _c.POINTER(_c.c_int)]),
    "tcx_group_unique_id": (_c.c_int, [_c.c_void_p]),
    "tcx_group_create": (_c.c_int, [_c.c_void_p, _c.c_int, _c.c_int, _c.c_int, _c.c_int64, _c.POINTER(_c.c_void_p)]),
    "tcx_group_join": (_c.c_int, [_c.c_char_p, _c.c_int, _c.c_int, _c.c_int, _c.c_int64, _c.POINTER(_c.c_void_p)]),
    "tcx_group_destroy": (_c.c_int, [_c.c_void_p]),
    "tcx_group_load": (_c.c_int, [_c.c_void_p, _c.POINTER(LoadPlan), _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                  _c.c_void_p, _c.POINTER(LoadResult), _c.c_void_p]),
    "tcx_group_load_files": (_c.c_int, [_c.c_void_p, _c.POINTER(LoadPlan), _c.POINTER(FileStage), _c.c_void_p,
                                        _c.c_void_p, _c.c_void_p, _c.POINTER(LoadResult), _c.c_void_p]),
}


def lib(build_if_missing: bool = True):
    """Load libtcx.so (building it first if it is absent and nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                if not build_if_missing:
                    raise RuntimeError(f"libtcx is not built ({LIB_PATH} missing)")
                build_native()
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise TcxError on failure."""
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != OK:
        _raise(rc)


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)
