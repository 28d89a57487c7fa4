"""Data multihash of an artifact directory on disk, hashed on the GPU.

Mirrors ``compute_data_multihash_from_disk_dir(artifact_dir, progress_cb)``
(core/store/materialization/dataplane/metadata/disk_dir_hash.cc:47-104), which the
reference runs on one CPU core. The directory's bytes form one stream, resolved here
with the reference's rules (disk_artifact_context.cc:380-550):

* ``tensor.data_<n>`` partitions in numeric order (ties by file name), else a single
  ``tensor.data``, else every ``*.safetensors`` file in file-name order (their payloads,
  after each header); ``artifact_descriptor.json`` and ``tensor_index.*`` are metadata;
* partitions with a ``tensor_index.json``: the logical total is max(offset + size) over
  its entries (index_reader.cc:24-45); one partition is cut to it, several have the last
  one cut (disk_artifact_context.cc:293-366);
* safetensors: the logical total is the canonical index total of the headers (sorted
  names, 8-byte aligned) or of ``tensor_index.json`` when present, and it may not exceed
  the payload bytes (disk_dir_hash.cc:91-95).

The stream is cut into 4 MiB leaves as given (the CPU path applies no adaptive
policy) and hashed by ``tcx_multihash_from_file_segments``: the leaves in waves of up to
4096, read in 256 KiB pieces by reader threads that copy each few leaves' pieces to the
device at once, every chain of a wave advanced by one pass of the SHA-256 leaf kernel per
slab, Merkle root on the device (short leaves, or ``direct_io``, in whole-leaf groups
through pinned slots). The result equals the reference's CPU result bit for bit.
"""
from __future__ import annotations

import ctypes
import json
import os
import re

from . import _native
from .artifact import build_canonical_index, build_source_index, parse_safetensors_header

HASH_LEAF_CHUNK_BYTES = 4 << 20  # kHashLeafChunkBytes
_PARTITION = re.compile(r"^tensor\.data_([0-9]+)$")
_PROGRESS = ctypes.CFUNCTYPE(None, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p)


class DiskHashError(RuntimeError):
    def __init__(self, message: str, status_code: str):
        super().__init__(message)
        self.status_code = status_code


def _index_total(path: str) -> int:
    """compute_total_size_bytes of a tensor_index.json (index_reader.cc:24-45)."""
    with open(path, "rb") as f:
        idx = json.load(f)
    total = 0
    for arr in idx.values():
        if isinstance(arr, list) and len(arr) >= 2:
            total = max(total, int(arr[0]) + int(arr[1]))
    return total


def disk_dir_layout(artifact_dir) -> tuple[list[tuple[str, int, int, int]], int, str]:
    """(segments, total, kind): segments (path, file_offset, stream_offset, length) tile
    the hashed stream [0, total); kind is "partitions" or "safetensors"."""
    d = os.fspath(artifact_dir)
    if not os.path.exists(d):
        raise DiskHashError(f"Artifact directory not found: {d}", "NOT_FOUND")
    if not os.path.isdir(d):
        raise DiskHashError(f"Expected artifact path to be a directory: {d}", "FAILED_PRECONDITION")
    multipart, single, safetensors = [], None, []
    has_json = has_cbor = False
    for name in os.listdir(d):
        p = os.path.join(d, name)
        if not os.path.isfile(p):
            continue
        if name == "artifact_descriptor.json":
            continue
        if name == "tensor_index.json":
            has_json = True
            continue
        if name == "tensor_index.cbor":
            has_cbor = True
            continue
        if name == "tensor.data":
            single = p
            continue
        m = _PARTITION.match(name)
        if m:
            multipart.append((int(m.group(1)), name, p))
            continue
        if name.endswith(".safetensors"):
            safetensors.append(p)
    index_json = os.path.join(d, "tensor_index.json")
    if multipart or single:
        if multipart:
            paths = [p for _, _, p in sorted(multipart)]
        else:
            paths = [single]
        sizes = [os.path.getsize(p) for p in paths]
        physical = sum(sizes)
        if has_json or has_cbor:
            if not has_json:
                raise DiskHashError("tensor_index.cbor is not read by this build; provide tensor_index.json",
                                    "UNIMPLEMENTED")
            logical = _index_total(index_json)
            if logical > 0:
                if logical > physical:
                    raise DiskHashError(f"disk artifact logical total size {logical} exceeds physical partition "
                                        f"bytes {physical} for artifact {d}", "FAILED_PRECONDITION")
                before_last = physical - sizes[-1]
                if logical < before_last:
                    raise DiskHashError(f"disk artifact logical total size {logical} falls before the final "
                                        f"partition under numeric concatenation for {d}", "FAILED_PRECONDITION")
                sizes[-1] = logical - before_last
        segs, off = [], 0
        for p, n in zip(paths, sizes):
            if n:
                segs.append((p, 0, off, n))
            off += n
        return segs, off, "partitions"
    if not safetensors:
        raise DiskHashError(f"No replica partition files found in: {d} (also no .safetensors)", "NOT_FOUND")
    safetensors.sort(key=lambda p: os.path.basename(p).encode("utf-8"))
    segs, off = [], 0
    for p in safetensors:
        start, _ = parse_safetensors_header(p)
        n = os.path.getsize(p) - start
        if n:
            segs.append((p, start, off, n))
        off += n
    physical = off
    if has_json:
        logical = _index_total(index_json)
    else:
        logical = build_canonical_index(build_source_index(safetensors)).total_bytes
    total = logical if logical > 0 else physical
    if total > physical:
        raise DiskHashError("tensor_index.json total size exceeds safetensors payload bytes", "FAILED_PRECONDITION")
    out = []
    for p, foff, soff, n in segs:
        if soff >= total:
            break
        out.append((p, foff, soff, min(n, total - soff)))
    return out, total, "safetensors"


def compute_data_multihash_from_segments(segments, total: int, *, device_id: int = 0,
                                         leaf_chunk_bytes: int = HASH_LEAF_CHUNK_BYTES, progress_cb=None,
                                         group_bytes: int = 0, depth: int = 0, read_threads: int = 0,
                                         direct_io: bool = False) -> str:
    """Multihash of the byte stream given as (path, file_offset, stream_offset, length) segments;
    direct_io reads past the page cache (O_DIRECT windows, buffered where refused)."""
    arr = (_native.FileSegment * max(len(segments), 1))()
    keep = []
    for i, (path, foff, soff, ln) in enumerate(segments):
        p = os.fsencode(path)
        keep.append(p)
        arr[i] = _native.FileSegment(p, int(foff), int(soff), int(ln))
    cb = None
    if progress_cb is not None:
        cb = _PROGRESS(lambda done, tot, _ctx: progress_cb(int(done), int(tot)))
    root = (ctypes.c_uint8 * 32)()
    out = ctypes.create_string_buffer(64)
    try:
        _native.call("tcx_multihash_from_file_segments", arr, len(segments), int(total), int(leaf_chunk_bytes),
                     int(device_id), int(group_bytes), int(depth), int(read_threads), 1 if direct_io else 0,
                     ctypes.cast(cb, ctypes.c_void_p) if cb is not None else None, None, root, out, 64)
    except _native.TcxError as e:
        code = {3: "INVALID_ARGUMENT", 5: "NOT_FOUND", 12: "UNIMPLEMENTED", 15: "DATA_LOSS"}.get(e.code, "INTERNAL")
        raise DiskHashError(str(e), code) from e
    return out.value.decode("ascii")


def compute_data_multihash_from_disk_dir(artifact_dir, progress_cb=None, *, device_id: int = 0,
                                         group_bytes: int = 0, depth: int = 0, read_threads: int = 0,
                                         direct_io: bool = False) -> str:
    """compute_data_multihash_from_disk_dir (disk_dir_hash.cc:47-104), hashed on the GPU.

    progress_cb(processed_bytes, total_bytes) is called with (0, total) first and then as
    groups of leaves finish, as the reference's leaf progress adapter does (:29-45)."""
    segs, total, _ = disk_dir_layout(artifact_dir)
    return compute_data_multihash_from_segments(segs, total, device_id=device_id, progress_cb=progress_cb,
                                                group_bytes=group_bytes, depth=depth, read_threads=read_threads,
                                                direct_io=direct_io)


def release_buffers(device_id: int = -1) -> None:
    """Frees the pinned and device buffers kept between disk hashes (-1: all devices)."""
    _native.call("tcx_file_hash_release", int(device_id))
