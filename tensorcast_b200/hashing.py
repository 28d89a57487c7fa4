"""Content hashing API: the Python face of the tcx_* hashing entry points.

Mirrors the reference's hashing surface (core/common/artifact_hash.h:16-48,
core/store/materialization/dataplane/metadata/source_hash.h:24-41):

* ``compute_data_multihash_from_gpu(gpu_ptr, total_size, device_id, leaf_chunk_bytes=4 MiB)``
* ``prewarm_gpu_hash_for_device(device_id)`` / ``prewarm_gpu_hash_for_visible_devices()``
* ``determine_leaf_chunk_size(total_size, requested)``
* ``multibase_multihash_sha256(digest)``

plus tensor-level helpers used by the loader: ``sha256_leaves`` (per-leaf digests
into a caller tensor, stream-ordered) and ``merkle_root``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native

DEFAULT_LEAF_CHUNK_BYTES = 4 << 20
MAX_LEAF_CHUNK_BYTES = 64 << 20


def _stream_handle(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ptr(x) -> int:
    return x.data_ptr() if isinstance(x, torch.Tensor) else int(x)


def determine_leaf_chunk_size(total_size: int, requested: int = DEFAULT_LEAF_CHUNK_BYTES) -> int:
    """determine_leaf_chunk_size (artifact_hash_cpu.cc:269-303)."""
    out = ctypes.c_uint64(0)
    _native.call("tcx_leaf_policy", total_size, requested, ctypes.byref(out))
    return int(out.value)


def leaf_count(total_size: int, leaf: int) -> int:
    return (total_size + leaf - 1) // leaf


def sha256_leaves(src: torch.Tensor, leaf_bytes: int, out: torch.Tensor | None = None, *, nbytes: int | None = None,
                  stream=None) -> torch.Tensor:
    """Digest of every leaf of the bytes of ``src`` (a CUDA tensor), as uint8 [n, 32].

    Stream-ordered on ``stream`` (default: the current stream); nothing is allocated
    by the library. ``nbytes`` hashes only the first nbytes bytes of ``src``."""
    if not src.is_cuda:
        raise ValueError("sha256_leaves needs a CUDA tensor")
    total = src.numel() * src.element_size() if nbytes is None else int(nbytes)
    n = leaf_count(total, leaf_bytes) if leaf_bytes > 0 else 0
    if out is None:
        out = torch.empty((max(n, 1), 32), dtype=torch.uint8, device=src.device)
    _native.call("tcx_sha256_leaves", src.data_ptr(), total, leaf_bytes, out.data_ptr(), out.numel() // 32,
                 _stream_handle(stream))
    return out[:n]


def merkle_root(digests: torch.Tensor, stream=None) -> torch.Tensor:
    """Merkle root (artifact_hash_cpu.cc:198-233) of uint8 [n, 32] device digests -> uint8 [32]."""
    d = digests.contiguous()
    n = d.numel() // 32
    L = _native.lib()
    scratch_bytes = int(L.tcx_merkle_scratch_bytes(n))
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device=d.device)
    root = torch.empty(32, dtype=torch.uint8, device=d.device)
    _native.call("tcx_merkle_root", d.data_ptr(), n, scratch.data_ptr(), scratch_bytes, root.data_ptr(),
                 _stream_handle(stream))
    return root


def multibase_multihash_sha256(digest: bytes) -> str:
    """to_multibase_multihash_sha256 (artifact_hash_cpu.cc:235-254)."""
    if len(digest) != 32:
        raise ValueError("SHA256 digest must be 32 bytes")
    buf = ctypes.create_string_buffer(64)
    src = (ctypes.c_uint8 * 32).from_buffer_copy(digest)
    _native.call("tcx_multihash_encode", ctypes.addressof(src), buf, 64)
    return buf.value.decode("ascii")


def compute_data_multihash_from_gpu(gpu_ptr, total_size: int, device_id: int,
                                    leaf_chunk_bytes: int = DEFAULT_LEAF_CHUNK_BYTES) -> str:
    """compute_data_multihash_from_gpu (artifact_hash_gpu.cc:903-957). Synchronous."""
    buf = ctypes.create_string_buffer(64)
    _native.call("tcx_multihash_from_gpu", _ptr(gpu_ptr), int(total_size), int(device_id), int(leaf_chunk_bytes),
                 buf, 64)
    return buf.value.decode("ascii")


def compute_data_multihash_from_gpu_memory(device_ptr, total_size: int, device_id: int,
                                           leaf_chunk_bytes: int = DEFAULT_LEAF_CHUNK_BYTES) -> str:
    """source_hash.cc:72-78: a thin wrapper of compute_data_multihash_from_gpu."""
    return compute_data_multihash_from_gpu(device_ptr, total_size, device_id, leaf_chunk_bytes)


def prewarm_gpu_hash_for_device(device_id: int) -> None:
    _native.call("tcx_prewarm_device", int(device_id))


def prewarm_gpu_hash_for_visible_devices() -> None:
    _native.call("tcx_prewarm_visible_devices")


def compute_canonical_leaf_digests(src: torch.Tensor, leaf_indices, chunk_bytes: int, *, nbytes: int | None = None,
                                   stream=None) -> list[bytes]:
    """Digests of the given leaves of a device buffer, in the order asked for.

    Mirrors compute_canonical_leaf_digests for GPU memory
    (core/store/materialization/dataplane/verification/verification_utils.cc:337-369, 851-868):
    leaf i is [i*chunk_bytes, (i+1)*chunk_bytes); indices whose leaf would run past the
    buffer are skipped (no entry). The reference copies each leaf to the host and hashes
    it there; here all leaves are hashed in one tcx_sha256_leaf_table launch and only the
    32-byte digests come back."""
    import numpy as np
    if chunk_bytes <= 0:
        raise ValueError("chunk_bytes must be > 0")
    total = src.numel() * src.element_size() if nbytes is None else int(nbytes)
    idx = [int(i) for i in leaf_indices if (int(i) + 1) * chunk_bytes <= total]
    if not idx:
        return []
    if chunk_bytes > 0xFFFFFFFF:
        raise ValueError("chunk_bytes must fit in 32 bits")
    offs = torch.from_numpy(np.asarray(idx, dtype=np.uint64).view(np.int64) * chunk_bytes).to(src.device)
    lens = torch.full((len(idx),), chunk_bytes, dtype=torch.int64).to(torch.int32).to(src.device)
    out = torch.empty((len(idx), 32), dtype=torch.uint8, device=src.device)
    aligned = src.data_ptr() % 16 == 0 and chunk_bytes % 16 == 0
    _native.call("tcx_sha256_leaf_table", src.data_ptr(), offs.data_ptr(), lens.data_ptr(), len(idx), int(aligned),
                 out.data_ptr(), _stream_handle(stream))
    return [bytes(r) for r in out.cpu().numpy()]
