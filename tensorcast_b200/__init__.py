"""tensorcast_b200: B200-native realization hot path for TensorCast.

GPU content hashing (per-leaf SHA-256, Merkle root, data multihash) and the
collective from-disk load with on-device view materialisation, behind a C ABI
(include/tcx.h) implemented by libtcx.so (hand-written sm_100a CUDA + C++).
"""
from ._native import TcxError, TcxInvalidArgument
from .hashing import (
    DEFAULT_LEAF_CHUNK_BYTES,
    compute_data_multihash_from_gpu,
    compute_data_multihash_from_gpu_memory,
    determine_leaf_chunk_size,
    merkle_root,
    multibase_multihash_sha256,
    prewarm_gpu_hash_for_device,
    prewarm_gpu_hash_for_visible_devices,
    sha256_leaves,
)

__all__ = [
    "TcxError",
    "TcxInvalidArgument",
    "DEFAULT_LEAF_CHUNK_BYTES",
    "compute_data_multihash_from_gpu",
    "compute_data_multihash_from_gpu_memory",
    "determine_leaf_chunk_size",
    "merkle_root",
    "multibase_multihash_sha256",
    "prewarm_gpu_hash_for_device",
    "prewarm_gpu_hash_for_visible_devices",
    "sha256_leaves",
]
