"""CPU oracle for the realization hot path. TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` import
this module; the product package (``tensorcast_b200``) never does. It is the
checker, never the thing measured or shipped.

Hashing is delegated to ``oracle/_build/libtcx_oracle.so`` (built from
``oracle/tcx_oracle.c`` by ``oracle/Makefile``), a plain-C restatement of the
reference's CPU hashing path:

* ``leaf_digests``           -> source_hash.cc:19-61 + artifact_hash_cpu.cc:161-196
* ``tree_root``              -> artifact_hash_cpu.cc:198-233
* ``multihash``              -> artifact_hash_cpu.cc:33-64, 235-254
* ``determine_leaf_chunk_size`` -> artifact_hash_cpu.cc:269-303
* ``multihash_from_cpu_memory`` -> source_hash.cc:63-70
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libtcx_oracle.so")
_lib = None

DEFAULT_LEAF = 4 << 20


def build() -> str:
    """Compile the C oracle (gcc + libcrypto) if the shared object is missing or stale."""
    src = os.path.join(_HERE, "tcx_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        u8p = ctypes.c_void_p
        L.tcxo_sha256.argtypes = [u8p, ctypes.c_uint64, u8p]
        L.tcxo_sha256_bytes.argtypes = [u8p, ctypes.c_uint64, u8p]
        L.tcxo_sha256_openssl.argtypes = [u8p, ctypes.c_uint64, u8p]
        L.tcxo_sha256_openssl.restype = ctypes.c_int
        L.tcxo_leaf_count.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.tcxo_leaf_count.restype = ctypes.c_uint64
        L.tcxo_leaf_digests.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint64, u8p]
        L.tcxo_leaf_digests.restype = ctypes.c_int
        L.tcxo_leaf_digests_openssl.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint64, u8p, ctypes.c_int]
        L.tcxo_leaf_digests_openssl.restype = ctypes.c_int
        L.tcxo_tree_root.argtypes = [u8p, ctypes.c_uint64, u8p]
        L.tcxo_tree_root.restype = ctypes.c_int
        L.tcxo_multihash.argtypes = [u8p, ctypes.c_char_p, ctypes.c_uint64]
        L.tcxo_multihash.restype = ctypes.c_int
        L.tcxo_determine_leaf_chunk_size.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.tcxo_determine_leaf_chunk_size.restype = ctypes.c_uint64
        L.tcxo_multihash_from_cpu_memory.argtypes = [
            u8p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        L.tcxo_multihash_from_cpu_memory.restype = ctypes.c_int
        _lib = L
    return _lib


def _as_u8(buf) -> np.ndarray:
    a = np.ascontiguousarray(np.frombuffer(buf, dtype=np.uint8) if isinstance(buf, (bytes, bytearray, memoryview))
                             else np.asarray(buf).view(np.uint8).reshape(-1))
    return a


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data if a.size else 0


def sha256(data) -> bytes:
    """FIPS 180-4 SHA-256 (the empty message hashes normally here)."""
    a = _as_u8(data)
    out = np.zeros(32, np.uint8)
    lib().tcxo_sha256(_ptr(a), a.size, out.ctypes.data)
    return out.tobytes()


def sha256_bytes(data) -> bytes:
    """artifact_hash_cpu.cc:161-164 semantics: empty input -> 32 zero bytes."""
    a = _as_u8(data)
    out = np.zeros(32, np.uint8)
    lib().tcxo_sha256_bytes(_ptr(a), a.size, out.ctypes.data)
    return out.tobytes()


def leaf_count(total: int, leaf: int) -> int:
    return (total + leaf - 1) // leaf


def leaf_digests(data, leaf: int, openssl: bool = False, threads: int = 1) -> np.ndarray:
    """Digest of every leaf [i*L, min((i+1)*L, T)) as a uint8 array [n, 32]."""
    a = _as_u8(data)
    n = leaf_count(a.size, leaf)
    out = np.zeros((n, 32), np.uint8)
    if openssl:
        rc = lib().tcxo_leaf_digests_openssl(_ptr(a), a.size, leaf, out.ctypes.data, threads)
    else:
        rc = lib().tcxo_leaf_digests(_ptr(a), a.size, leaf, out.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle leaf_digests failed (status {rc})")
    return out


def tree_root(digests: np.ndarray) -> bytes:
    d = np.ascontiguousarray(digests, dtype=np.uint8).reshape(-1, 32)
    out = np.zeros(32, np.uint8)
    rc = lib().tcxo_tree_root(d.ctypes.data, d.shape[0], out.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle tree_root failed (status {rc})")
    return out.tobytes()


def multihash(digest: bytes) -> str:
    d = np.frombuffer(digest, np.uint8).copy()
    buf = ctypes.create_string_buffer(64)
    rc = lib().tcxo_multihash(d.ctypes.data, buf, 64)
    if rc != 0:
        raise ValueError("oracle multihash failed")
    return buf.value.decode("ascii")


def determine_leaf_chunk_size(total: int, requested: int = DEFAULT_LEAF) -> int:
    return int(lib().tcxo_determine_leaf_chunk_size(total, requested))


def multihash_from_cpu_memory(data, leaf: int = DEFAULT_LEAF, openssl: bool = False, threads: int = 1) -> str:
    """compute_data_multihash_from_cpu_memory: leaf size used as given (source_hash.cc:63-70)."""
    a = _as_u8(data)
    if a.size == 0 or leaf == 0:
        raise ValueError("total_size and leaf_chunk_bytes must be > 0")
    buf = ctypes.create_string_buffer(64)
    rc = lib().tcxo_multihash_from_cpu_memory(_ptr(a), a.size, leaf, buf, 64, int(openssl), threads)
    if rc != 0:
        raise ValueError(f"oracle multihash_from_cpu_memory failed (status {rc})")
    return buf.value.decode("ascii")


def multihash_gpu_semantics(data, leaf: int = DEFAULT_LEAF) -> str:
    """What compute_data_multihash_from_gpu returns for these bytes: the leaf size first goes
    through determine_leaf_chunk_size (artifact_hash_gpu.cc:931), then the same tree/multihash."""
    a = _as_u8(data)
    return multihash_from_cpu_memory(a, determine_leaf_chunk_size(a.size, leaf))
