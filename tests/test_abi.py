"""CPU checks of the C ABI: the library loads, exports every symbol include/*.h declares,
and its host-only logic (leaf policy, multihash encoding, argument checks) agrees with
the oracle. No call here reaches a GPU."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

from oracle import oracle
from tensorcast_b200 import _native
from tensorcast_b200.hashing import determine_leaf_chunk_size, multibase_multihash_sha256

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(tcx_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = _native.lib()
    decl = declared_functions()
    assert decl, "no declarations found in include/"
    for name in decl:
        assert hasattr(L, name), f"{name} declared but not exported"
    assert set(decl) <= set(_native.exported_symbols()), "ctypes signature table is missing entries"


def test_version():
    assert b"sm_100a" in _native.lib().tcx_version()


@pytest.mark.parametrize("total", [1, 64, 65536, 1 << 20, (1 << 30) + 7, 16_060_522_496, 141_107_412_992,
                                   1 << 40])
@pytest.mark.parametrize("req", [0, 1, 63, 64, 100, 1000, 4096, 512 << 10, 2 << 20, 4 << 20, 64 << 20, 65 << 20])
def test_leaf_policy_matches_oracle(total, req):
    assert determine_leaf_chunk_size(total, req) == oracle.determine_leaf_chunk_size(total, req)


def test_multihash_encoding_matches_oracle():
    rng = np.random.default_rng(11)
    for _ in range(200):
        d = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
        assert multibase_multihash_sha256(d) == oracle.multihash(d)
    assert len(multibase_multihash_sha256(bytes(32))) == 56


def _mh(ptr, total, dev, leaf):
    buf = ctypes.create_string_buffer(64)
    rc = _native.lib().tcx_multihash_from_gpu(ptr, total, dev, leaf, buf, 64)
    return rc, _native.lib().tcx_last_error().decode()


def test_multihash_from_gpu_argument_checks():
    # artifact_hash_gpu.cc:907-927, checked before any device is touched
    assert _mh(None, 64, 0, 4 << 20) == (3, "GPU pointer is null")
    assert _mh(0x1000, 0, 0, 4 << 20) == (3, "Cannot hash empty GPU buffer")
    assert _mh(0x1000, (1 << 40) + 1, 0, 4 << 20) == (3, f"GPU buffer too large for hashing: {(1 << 40) + 1} bytes")
    assert _mh(0x1000, 64, 0, 0) == (3, "leaf_chunk_bytes must be > 0")
    assert _mh(0x1000, 64, 0, (64 << 20) + 1) == (3, f"Chunk size too large: {(64 << 20) + 1} (max: {64 << 20})")


def test_sha256_leaves_argument_checks():
    L = _native.lib()
    f = L.tcx_sha256_leaves
    assert f(None, 64, 64, 0x1000, 1, None) == 3
    assert f(0x1000, 64, 64, None, 1, None) == 3
    assert f(0x1000, 64, 64, 0x1001, 1, None) == 3  # unaligned digest buffer
    assert f(0x1000, 128, 64, 0x1000, 1, None) == 3  # capacity 1 < 2 leaves
    assert "2 needed" in L.tcx_last_error().decode()
    assert f(0x1000, 1 << 33, 1, 0x1000, 1 << 40, None) == 3  # leaf count >= 2^32
    with pytest.raises(_native.TcxInvalidArgument):
        _native.call("tcx_sha256_leaves", 0x1000, 0, 64, 0x1000, 1, None)


def test_merkle_argument_checks():
    L = _native.lib()
    assert L.tcx_merkle_root(0x1000, 0, None, 0, 0x2000, None) == 3
    assert L.tcx_merkle_root(0x1000, 5000, None, 0, 0x2000, None) == 3  # needs scratch
    assert L.tcx_merkle_scratch_bytes(5000) >= (2500 + 1250) * 32
