"""Pins the CPU oracle (oracle/tcx_oracle.c) before anything is checked against it.

Anchors, in order of independence:
  * FIPS 180-4 / NIST example vectors for SHA-256;
  * Python hashlib (the same OpenSSL the reference calls, artifact_hash_cpu.cc:161-196);
  * the committed golden fixtures (tests/golden/make_golden.py: hashlib + a separate
    pure-Python tree/multihash restatement);
  * the reference's own golden vectors: the view id of
    core/store/materialization/dataplane/view/tests/view_identity_test.cc:51-68
    (pins SHA-256 + multihash encoding end to end), the KV byte-artifact payload
    digest of tests/python/test_kvcache_adapter.py:33-36, and the leaf-size column
    of examples/gpu_hash_benchmark.txt:5-18.
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def seeded(seed, size):
    return np.random.default_rng(seed).integers(0, 256, size=size, dtype=np.uint8)


NIST = [
    (b"", "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"),
    (b"abc", "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"),
    (b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq",
     "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1"),
    (b"a" * 1_000_000, "cdc76e5c9914fb9281a1c7e284d73e67f1809a48a497200e046d39ccc7112cd0"),
]


@pytest.mark.parametrize("msg,hexd", NIST)
def test_nist_vectors(msg, hexd):
    assert oracle.sha256(msg).hex() == hexd


def test_reference_empty_span_quirk():
    # artifact_hash_cpu.cc:161-164: sha256_bytes of an empty span is 32 zero bytes
    assert oracle.sha256_bytes(b"") == bytes(32)


def test_matches_hashlib_and_openssl_on_every_tail_length():
    buf = seeded(7, 4096)
    for n in list(range(0, 200)) + [1000, 4095, 4096]:
        want = hashlib.sha256(buf[:n].tobytes()).digest()
        assert oracle.sha256(buf[:n]) == want
    d1 = oracle.leaf_digests(buf, 100)
    d2 = oracle.leaf_digests(buf, 100, openssl=True)
    d3 = oracle.leaf_digests(buf, 100, openssl=True, threads=4)
    assert (d1 == d2).all() and (d1 == d3).all()


def test_kvcache_payload_digest_golden():
    # tests/python/test_kvcache_adapter.py:33-36
    assert oracle.sha256(b"abc123").hex() == "6ca13d52ca70c883e0f0bb101e425a89e8624de51db2d2392593af6a84118090"


def test_reference_view_id_golden_vector():
    """view_identity.cc:39-85 restated; the expected id is the reference's own golden value."""
    canonical_index_json = b'{"a":[0,16,[2,2],[2,1],"torch.float32",0],"b":[16,16,[2,2],[2,1],"torch.float32",0]}'
    index_mh = oracle.multihash(oracle.sha256_bytes(canonical_index_json)).encode()

    def s(name):
        return struct.pack("<I", len(name)) + name

    payload = struct.pack("<II", 1, 2)  # encoding version, tensor count (std::map order: a, b)
    payload += s(b"a") + struct.pack("<I", 1) + b"\x01" + struct.pack("<ii", 0, 1)  # transpose(0, 1)
    payload += s(b"b") + struct.pack("<I", 1) + b"\x00" + struct.pack("<iqQ", 1, 0, 1)  # narrow(dim 1, 0, 1)
    view_id = oracle.multihash(oracle.sha256_bytes(payload + index_mh))
    assert view_id == "bciqd3js2h75e5gw6cagg5kp3d6xc7laeqca263wrnmirudisjlwuwwa"


# (size, leaf chosen by the reference GPU policy) from examples/gpu_hash_benchmark.txt:5-18
BENCH_POLICY = [
    (65536, 524288), (524288, 524288), (1048576, 524288), (8388608, 524288), (33554432, 524288),
    (134217728, 524288), (536870912, 524288), (1073741824, 524288), (2147483648, 524288),
    (4294967296, 1048576), (8589934592, 2097152), (17179869184, 4194304), (34359738368, 4194304),
    (51539607552, 4194304),
]


@pytest.mark.parametrize("size,leaf", BENCH_POLICY)
def test_leaf_policy_matches_reference_benchmark_table(size, leaf):
    assert oracle.determine_leaf_chunk_size(size, 4 << 20) == leaf


def test_leaf_policy_non_default_requests():
    # Only the exact default request is adapted; others are clamped and 64-aligned.
    assert oracle.determine_leaf_chunk_size(1 << 30, 1000) == 960
    assert oracle.determine_leaf_chunk_size(1 << 30, 63) == 64
    assert oracle.determine_leaf_chunk_size(1 << 30, 0) == 4 << 20  # 0 != default: no halving
    assert oracle.determine_leaf_chunk_size(1 << 30, 128 << 20) == 64 << 20
    assert oracle.determine_leaf_chunk_size(1 << 30, 2 << 20) == 2 << 20
    # benchmark sizes: Llama-3-8B-shaped (16 060 522 496 B) and 70B-shaped artifacts
    assert oracle.determine_leaf_chunk_size(16_060_522_496, 4 << 20) == 2 << 20
    assert oracle.determine_leaf_chunk_size(141_107_412_992, 4 << 20) == 4 << 20


def test_small_golden_cases():
    with open(os.path.join(GOLDEN, "hash_golden.json")) as f:
        g = json.load(f)
    for c in g["small"]:
        buf = seeded(c["seed"], c["size"])
        d = oracle.leaf_digests(buf, c["leaf"])
        assert d.shape[0] == c["n_leaves"]
        assert d[0].tobytes().hex() == c["first_leaf"]
        assert d[-1].tobytes().hex() == c["last_leaf"]
        root = oracle.tree_root(d)
        assert root.hex() == c["root"]
        assert oracle.multihash(root) == c["multihash"]
        assert oracle.multihash_from_cpu_memory(buf, c["leaf"]) == c["multihash"]


def test_c1_golden_1gib():
    """The 1 GiB hash-parity case: seed-0 bytes, 4 MiB leaves (256 digests) through the CPU path,
    and the reference GPU policy's 512 KiB leaves (2048 digests)."""
    with open(os.path.join(GOLDEN, "hash_golden.json")) as f:
        g = json.load(f)
    buf = seeded(0, 1 << 30)
    for c in g["c1"]:
        want = np.fromfile(os.path.join(GOLDEN, c["digests_file"]), dtype=np.uint8).reshape(-1, 32)
        d = oracle.leaf_digests(buf, c["leaf"], openssl=True, threads=8)
        assert d.shape == want.shape and (d == want).all()
        assert oracle.tree_root(d).hex() == c["root"]
    # the C restatement of SHA-256 itself on a subset of leaves
    c = g["c1"][0]
    want = np.fromfile(os.path.join(GOLDEN, c["digests_file"]), dtype=np.uint8).reshape(-1, 32)
    sub = buf[: 8 * c["leaf"]]
    assert (oracle.leaf_digests(sub, c["leaf"]) == want[:8]).all()
    assert oracle.multihash_from_cpu_memory(buf, 4 << 20, openssl=True, threads=8) == c["multihash"]


def test_tree_odd_promotion():
    d = seeded(3, 5 * 32).reshape(5, 32)
    h = lambda a, b: hashlib.sha256(a + b).digest()  # noqa: E731
    l = [r.tobytes() for r in d]
    want = h(h(h(l[0], l[1]), h(l[2], l[3])), l[4])
    assert oracle.tree_root(d) == want
    assert oracle.tree_root(d[:1]) == l[0]
