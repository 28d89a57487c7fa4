"""GPU parity of the content-hashing path against the pinned CPU oracle.

Bit-exact: every leaf digest, Merkle root and multihash must equal the oracle's
(and the committed golden fixtures) on the same seeded bytes."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle
import tensorcast_b200 as tcx
from tensorcast_b200 import _native

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def seeded(seed, size):
    return np.random.default_rng(seed).integers(0, 256, size=size, dtype=np.uint8)


def to_dev(a: np.ndarray, offset: int = 0) -> torch.Tensor:
    """Device copy of a at byte offset `offset` inside a larger allocation."""
    buf = torch.zeros(a.size + offset + 64, dtype=torch.uint8, device="cuda")
    buf[offset:offset + a.size] = torch.from_numpy(a).cuda()
    torch.cuda.synchronize()
    return buf[offset:offset + a.size]


def test_small_golden_cases_on_gpu(cuda_device):
    with open(os.path.join(GOLDEN, "hash_golden.json")) as f:
        g = json.load(f)
    for c in g["small"]:
        a = seeded(c["seed"], c["size"])
        d = tcx.sha256_leaves(to_dev(a), c["leaf"]).cpu().numpy()
        assert d.shape[0] == c["n_leaves"]
        assert (d == oracle.leaf_digests(a, c["leaf"])).all()
        assert d[0].tobytes().hex() == c["first_leaf"] and d[-1].tobytes().hex() == c["last_leaf"]
        root = tcx.merkle_root(torch.from_numpy(d).cuda()).cpu().numpy().tobytes()
        assert root.hex() == c["root"]


@pytest.mark.parametrize("offset", [0, 1, 2, 3, 4, 5, 8, 13, 16])
@pytest.mark.parametrize("leaf", [64, 100, 1000, 4096, 4097, 65536 + 3])
def test_alignment_and_ragged_leaves(cuda_device, offset, leaf):
    a = seeded(offset * 1000 + leaf, 3 * leaf + 57)
    d = tcx.sha256_leaves(to_dev(a, offset), leaf).cpu().numpy()
    assert (d == oracle.leaf_digests(a, leaf)).all()


@pytest.mark.parametrize("size", [1, 55, 56, 57, 63, 64, 65, 119, 120, 128, 4096 + 55])
def test_single_leaf_tail_lengths(cuda_device, size):
    a = seeded(size, size)
    d = tcx.sha256_leaves(to_dev(a), 4 << 20).cpu().numpy()
    assert d.shape == (1, 32) and d[0].tobytes() == oracle.sha256(a)


def test_reference_gpu_vs_cpu_64_bytes(cuda_device):
    """verification_utils_test.cc:123-150: 64 bytes of 0xAA ^ i hash equal on GPU and CPU."""
    host = np.array([0xAA ^ i for i in range(64)], dtype=np.uint8)
    dev = to_dev(host)
    got = tcx.compute_data_multihash_from_gpu(dev.data_ptr(), 64, 0)
    assert got == oracle.multihash_from_cpu_memory(host, 4 << 20)


def test_c1_1gib_golden_digests(cuda_device):
    """The 1 GiB hash-parity case on the GPU: 256 x 4 MiB and 2048 x 512 KiB leaves of 1 GiB seed-0 bytes."""
    with open(os.path.join(GOLDEN, "hash_golden.json")) as f:
        g = json.load(f)
    dev = to_dev(seeded(0, 1 << 30))
    for c in g["c1"]:
        want = np.fromfile(os.path.join(GOLDEN, c["digests_file"]), dtype=np.uint8).reshape(-1, 32)
        d = tcx.sha256_leaves(dev, c["leaf"])
        assert (d.cpu().numpy() == want).all()
        assert tcx.merkle_root(d).cpu().numpy().tobytes().hex() == c["root"]
    # The GPU entry point adapts a request of exactly 4 MiB (the default) to 512 KiB leaves for
    # 1 GiB (artifact_hash_cpu.cc:281-296), so both requests give the 512 KiB multihash.
    for req in (4 << 20, 512 << 10):
        assert tcx.compute_data_multihash_from_gpu(dev.data_ptr(), 1 << 30, 0, req) == g["c1"][1]["multihash"]
    assert tcx.compute_data_multihash_from_gpu(dev.data_ptr(), 1 << 30, 0) == g["c1"][1]["multihash"]


@pytest.mark.parametrize("size", [64, 65536, 1 << 20, (8 << 20) + 17, (32 << 20) + 1000, 3 << 28])
def test_multihash_from_gpu_policy_matches_oracle(cuda_device, size):
    a = seeded(size % 9973, size)
    dev = to_dev(a)
    assert tcx.compute_data_multihash_from_gpu(dev.data_ptr(), size, 0) == oracle.multihash_gpu_semantics(a)
    assert tcx.compute_data_multihash_from_gpu(dev.data_ptr(), size, 0, 1 << 20) == \
        oracle.multihash_from_cpu_memory(a, 1 << 20, openssl=True, threads=8)


@pytest.mark.parametrize("n", [1, 2, 3, 5, 255, 2047, 2048, 2049, 4097, 7659, 33643])
def test_merkle_root_matches_oracle(cuda_device, n):
    d = seeded(n, n * 32).reshape(n, 32)
    root = tcx.merkle_root(torch.from_numpy(d).cuda()).cpu().numpy().tobytes()
    assert root == oracle.tree_root(d)


def test_device_errors_are_reported(cuda_device):
    dev = to_dev(seeded(1, 4096))
    with pytest.raises(tcx.TcxInvalidArgument, match="Chunk size too large"):
        tcx.compute_data_multihash_from_gpu(dev.data_ptr(), 4096, 0, 128 << 20)
    with pytest.raises(tcx.TcxError, match="Failed to set CUDA device"):
        tcx.compute_data_multihash_from_gpu(dev.data_ptr(), 4096, 4096)
    tcx.prewarm_gpu_hash_for_device(0)
    tcx.prewarm_gpu_hash_for_visible_devices()
    with pytest.raises(tcx.TcxInvalidArgument):
        tcx.prewarm_gpu_hash_for_device(torch.cuda.device_count())


def test_leaf_digests_are_stream_ordered(cuda_device):
    a = seeded(5, 1 << 24)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        dev = torch.from_numpy(a).to("cuda", non_blocking=False)
        d = tcx.sha256_leaves(dev, 1 << 16, stream=s)
    s.synchronize()
    assert (d.cpu().numpy() == oracle.leaf_digests(a, 1 << 16, openssl=True, threads=8)).all()


def test_canonical_leaf_digests_skip_partial_leaves(cuda_device):
    """verification_utils.cc:337-369: digests of the requested full leaves, in request order."""
    a = seeded(77, 10 * 4096 + 100)
    got = tcx.hashing.compute_canonical_leaf_digests(to_dev(a), [3, 0, 9, 10, 11], 4096)
    want = oracle.leaf_digests(a, 4096)
    assert got == [want[3].tobytes(), want[0].tobytes(), want[9].tobytes()]  # 10 is partial, 11 beyond


@pytest.mark.parametrize("layout", ["0", "1", "2"])
def test_warp_specialised_layouts_bit_exact(cuda_device, layout, monkeypatch):
    """Every CTA layout of the warp-specialised kernel (2 pairs x 4 blocks, 4 pairs x 2
    blocks, 2 pairs x 2 blocks per stage), forced, on chain counts below, inside and above
    one wave, single pass and streamed passes: digests equal to the oracle's."""
    monkeypatch.setenv("TCX_HASH_KERNEL", "ws")
    monkeypatch.setenv("TCX_WS_LAYOUT", layout)
    for size, leaf in ((1000, 64), ((10 << 20) + 100, 1024), (64 << 20, 4096), ((80 << 20) + 4000, 2048)):
        a = seeded(size + int(layout), size)
        d = to_dev(a)
        want = oracle.leaf_digests(a, leaf, openssl=True, threads=8)
        assert (tcx.sha256_leaves(d, leaf).cpu().numpy() == want).all(), (size, leaf)
        n = (size + leaf - 1) // leaf
        digests = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
        states = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
        seg = max(64, (leaf // 3) // 64 * 64)
        for off in range(0, leaf, seg):
            _native.call("tcx_sha256_leaves_pass", d.data_ptr(), size, leaf, off, seg, states.data_ptr(),
                         digests.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
        assert (digests.cpu().numpy() == want).all(), (size, leaf, "streamed")
