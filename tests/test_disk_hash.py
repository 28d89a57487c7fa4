"""compute_data_multihash_from_disk_dir on the GPU (tensorcast_b200.disk_hash).

The layout cases restate disk_dir_hash_test.cc:44-137 and disk_artifact_context_test.cc
(numeric partition order, safetensors payloads, no index); the expected value is always
the CPU oracle's multihash of the concatenated bytes with 4 MiB leaves, as the
reference tests compare against compute_data_multihash_from_cpu_memory."""
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle
from tensorcast_b200 import disk_hash
from tensorcast_b200.synthetic import llama_shapes, tiny_llama, write_safetensors


def _write_safetensors_u8(path, name, payload: bytes):
    hdr = json.dumps({name: {"dtype": "U8", "shape": [len(payload)], "data_offsets": [0, len(payload)]}}).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hdr)) + hdr + payload)


def _numbered_parts(d, count=12, size=7):
    expected = bytearray()
    for i in range(count):
        start = ord("A") + i
        chunk = bytes(start + (j % 26) for j in range(size))
        with open(os.path.join(d, f"tensor.data_{i}"), "wb") as f:
            f.write(chunk)
        expected += chunk
    return bytes(expected)


def test_layout_orders_partitions_numerically(tmp_path):
    expected = _numbered_parts(tmp_path)
    with open(tmp_path / "tensor_index.json", "w") as f:
        json.dump({"__dummy__": [0, len(expected), [], [], "torch.uint8", 0]}, f)
    segs, total, kind = disk_hash.disk_dir_layout(tmp_path)
    assert kind == "partitions" and total == len(expected)
    assert [os.path.basename(s[0]) for s in segs] == [f"tensor.data_{i}" for i in range(12)]
    assert [s[2] for s in segs] == [7 * i for i in range(12)]


def test_layout_without_index_uses_physical_bytes(tmp_path):
    (tmp_path / "tensor.data_10").write_bytes(b"ghijkl")
    (tmp_path / "tensor.data_2").write_bytes(b"abcdef")
    segs, total, _ = disk_hash.disk_dir_layout(tmp_path)
    assert total == 12 and [os.path.basename(s[0]) for s in segs] == ["tensor.data_2", "tensor.data_10"]


def test_layout_index_cuts_last_partition_and_errors(tmp_path):
    (tmp_path / "tensor.data_0").write_bytes(b"a" * 10)
    (tmp_path / "tensor.data_1").write_bytes(b"b" * 10)
    with open(tmp_path / "tensor_index.json", "w") as f:
        json.dump({"x": [0, 15, [15], [1], "torch.uint8", 0]}, f)
    segs, total, _ = disk_hash.disk_dir_layout(tmp_path)
    assert total == 15 and segs[-1][3] == 5
    with open(tmp_path / "tensor_index.json", "w") as f:
        json.dump({"x": [0, 25, [25], [1], "torch.uint8", 0]}, f)
    with pytest.raises(disk_hash.DiskHashError, match="exceeds physical partition bytes") as ei:
        disk_hash.disk_dir_layout(tmp_path)
    assert ei.value.status_code == "FAILED_PRECONDITION"
    with open(tmp_path / "tensor_index.json", "w") as f:
        json.dump({"x": [0, 5, [5], [1], "torch.uint8", 0]}, f)
    with pytest.raises(disk_hash.DiskHashError, match="falls before the final partition"):
        disk_hash.disk_dir_layout(tmp_path)


def test_layout_safetensors_payloads_in_name_order(tmp_path):
    _write_safetensors_u8(tmp_path / "b.safetensors", "w_b", b"BBBBBBBB")
    _write_safetensors_u8(tmp_path / "a.safetensors", "w_a", b"AAAAAAAA")
    (tmp_path / "artifact_descriptor.json").write_text("{}")
    segs, total, kind = disk_hash.disk_dir_layout(tmp_path)
    assert kind == "safetensors" and total == 16
    assert [os.path.basename(s[0]) for s in segs] == ["a.safetensors", "b.safetensors"]
    # the payload starts after the 8-byte length and the header
    with open(segs[0][0], "rb") as f:
        f.seek(segs[0][1])
        assert f.read(8) == b"AAAAAAAA"


def test_layout_errors(tmp_path):
    with pytest.raises(disk_hash.DiskHashError, match="Artifact directory not found") as ei:
        disk_hash.disk_dir_layout(tmp_path / "missing")
    assert ei.value.status_code == "NOT_FOUND"
    (tmp_path / "notes.txt").write_text("x")
    with pytest.raises(disk_hash.DiskHashError, match="No replica partition files found"):
        disk_hash.disk_dir_layout(tmp_path)
    with pytest.raises(disk_hash.DiskHashError, match="Expected artifact path to be a directory"):
        disk_hash.disk_dir_layout(tmp_path / "notes.txt")
    # a canonical total (8-byte aligned starts) larger than the payload bytes
    _write_safetensors_u8(tmp_path / "m.safetensors", "a", b"123")
    hdr = json.dumps({"b": {"dtype": "U8", "shape": [3], "data_offsets": [0, 3]}}).encode()
    (tmp_path / "n.safetensors").write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"456")
    with pytest.raises(disk_hash.DiskHashError, match="exceeds safetensors payload bytes"):
        disk_hash.disk_dir_layout(tmp_path)


@pytest.mark.gpu
def test_disk_dir_hash_matches_reference_cases(cuda_device, tmp_path):
    d1 = tmp_path / "parts"
    d1.mkdir()
    expected = _numbered_parts(d1)
    with open(d1 / "tensor_index.json", "w") as f:
        json.dump({"__dummy__": [0, len(expected), [], [], "torch.uint8", 0]}, f)
    assert disk_hash.compute_data_multihash_from_disk_dir(d1) == oracle.multihash_from_cpu_memory(expected)
    d2 = tmp_path / "st"
    d2.mkdir()
    _write_safetensors_u8(d2 / "part0.safetensors", "weights", b"abcdefgh")
    assert disk_hash.compute_data_multihash_from_disk_dir(d2) == oracle.multihash_from_cpu_memory(b"abcdefgh")
    d3 = tmp_path / "noindex"
    d3.mkdir()
    (d3 / "tensor.data_10").write_bytes(b"ghijkl")
    (d3 / "tensor.data_2").write_bytes(b"abcdef")
    assert disk_hash.compute_data_multihash_from_disk_dir(d3) == oracle.multihash_from_cpu_memory(b"abcdefghijkl")


@pytest.mark.gpu
@pytest.mark.parametrize("stage", ["pieces", "slabs"])
@pytest.mark.parametrize("group_bytes,depth", [(0, 0), (4 << 20, 2), (12 << 20, 3)])
def test_disk_dir_hash_streams_many_groups(cuda_device, tmp_path, monkeypatch, group_bytes, depth, stage):
    """Partitions with ragged sizes that straddle leaves and groups; several groups in flight
    (TCX_STAGE=slabs: whole-leaf groups; default: the leaves streamed in 256 KiB pieces)."""
    monkeypatch.setenv("TCX_STAGE", stage)
    rng = np.random.default_rng(11)
    sizes = [5 << 20, 1, (3 << 20) + 17, 0, 9 << 20, 12345]
    blobs = [rng.integers(0, 256, n, dtype=np.uint8).tobytes() for n in sizes]
    for i, b in enumerate(blobs):
        (tmp_path / f"tensor.data_{i}").write_bytes(b)
    stream = b"".join(blobs)
    seen = []
    got = disk_hash.compute_data_multihash_from_disk_dir(tmp_path, lambda done, tot: seen.append((done, tot)),
                                                         group_bytes=group_bytes, depth=depth, read_threads=3)
    assert got == oracle.multihash_from_cpu_memory(stream)
    assert seen[0] == (0, len(stream)) and seen[-1] == (len(stream), len(stream))
    assert all(a[0] <= b[0] for a, b in zip(seen, seen[1:]))


@pytest.mark.gpu
@pytest.mark.parametrize("leaf,wave,threads", [(1 << 18, 3, 2), (1 << 17, 1, 5), ((1 << 18) + 64, 7, 16)])
def test_streamed_file_hash_in_waves(cuda_device, tmp_path, monkeypatch, leaf, wave, threads):
    """The streamed path with waves of a few leaves (each slab a piece of every leaf of the wave,
    copies of several leaves at once, a ring of three slab buffers reused many times), ragged
    segments over three files and a short last leaf; equal to the CPU oracle with that leaf."""
    monkeypatch.setenv("TCX_HASH_WAVE_LEAVES", str(wave))
    rng = np.random.default_rng(leaf + wave)
    data = rng.integers(0, 256, size=13 * leaf + 4321, dtype=np.uint8)
    segs, pos, k = [], 0, 0
    files = [bytearray() for _ in range(3)]
    while pos < data.size:
        ln = min(int(rng.integers(1, 400000)), data.size - pos)
        f = k % 3
        files[f] += bytes(int(rng.integers(0, 9)))
        segs.append((str(tmp_path / f"s{f}.bin"), len(files[f]), pos, ln))
        files[f] += data[pos:pos + ln].tobytes()
        pos, k = pos + ln, k + 1
    for f in range(3):
        (tmp_path / f"s{f}.bin").write_bytes(bytes(files[f]))
    seen = []
    got = disk_hash.compute_data_multihash_from_segments(segs, data.size, leaf_chunk_bytes=leaf, read_threads=threads,
                                                         progress_cb=lambda d, t: seen.append(d))
    want = oracle.multihash(oracle.tree_root(oracle.leaf_digests(data, leaf)))
    assert got == want
    assert seen[0] == 0 and seen[-1] == data.size and seen == sorted(seen)
    short = tmp_path / "short.bin"
    short.write_bytes(data[: data.size - 10].tobytes())
    with pytest.raises(disk_hash.DiskHashError, match="short read while hashing source"):
        disk_hash.compute_data_multihash_from_segments([(str(short), 0, 0, data.size)], data.size,
                                                       leaf_chunk_bytes=leaf, read_threads=threads)
    assert disk_hash.compute_data_multihash_from_segments(segs, data.size, leaf_chunk_bytes=leaf,
                                                          read_threads=threads) == want


@pytest.mark.gpu
def test_disk_dir_hash_of_safetensors_model(cuda_device, tmp_path):
    """A Llama-shaped bf16 safetensors file: the hash equals the payload's CPU multihash."""
    path = tmp_path / "model.safetensors"
    info = write_safetensors(str(path), llama_shapes(tiny_llama(layers=3, hidden=256, ffn=512, vocab=4096)), 5)
    raw = np.fromfile(path, dtype=np.uint8)[info["payload_offset"]:]
    assert disk_hash.compute_data_multihash_from_disk_dir(tmp_path, group_bytes=1 << 20) == \
        oracle.multihash_from_cpu_memory(raw)


@pytest.mark.gpu
def test_disk_hash_errors(cuda_device, tmp_path):
    p = tmp_path / "tensor.data"
    p.write_bytes(b"x" * 100)
    with pytest.raises(disk_hash.DiskHashError, match="short read while hashing source") as ei:
        disk_hash.compute_data_multihash_from_segments([(str(p), 0, 0, 200)], 200)
    assert ei.value.status_code == "DATA_LOSS"
    with pytest.raises(disk_hash.DiskHashError, match="total_size must be > 0"):
        disk_hash.compute_data_multihash_from_segments([], 0)
    with pytest.raises(disk_hash.DiskHashError, match="segments cover"):
        disk_hash.compute_data_multihash_from_segments([(str(p), 0, 0, 50)], 100)
    p.write_bytes(b"")
    with pytest.raises(disk_hash.DiskHashError, match="total_size must be > 0"):
        disk_hash.compute_data_multihash_from_disk_dir(tmp_path)
