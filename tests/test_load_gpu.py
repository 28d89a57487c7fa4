"""GPU parity of the view kernels and of the single-rank collective load (tcx_group_load)
against the numpy view oracle and the hashing oracle: byte-identical views, bit-exact roots."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from oracle import views as oviews
from tensorcast_b200 import _native
from tensorcast_b200.loader import Group, stage_bounds
from tensorcast_b200.views import JOB_DTYPE, ViewSpec, NarrowOp, TransposeOp, plan_view, permute_array
from viewtools import index_from_meta, random_tensors, random_view

pytestmark = pytest.mark.gpu


def dev(a: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def pinned(a: np.ndarray) -> torch.Tensor:
    t = torch.empty(a.size, dtype=torch.uint8, pin_memory=True)
    t.numpy()[:] = a
    return t


def run_copy_jobs(src: torch.Tensor, dst: torch.Tensor, jobs: np.ndarray) -> None:
    L = _native.lib()
    dj = dev(jobs.view(np.uint8)) if jobs.size else torch.zeros(8, dtype=torch.uint8, device="cuda")
    sb = int(L.tcx_copy_jobs_scratch_bytes(len(jobs)))
    scratch = torch.empty(sb, dtype=torch.uint8, device="cuda")
    _native.call("tcx_copy_jobs", src.data_ptr(), dst.data_ptr(), dj.data_ptr(), len(jobs), scratch.data_ptr(), sb,
                 torch.cuda.current_stream().cuda_stream)


def test_copy_jobs_and_permutes_match_oracle(cuda_device):
    for seed in range(12):
        canon, meta = oviews.canonical_bytes(random_tensors(seed))
        index = index_from_meta(meta, canon.size)
        rng = np.random.default_rng(seed)
        slices, transpose, subset, spec = random_view(meta, rng)
        plan = plan_view(index, spec, subset)
        src = dev(canon)
        view = torch.zeros(max(plan.view_bytes, 1), dtype=torch.uint8, device="cuda")
        run_copy_jobs(src, view, plan.jobs)
        tmp = torch.empty_like(view)
        for p in permute_array(plan.permutes):
            pj = _native.PermuteJob.from_buffer_copy(p.tobytes())
            nbytes = int(np.prod(p["shape"][: p["ndim"]])) * int(p["esize"])
            pj.src_off, pj.dst_off = int(p["dst_off"]), 0
            _native.call("tcx_permute", view.data_ptr(), tmp.data_ptr(), ctypes.byref(pj),
                         torch.cuda.current_stream().cuda_stream)
            view[int(p["dst_off"]): int(p["dst_off"]) + nbytes] = tmp[:nbytes]
        want = oviews.materialize_view(canon, meta, slices, transpose, subset)
        assert (view.cpu().numpy()[: plan.view_bytes] == want).all()


@pytest.mark.parametrize("esize", [2, 1, 4, 8])
@pytest.mark.parametrize("rows,cols", [(64, 64), (4096, 1024), (130, 77), (8192, 8192), (1, 640), (640, 1),
                                       (200, 136), (256, 144), (136, 4096)])
def test_transpose_shapes(cuda_device, rows, cols, esize):
    """2-D transposes: full and edge tiles, aligned (16-byte rows) and unaligned shapes."""
    dt = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[esize]
    if esize == 8 and rows * cols > 1 << 24:
        pytest.skip("large 8-byte case adds nothing over the 2-byte one")
    a = np.random.default_rng(rows + cols).integers(0, np.iinfo(dt).max, size=(rows, cols), dtype=dt)
    src, out = dev(a.view(np.uint8).reshape(-1)), torch.empty(a.size * esize, dtype=torch.uint8, device="cuda")
    pj = _native.PermuteJob(0, 0, esize, 2)
    pj.shape[0], pj.shape[1], pj.perm[0], pj.perm[1] = rows, cols, 1, 0
    _native.call("tcx_permute", src.data_ptr(), out.data_ptr(), ctypes.byref(pj), torch.cuda.current_stream().cuda_stream)
    assert (out.cpu().numpy().view(dt).reshape(cols, rows) == a.T).all()


def test_streamed_passes_match_single_pass(cuda_device):
    a = np.random.default_rng(9).integers(0, 256, size=(7 << 20) + 4133, dtype=np.uint8)
    src = dev(a)
    for leaf, seg in ((1 << 20, 64 << 10), (1 << 20, 192), (4096, 1 << 20), (65536 + 64, 4096)):
        n = (a.size + leaf - 1) // leaf
        digests = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
        states = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        for off in range(0, leaf, seg):
            _native.call("tcx_sha256_leaves_pass", src.data_ptr(), a.size, leaf, off, seg, states.data_ptr(),
                         digests.data_ptr(), n, s)
        assert (digests.cpu().numpy() == oracle.leaf_digests(a, leaf, openssl=True, threads=8)).all()


@pytest.mark.parametrize("kernel", ["plain", "ws"])
def test_both_leaf_kernels_bit_exact(cuda_device, kernel, monkeypatch):
    monkeypatch.setenv("TCX_HASH_KERNEL", kernel)
    import tensorcast_b200 as tcx
    for size, leaf in ((1, 64), (1000, 64), (1 << 20, 4096), ((3 << 20) + 57, 1 << 18), (70 << 20, 4 << 20)):
        a = np.random.default_rng(size).integers(0, 256, size=size, dtype=np.uint8)
        d = tcx.sha256_leaves(dev(a), leaf).cpu().numpy()
        assert (d == oracle.leaf_digests(a, leaf, openssl=True, threads=8)).all()


@pytest.mark.parametrize("host", [True, False])
def test_single_rank_load_random_views(cuda_device, host):
    g = Group(1, 0, 0)
    try:
        for seed in range(8):
            canon, meta = oviews.canonical_bytes(random_tensors(seed, n=20))
            index = index_from_meta(meta, canon.size)
            rng = np.random.default_rng(seed)
            slices, transpose, subset, spec = random_view(meta, rng)
            plan = plan_view(index, spec, subset)
            leaf = int(rng.choice([64, 256, 1024]))
            d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
            if not host:
                d_stage.copy_(dev(canon))
            d_view = torch.full((max(plan.view_bytes, 1),), 0x5A, dtype=torch.uint8, device="cuda")
            expected = oracle.tree_root(oracle.leaf_digests(canon, leaf))
            res = g.load(canon.size, leaf, [0, canon.size], [plan.jobs], d_stage=d_stage, d_view=d_view,
                         h_stage=pinned(canon) if host else None, permutes=plan.permutes,
                         view_bytes=plan.view_bytes, expected_root=expected, slab_bytes=128, view_hash=True)
            assert res["root"] == expected
            assert res["multihash"] == oracle.multihash(expected)
            want = oviews.materialize_view(canon, meta, slices, transpose, subset)
            assert (d_view.cpu().numpy()[: plan.view_bytes] == want).all()
            # the view hash: the GPU entry's data multihash of the view bytes (adaptive leaf policy),
            # as view_hash_utils_test.cc:94-145 / store_engine_view_test.cc:93-161 pin it: equal to
            # the CPU hash of the expected view bytes
            assert res["view_multihash"] == oracle.multihash_gpu_semantics(want)
    finally:
        g.close()


def test_load_detects_corruption(cuda_device):
    canon, meta = oviews.canonical_bytes(random_tensors(3))
    index = index_from_meta(meta, canon.size)
    plan = plan_view(index)
    g = Group(1, 0, 0)
    try:
        expected = oracle.tree_root(oracle.leaf_digests(canon, 64))
        bad = canon.copy()
        bad[bad.size // 2] ^= 1
        d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
        with pytest.raises(_native.TcxError, match="ARTIFACT_ID_MISMATCH"):
            g.load(canon.size, 64, [0, canon.size], [plan.jobs], d_stage=d_stage, d_view=d_stage,
                   h_stage=pinned(bad), view_bytes=plan.view_bytes, expected_root=expected)
        res = g.load(canon.size, 64, [0, canon.size], [plan.jobs], d_stage=d_stage, d_view=d_stage,
                     h_stage=pinned(canon), view_bytes=plan.view_bytes, expected_root=expected)
        assert res["root"] == expected
    finally:
        g.close()


def test_load_from_registered_file_mapping(cuda_device, tmp_path):
    """Staging straight from a file's page-cache pages (tcx_host_map_file) gives the same root."""
    from tensorcast_b200.loader import FileMapping
    canon, meta = oviews.canonical_bytes(random_tensors(9, n=30))
    index = index_from_meta(meta, canon.size)
    plan = plan_view(index)
    base = "/dev/shm" if os.path.isdir("/dev/shm") else str(tmp_path)
    path = os.path.join(base, f"tcx_map_test_{os.getpid()}.bin")
    head = 4096 + 123  # the staged range starts at an unaligned file offset
    with open(path, "wb") as f:
        f.write(b"\0" * head)
        f.write(canon.tobytes())
    try:
        m = FileMapping(str(path), head, canon.size, register=True)
    except _native.TcxError as e:
        os.unlink(path)
        pytest.skip(f"driver does not register file mappings here: {e}")
    g = Group(1, 0, 0)
    try:
        d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
        expected = oracle.tree_root(oracle.leaf_digests(canon, 256))
        res = g.load(canon.size, 256, [0, canon.size], [plan.jobs], d_stage=d_stage, d_view=d_stage, h_stage=m,
                     view_bytes=plan.view_bytes, expected_root=expected)
        assert res["root"] == expected
        assert (d_stage.cpu().numpy() == canon).all()
    finally:
        g.close()
        m.close()
        os.unlink(path)


def _rect_job(src_cols, dst_cols, sr0, sr1, sc0, sc1, dr0, dc0, esize=1):
    return (sr0 * src_cols * esize + sc0 * esize, dr0 * dst_cols * esize + dc0 * esize, src_cols * esize,
            dst_cols * esize, (sc1 - sc0) * esize, sr1 - sr0)


@pytest.mark.parametrize("case", ["4x6", "6x8_to_6x9"])
def test_reference_rect2d_cases_into_target(cuda_device, case):
    """collective_disk_loader_test.cc:707-900: rect2d copies of a U8 payload 0..n-1 into a
    target pre-filled with 0xEE, through tcx_group_load with TCX_LOAD_TARGETS (the local
    mapped-target load): the rectangles land exactly, every other byte stays 0xEE."""
    if case == "4x6":
        rows, cols, drows, dcols = 4, 6, 4, 6
        rects = [(1, 3, 2, 5, 0, 1)]
    else:
        rows, cols, drows, dcols = 6, 8, 6, 9
        rects = [(1, 3, 2, 6, 0, 1), (3, 6, 0, 3, 3, 5)]
    payload = np.arange(rows * cols, dtype=np.uint8)
    want = np.full((drows, dcols), 0xEE, np.uint8)
    src2 = payload.reshape(rows, cols)
    jobs = []
    for sr0, sr1, sc0, sc1, dr0, dc0 in rects:
        want[dr0:dr0 + sr1 - sr0, dc0:dc0 + sc1 - sc0] = src2[sr0:sr1, sc0:sc1]
        jobs.append(_rect_job(cols, dcols, sr0, sr1, sc0, sc1, dr0, dc0))
    jobs = np.array(jobs, dtype=JOB_DTYPE)
    target = torch.full((drows * dcols,), 0xEE, dtype=torch.uint8, device="cuda")
    d_stage = torch.empty(payload.size, dtype=torch.uint8, device="cuda")
    g = Group(1, 0, 0)
    try:
        expected = oracle.tree_root(oracle.leaf_digests(payload, 64))
        res = g.load(payload.size, 64, [0, payload.size], [jobs], d_stage=d_stage, d_view=target.data_ptr(),
                     h_stage=pinned(payload), view_bytes=target.numel(), expected_root=expected,
                     target_ranges=[(0, target.numel())])
        assert res["root"] == expected
        torch.cuda.synchronize()
        assert (target.cpu().numpy().reshape(drows, dcols) == want).all()
    finally:
        g.close()


def test_reference_replicated_case_into_target(cuda_device):
    """collective_disk_loader_test.cc:492-590: a replicated U8[16] tensor (0x40..0x4F) copied
    whole into a 16-byte target pre-filled with 0xEE."""
    payload = (0x40 + np.arange(16)).astype(np.uint8)
    target = torch.full((16,), 0xEE, dtype=torch.uint8, device="cuda")
    d_stage = torch.empty(16, dtype=torch.uint8, device="cuda")
    g = Group(1, 0, 0)
    try:
        jobs = np.array([(0, 0, 16, 16, 16, 1)], dtype=JOB_DTYPE)
        g.load(16, 64, [0, 16], [jobs], d_stage=d_stage, d_view=target.data_ptr(), h_stage=pinned(payload),
               view_bytes=16, target_ranges=[(0, 16)])
        torch.cuda.synchronize()
        assert (target.cpu().numpy() == payload).all()
    finally:
        g.close()


def _write_shuffled_files(tmp_path, canon, meta, n_files=2, seed=0):
    """Writes every tensor's bytes into one of n_files files, in a shuffled payload order with
    junk between them; returns (path, file_offset, canonical_offset, length) per tensor."""
    rng = np.random.default_rng(seed)
    names = list(meta)
    order = [names[i] for i in rng.permutation(len(names))]
    bufs = [bytearray(int(rng.integers(0, 64))) for _ in range(n_files)]
    out = []
    for k, n in enumerate(order):
        off, shape, es = meta[n]
        ln = (int(np.prod(shape)) if shape else 1) * es
        f = k % n_files
        bufs[f] += bytes(int(rng.integers(0, 24)))  # junk before the tensor
        out.append((str(tmp_path / f"part{f}.bin"), len(bufs[f]), off, ln))
        bufs[f] += canon[off:off + ln].tobytes()
    for f in range(n_files):
        (tmp_path / f"part{f}.bin").write_bytes(bytes(bufs[f]) + bytes(100))
    return out


def _segments_for(tensor_segs, lo, hi):
    segs = []
    for path, foff, coff, ln in tensor_segs:
        a, b = max(lo, coff), min(hi, coff + ln)
        if a < b:
            segs.append((path, foff + (a - coff), a - lo, b - a))
    return segs


@pytest.mark.parametrize("threads,slot_bytes", [(1, 0), (4, 1 << 16), (7, 3 << 12)])
def test_file_staged_load_matches_oracle(cuda_device, tmp_path, threads, slot_bytes):
    """tcx_group_load_files: the range read from several files (shuffled payload order, pads
    between tensors left to the loader), slabs smaller than the ring so slots are reused;
    root and view bit-exact against the oracles."""
    g = Group(1, 0, 0)
    try:
        for seed in range(4):
            canon, meta = oviews.canonical_bytes(random_tensors(seed + 100, n=24))
            index = index_from_meta(meta, canon.size)
            tseg = _write_shuffled_files(tmp_path, canon, meta, n_files=1 + seed % 3, seed=seed)
            rng = np.random.default_rng(seed)
            slices, transpose, subset, spec = random_view(meta, rng)
            plan = plan_view(index, spec, subset)
            for leaf in (64, 1024, 4096 + 64):
                d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
                d_view = torch.zeros(max(plan.view_bytes, 1), dtype=torch.uint8, device="cuda")
                res = g.load(canon.size, leaf, [0, canon.size], [plan.jobs], d_stage=d_stage, d_view=d_view,
                             files=_segments_for(tseg, 0, canon.size), permutes=plan.permutes,
                             view_bytes=plan.view_bytes, read_threads=threads, ring_slots=2,
                             slot_bytes=slot_bytes)
                assert res["root"] == oracle.tree_root(oracle.leaf_digests(canon, leaf))
                assert (d_stage.cpu().numpy() == canon).all()
                want = oviews.materialize_view(canon, meta, slices, transpose, subset)
                assert (d_view.cpu().numpy()[: plan.view_bytes] == want).all()
    finally:
        g.close()


def test_file_staged_load_errors_then_recovers(cuda_device, tmp_path, monkeypatch):
    monkeypatch.setenv("TCX_STAGE", "slabs")  # the slab ring (leaves this long default to pieces)
    canon = np.random.default_rng(5).integers(0, 256, size=(3 << 20) + 4000, dtype=np.uint8)
    path = tmp_path / "a.bin"
    path.write_bytes(canon.tobytes())
    leaf = 1 << 18
    g = Group(1, 0, 0)
    try:
        d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
        kw = dict(d_stage=d_stage, d_view=d_stage, view_bytes=canon.size, read_threads=3, ring_slots=2,
                  slot_bytes=1 << 16)
        with pytest.raises(_native.TcxError) as e:
            g.load(canon.size, leaf, [0, canon.size], [np.zeros(0, JOB_DTYPE)],
                   files=[(str(tmp_path / "missing.bin"), 0, 0, canon.size)], **kw)
        assert e.value.code == _native.NOT_FOUND
        short = tmp_path / "short.bin"
        short.write_bytes(canon[: canon.size - 100].tobytes())
        with pytest.raises(_native.TcxError) as e:
            g.load(canon.size, leaf, [0, canon.size], [np.zeros(0, JOB_DTYPE)],
                   files=[(str(short), 0, 0, canon.size)], **kw)
        assert e.value.code == _native.DATA_LOSS and "short read" in e.value.message
        res = g.load(canon.size, leaf, [0, canon.size], [np.zeros(0, JOB_DTYPE)],
                     files=[(str(path), 0, 0, canon.size)], **kw)
        assert res["root"] == oracle.tree_root(oracle.leaf_digests(canon, leaf))
        assert res["stage_read_ms"] > 0
    finally:
        g.close()


def _random_segments(tmp_path, canon, rng, n_files=2):
    """Covers canon with file segments of random lengths in two files (junk before each
    segment); holes between segments are zeroed in canon, as the loader fills them."""
    bufs = [bytearray(int(rng.integers(0, 64))) for _ in range(n_files)]
    segs, pos, k = [], 0, 0
    while pos < canon.size:
        hole = int(rng.integers(0, 100)) if rng.random() < 0.3 else 0
        canon[pos:pos + hole] = 0
        pos = min(canon.size, pos + hole)
        ln = min(int(rng.integers(1000, 300000)), canon.size - pos)
        if ln <= 0:
            break
        f = k % n_files
        bufs[f] += bytes(int(rng.integers(0, 24)))
        segs.append((str(tmp_path / f"piece{f}.bin"), len(bufs[f]), pos, ln))
        bufs[f] += canon[pos:pos + ln].tobytes()
        pos += ln
        k += 1
    for f in range(n_files):
        (tmp_path / f"piece{f}.bin").write_bytes(bytes(bufs[f]))
    return segs


@pytest.mark.parametrize("threads,bufs,leaf,copy", [(1, 1, 1 << 18, 1 << 16), (4, 3, 1 << 17, 3 << 16),
                                                     (7, 2, (1 << 18) + 4096, 1 << 20), (3, 2, 1 << 18, 1 << 30)])
def test_piece_staged_load_matches_oracle(cuda_device, tmp_path, monkeypatch, threads, bufs, leaf, copy):
    """Piece staging (each reader queues one host-to-device copy of the pieces of a few
    consecutive leaves it has read, on its own stream, from a few reused pinned buffers):
    several files with holes and junk, a short last leaf alone or inside a group, one leaf
    per copy up to all leaves in one copy, one to seven readers; root, staged bytes and a
    strided view bit-exact, and the same group loads again after the reader count changes."""
    from viewtools import apply_jobs
    monkeypatch.setenv("TCX_STAGE", "pieces")
    monkeypatch.setenv("TCX_STAGE_PIECE", str(1 << 16))
    monkeypatch.setenv("TCX_STAGE_PIECE_BUFS", str(bufs))
    monkeypatch.setenv("TCX_STAGE_COPY", str(copy))
    rng = np.random.default_rng(threads)
    canon = rng.integers(0, 256, size=5 * leaf + 12345, dtype=np.uint8)
    segs = _random_segments(tmp_path, canon, rng)
    jobs = np.zeros(3, JOB_DTYPE)
    jobs[0] = (1000, 0, 2048, 1024, 1024, 300)          # a strided 2-D piece
    jobs[1] = (canon.size - 5000, 300 * 1024, 0, 0, 5000, 1)  # the short last leaf's end
    jobs[2] = (3 * leaf - 7, 300 * 1024 + 5000, 0, 0, 777, 1)  # across a leaf boundary
    view_bytes = 300 * 1024 + 5000 + 777
    want = np.zeros(view_bytes, np.uint8)
    apply_jobs(canon, want, jobs)
    g = Group(1, 0, 0)
    try:
        for nt in (threads, threads + 2):
            d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
            d_view = torch.zeros(view_bytes, dtype=torch.uint8, device="cuda")
            res = g.load(canon.size, leaf, [0, canon.size], [jobs], d_stage=d_stage, d_view=d_view, files=segs,
                         view_bytes=view_bytes, read_threads=nt)
            assert res["root"] == oracle.tree_root(oracle.leaf_digests(canon, leaf))
            assert (d_stage.cpu().numpy() == canon).all()
            assert (d_view.cpu().numpy() == want).all()
            assert res["stage_read_ms"] > 0
    finally:
        g.close()


def test_piece_staged_load_errors_then_recovers(cuda_device, tmp_path, monkeypatch):
    monkeypatch.setenv("TCX_STAGE", "pieces")
    monkeypatch.setenv("TCX_STAGE_PIECE", str(1 << 16))
    canon = np.random.default_rng(6).integers(0, 256, size=(3 << 20) + 4000, dtype=np.uint8)
    path = tmp_path / "a.bin"
    path.write_bytes(canon.tobytes())
    leaf = 1 << 18
    g = Group(1, 0, 0)
    try:
        d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
        d_view = torch.zeros(canon.size, dtype=torch.uint8, device="cuda")
        whole = np.zeros(1, JOB_DTYPE)
        whole[0] = (0, 0, 0, 0, canon.size, 1)
        kw = dict(d_stage=d_stage, d_view=d_view, view_bytes=canon.size, read_threads=3)
        short = tmp_path / "short.bin"
        short.write_bytes(canon[: canon.size - 100].tobytes())
        with pytest.raises(_native.TcxError) as e:
            g.load(canon.size, leaf, [0, canon.size], [whole], files=[(str(short), 0, 0, canon.size)], **kw)
        assert e.value.code == _native.DATA_LOSS and "short read" in e.value.message
        res = g.load(canon.size, leaf, [0, canon.size], [whole], files=[(str(path), 0, 0, canon.size)], **kw)
        assert res["root"] == oracle.tree_root(oracle.leaf_digests(canon, leaf))
        assert (d_stage.cpu().numpy() == canon).all()
        assert (d_view.cpu().numpy() == canon).all()
    finally:
        g.close()


@pytest.mark.parametrize("size,leaf", [(300 << 10, 1 << 20), (6 << 18, 1 << 18)])
def test_piece_staged_load_edges(cuda_device, tmp_path, monkeypatch, size, leaf):
    """Piece staging of a range shorter than one leaf (only the short leaf, in pieces) and of
    a range of whole leaves (no short leaf); root and staged bytes bit-exact."""
    monkeypatch.setenv("TCX_STAGE", "pieces")
    monkeypatch.setenv("TCX_STAGE_PIECE", str(1 << 16))
    canon = np.random.default_rng(size).integers(0, 256, size=size, dtype=np.uint8)
    segs = _random_segments(tmp_path, canon, np.random.default_rng(size + 1))
    g = Group(1, 0, 0)
    try:
        d_stage = torch.empty(canon.size, dtype=torch.uint8, device="cuda")
        d_view = torch.zeros(canon.size, dtype=torch.uint8, device="cuda")
        whole = np.zeros(1, JOB_DTYPE)
        whole[0] = (0, 0, 0, 0, canon.size, 1)
        res = g.load(canon.size, leaf, [0, canon.size], [whole], d_stage=d_stage, d_view=d_view, files=segs,
                     view_bytes=canon.size, read_threads=3)
        assert res["root"] == oracle.tree_root(oracle.leaf_digests(canon, leaf))
        assert (d_stage.cpu().numpy() == canon).all() and (d_view.cpu().numpy() == canon).all()
    finally:
        g.close()
