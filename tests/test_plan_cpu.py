"""CPU checks of the view planner and of the native exchange schedule (tcx_plan_exchange):
for random artifacts, views and world sizes, executing every rank's schedule in numpy must
give each rank exactly the view the independent numpy oracle materialises."""
import numpy as np
import pytest

from oracle import views as oviews
from tensorcast_b200.loader import plan_exchange, plan_push_split, stage_bounds
from tensorcast_b200.views import ViewSpec, NarrowOp, TransposeOp, plan_view
from viewtools import emulate_load, index_from_meta, random_tensors, random_view, apply_jobs, apply_permutes


def test_planner_matches_oracle_single_rank():
    for seed in range(30):
        canon, meta = oviews.canonical_bytes(random_tensors(seed))
        index = index_from_meta(meta, canon.size)
        rng = np.random.default_rng(1000 + seed)
        for _ in range(4):
            slices, transpose, subset, spec = random_view(meta, rng)
            plan = plan_view(index, spec, subset)
            view = np.full(plan.view_bytes, 0, np.uint8)
            apply_jobs(canon, view, plan.jobs)
            apply_permutes(view, plan.permutes)
            want = oviews.materialize_view(canon, meta, slices, transpose, subset)
            assert view.size == want.size and (view == want).all()


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("leaf", [64, 256, 1000])
def test_exchange_schedule_matches_oracle(world, leaf):
    for seed in range(6):
        canon, meta = oviews.canonical_bytes(random_tensors(seed * 7 + world))
        index = index_from_meta(meta, canon.size)
        rng = np.random.default_rng(seed)
        bounds = stage_bounds(canon.size, leaf, world)
        views = [random_view(meta, rng) for _ in range(world)]
        plans = [plan_view(index, v[3], v[2]) for v in views]
        exch = [plan_exchange(canon.size, leaf, bounds, [p.jobs for p in plans], r, plans[r].view_bytes)
                for r in range(world)]
        got = emulate_load(canon, bounds, plans, exch)
        for r in range(world):
            slices, transpose, subset, _ = views[r]
            want = oviews.materialize_view(canon, meta, slices, transpose, subset)
            assert got[r].size == want.size and (got[r] == want).all(), (seed, r)


def test_tp_llama_schedule_is_direct_and_balanced():
    """Tiny Llama-shaped bf16 artifact, TP-4: every receive lands directly in the view and
    every rank sends and receives about 1/N of its view."""
    from tensorcast_b200.synthetic import llama_shapes, tiny_llama
    shapes = llama_shapes(tiny_llama(layers=3, hidden=64, ffn=128, vocab=512))
    rng = np.random.default_rng(0)
    tensors = {n: (rng.integers(0, 256, int(np.prod(s)) * 2, dtype=np.uint8), s, 2) for n, s in shapes.items()}
    canon, meta = oviews.canonical_bytes(tensors)
    index = index_from_meta(meta, canon.size)
    world, leaf = 4, 4096
    bounds = stage_bounds(canon.size, leaf, world)
    specs = []
    for r in range(world):
        sl = oviews.tp_slices(meta, world, r)
        spec = ViewSpec({n: [NarrowOp(*v)] for n, v in sl.items()})
        specs.append((sl, plan_view(index, spec)))
    exch = [plan_exchange(canon.size, leaf, bounds, [p.jobs for _, p in specs], r, specs[r][1].view_bytes)
            for r in range(world)]
    got = emulate_load(canon, bounds, [p for _, p in specs], exch)
    for r in range(world):
        assert (got[r] == oviews.materialize_view(canon, meta, specs[r][0])).all()
        assert exch[r]["direct"].sum() == world - 1
        assert len(exch[r]["scatter"]) == 0 and len(exch[r]["gaps"]) == 0


def test_reference_planner_cases():
    """view_planner_test.cc-style cases: 8-byte aligned subset packing and narrow segments;
    collective_disk_loader_test.cc:707-826 rect (rows 1-3, cols 2-5 of a 4x6 U8 payload 0..23)."""
    tensors = {"t": (np.arange(256, dtype=np.uint8), (64,), 4), "u": (np.arange(16, dtype=np.uint8), (16,), 1)}
    canon, meta = oviews.canonical_bytes(tensors)
    index = index_from_meta(meta, canon.size)
    # canonical offsets coalesced by sorted name: t -> (0, 256), u -> (256, 16)
    assert index.entries["t"].offset == 0 and index.entries["u"].offset == 256
    plan = plan_view(index, None, ["u", "t"])
    assert [(v.name, v.offset, v.nbytes) for v in plan.tensors] == [("u", 0, 16), ("t", 16, 256)]
    rect = {"r": (np.arange(24, dtype=np.uint8), (4, 6), 1)}
    canon, meta = oviews.canonical_bytes(rect)
    index = index_from_meta(meta, canon.size)
    rows = plan_view(index, ViewSpec({"r": [NarrowOp(0, 1, 3)]}))
    view = np.zeros(rows.view_bytes, np.uint8)
    apply_jobs(canon, view, rows.jobs)
    assert list(view) == list(range(6, 24))
    cols = plan_view(index, ViewSpec({"r": [NarrowOp(1, 2, 4)]}))
    view = np.zeros(cols.view_bytes, np.uint8)
    apply_jobs(canon, view, cols.jobs)
    assert list(view) == [2, 3, 4, 5, 8, 9, 10, 11, 14, 15, 16, 17, 20, 21, 22, 23]


def test_planner_rejects_reference_invalid_views():
    canon, meta = oviews.canonical_bytes({"a": (np.zeros(32, np.uint8), (4, 4), 2)})
    index = index_from_meta(meta, canon.size)
    with pytest.raises(ValueError, match="mixing transpose and narrow"):
        plan_view(index, ViewSpec({"a": [NarrowOp(0, 0, 2), TransposeOp(0, 1)]}))
    with pytest.raises(ValueError, match="multiple narrow"):
        plan_view(index, ViewSpec({"a": [NarrowOp(0, 0, 2), NarrowOp(1, 0, 2)]}))
    with pytest.raises(ValueError, match="unknown tensor"):
        plan_view(index, ViewSpec({"zz": [NarrowOp(0, 0, 1)]}))
    with pytest.raises(ValueError, match="narrow length exceeds"):
        plan_view(index, ViewSpec({"a": [NarrowOp(0, 3, 2)]}))
    fused = plan_view(index, ViewSpec({"a": [NarrowOp(0, 1, 2), TransposeOp(0, 1)]}), allow_fused=True)
    assert fused.tensors[0].shape == (4, 2)


def test_stage_bounds():
    assert stage_bounds(1000, 64, 1) == [0, 1000]
    b = stage_bounds(16_060_522_496, 4 << 20, 8)
    assert b[0] == 0 and b[-1] == 16_060_522_496 and all(x % (4 << 20) == 0 for x in b[:-1])
    n = [(b[i + 1] - b[i] + (4 << 20) - 1) // (4 << 20) for i in range(8)]
    assert sum(n) == 3830 and max(n) - min(n) <= 1


@pytest.mark.parametrize("world", [1, 2, 4])
def test_exchange_schedule_into_sparse_targets(world):
    """bind_into-style destinations: every view tensor relocated to its own place in a sparse
    address space (gaps between targets). The schedule must fill each target exactly, with
    direct receives only where a peer's bytes are contiguous in that space, and the bytes
    between targets must stay untouched (no gap fill for target loads)."""
    from types import SimpleNamespace

    import torch

    from tensorcast_b200.api import _TORCH_DTYPES
    from tensorcast_b200.binding import target_ranges, view_target_jobs
    for seed in range(4):
        canon, meta = oviews.canonical_bytes(random_tensors(50 + seed, n=16))
        index = index_from_meta(meta, canon.size)
        rng = np.random.default_rng(seed)
        leaf = 256
        bounds = stage_bounds(canon.size, leaf, world)
        views, plans, targets_all, sparse = [], [], [], []
        for r in range(world):
            slices, transpose, subset, spec = random_view(meta, rng)
            plan = plan_view(index, spec, subset)
            # one "allocation" per tensor inside a host arena, shuffled order, random gaps
            arena = torch.zeros(plan.view_bytes * 3 + 4096 * len(plan.tensors), dtype=torch.uint8)
            order = rng.permutation(len(plan.tensors))
            cur, targets = 0, {}
            for i in order:
                t = plan.tensors[i]
                cur += int(rng.integers(0, 64)) * 16
                targets[t.name] = arena[cur:cur + t.nbytes].view(_TORCH_DTYPES[t.dtype]).view(t.shape)
                cur = (cur + t.nbytes + 15) // 16 * 16
            base, ranges, vbytes = target_ranges(targets)
            jobs, perms = view_target_jobs(plan, targets, base)
            views.append((slices, transpose, subset))
            plans.append(SimpleNamespace(jobs=jobs, permutes=perms, view_bytes=vbytes))
            targets_all.append((plan, targets, base))
            sparse.append(ranges)
        exch = [plan_exchange(canon.size, leaf, bounds, [p.jobs for p in plans], r, plans[r].view_bytes)
                for r in range(world)]
        got = emulate_load(canon, bounds, plans, exch)
        for r in range(world):
            plan, targets, base = targets_all[r]
            want = oviews.materialize_view(canon, meta, *views[r])
            for t in plan.tensors:
                off = targets[t.name].data_ptr() - base
                assert (got[r][off:off + t.nbytes] == want[t.offset:t.offset + t.nbytes]).all(), (seed, r, t.name)
            # bytes outside every target: only the gap fill may have written them, and a
            # target load skips the gap fill
            covered = np.zeros(got[r].size, bool)
            for a, n in sparse[r]:
                covered[a:a + n] = True
            written_outside = False
            for p in range(world):
                if p != r and exch[r]["direct"][p]:
                    o, n = int(exch[r]["recv_view_off"][p]), int(exch[r]["recv_counts"][p])
                    written_outside |= bool((~covered[o:o + n]).any())
            assert not written_outside, (seed, r)


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("share", [0.0, 0.3, 0.5, 1.0])
def test_push_split_schedule_matches_oracle(world, share):
    """The push exchange with a share over NCCL (tcx_plan_push_split): every rank derives the
    same NCCL pieces; executing, per rank, the full plan's local pieces and gap fill, the NCCL
    part's schedule (tcx_plan_exchange of a plan of only the NCCL pieces) and every sender's
    copy-engine pieces gives each rank exactly the oracle's view, and the NCCL part carries
    at least `share` of the bytes (whole pieces)."""
    leaf = 256
    for seed in range(5):
        canon, meta = oviews.canonical_bytes(random_tensors(seed * 11 + world, n=20))
        index = index_from_meta(meta, canon.size)
        rng = np.random.default_rng(seed + 100)
        bounds = stage_bounds(canon.size, leaf, world)
        views = [random_view(meta, rng) for _ in range(world)]
        plans = [plan_view(index, v[3], v[2]) for v in views]
        rank_jobs = [p.jobs for p in plans]
        splits = [plan_push_split(canon.size, leaf, bounds, rank_jobs, r, share) for r in range(world)]
        for r in range(1, world):
            for q in range(world):
                assert splits[r]["nccl"][q].tobytes() == splits[0]["nccl"][q].tobytes()
        nccl_jobs = splits[0]["nccl"]
        full = [plan_exchange(canon.size, leaf, bounds, rank_jobs, r, plans[r].view_bytes) for r in range(world)]
        part = [plan_exchange(canon.size, leaf, bounds, nccl_jobs, r, plans[r].view_bytes) for r in range(world)]
        views_out, sends = [], []
        for r in range(world):
            stage = canon[bounds[r]:bounds[r + 1]]
            view = np.full(plans[r].view_bytes, 0xA5, np.uint8)
            for off, ln in full[r]["gaps"]:
                view[int(off): int(off) + int(ln)] = 0
            apply_jobs(stage, view, full[r]["local"])
            views_out.append(view)
            send = np.zeros(int(part[r]["send_offsets"][-1]), np.uint8)
            apply_jobs(stage, send, part[r]["pack"])
            sends.append(send)
            assert len(part[r]["local"]) == 0
        nccl_bytes = total_bytes = 0
        for r in range(world):
            x = part[r]
            recv = np.zeros(int(x["recv_offsets"][-1]), np.uint8)
            for p in range(world):
                if p == r:
                    continue
                data = sends[p][int(part[p]["send_offsets"][r]): int(part[p]["send_offsets"][r + 1])]
                nccl_bytes += data.size
                if x["direct"][p]:
                    views_out[r][int(x["recv_view_off"][p]): int(x["recv_view_off"][p]) + data.size] = data
                else:
                    recv[int(x["recv_offsets"][p]): int(x["recv_offsets"][p]) + data.size] = data
                # sender p's copy-engine pieces into r's view
                apply_jobs(canon[bounds[p]:bounds[p + 1]], views_out[r], splits[p]["ce"][r])
                total_bytes += int(full[r]["recv_counts"][p])
            apply_jobs(recv, views_out[r], x["scatter"])
            apply_permutes(views_out[r], plans[r].permutes)
        for r in range(world):
            slices, transpose, subset, _ = views[r]
            want = oviews.materialize_view(canon, meta, slices, transpose, subset)
            assert views_out[r].size == want.size and (views_out[r] == want).all(), (seed, r)
        if share == 0.0:
            assert nccl_bytes == 0
        elif share == 1.0:
            assert nccl_bytes == total_bytes
        else:  # whole pieces in order until the share is reached: at least the share of every pair
            assert share * total_bytes <= nccl_bytes <= total_bytes
