"""The multi-rank collective-load parity cases, shared by both process models: one process
per GPU (tests/mp_load_worker.py, torch.distributed) and one thread per GPU in one process
(tests/threads_load_worker.py, tcx_group_join). Every case checks this rank's view against
the numpy oracle byte for byte and the Merkle root against the CPU oracle."""
from __future__ import annotations

import os

import numpy as np
import torch

from oracle import oracle
from oracle import views as oviews
from tensorcast_b200.loader import stage_bounds
from tensorcast_b200.synthetic import llama_shapes, tiny_llama
from tensorcast_b200.views import NarrowOp, TransposeOp, ViewSpec, plan_view
from viewtools import index_from_meta, random_tensors, random_view


def llama_tensors() -> dict:
    shapes = llama_shapes(tiny_llama(layers=4, hidden=256, heads=8, kv_heads=4, head_dim=32, ffn=512, vocab=1024))
    rng = np.random.default_rng(7)
    return {n: (rng.integers(0, 256, int(np.prod(s)) * 2, dtype=np.uint8), s, 2) for n, s in shapes.items()}


def run_cases(group, world: int, rank: int, gather, tmpdir: str, log=print) -> int:
    """All exchange modes (NCCL send/recv with and without windows, peer push, the push with
    a share of every pair's bytes over NCCL, windowed all-gather), staged from pinned
    memory, from files, or device-resident; then the
    bind-into targets case. gather(jobs) returns every rank's jobs. Returns the failures."""
    failures = 0
    llama = llama_tensors()
    # 64 KiB leaves stage from files in slabs, 256 KiB leaves in pieces.
    cases = [("llama", llama, 1 << 16), ("llama_pieces", llama, 1 << 18)]
    for seed in range(3):
        cases.append((f"random{seed}", random_tensors(100 + seed, n=24),
                      int(np.random.default_rng(seed).choice([64, 512, 4096]))))
    for name, tensors, leaf in cases:
        canon, meta = oviews.canonical_bytes(tensors)
        index = index_from_meta(meta, canon.size)
        if name.startswith("llama"):
            sl = oviews.tp_slices(meta, world, rank)
            o = "model.layers.1.self_attn.o_proj.weight"
            sl.pop(o)
            spec = ViewSpec({n: [NarrowOp(*v)] for n, v in sl.items()})
            spec.tensors[o] = [TransposeOp(0, 1)]
            slices, transpose, subset = sl, {o: [(0, 1)]}, None
        else:
            slices, transpose, subset, spec = random_view(meta, np.random.default_rng(1000 * rank + leaf))
        plan = plan_view(index, spec, subset)
        rank_jobs = gather(plan.jobs)
        bounds = stage_bounds(canon.size, leaf, world)
        lo, hi = bounds[rank], bounds[rank + 1]
        h = torch.empty(max(hi - lo, 1), dtype=torch.uint8, pin_memory=True)
        h.numpy()[: hi - lo] = canon[lo:hi]
        path = os.path.join(tmpdir, f"{name}.r{rank}.bin")
        with open(path, "wb") as f:
            f.write(b"\xee" * 40 + canon.tobytes())
        files = [(path, 40 + lo, 0, hi - lo)] if hi > lo else []
        d_stage = torch.empty(max(hi - lo, 1), dtype=torch.uint8, device="cuda")
        d_view = torch.full((max(plan.view_bytes, 1),), 0x3C, dtype=torch.uint8, device="cuda")
        want_root = oracle.tree_root(oracle.leaf_digests(canon, leaf))
        want = oviews.materialize_view(canon, meta, slices, transpose, subset)
        for src, window, push, ag, share in (("host", 0, False, False, 0), ("device", 0, False, False, 0),
                                             ("device", 1000, False, False, 0), ("host", 4096, False, False, 0),
                                             ("files", 0, False, False, 0), ("host", 0, True, False, 0),
                                             ("device", 0, True, False, 0), ("files", 0, True, False, 0),
                                             ("device", 0, True, False, 0.5), ("files", 2048, True, False, 0.3),
                                             ("host", 1000, True, False, 1.0),
                                             ("host", 0, False, True, 0), ("device", 3000, False, True, 0),
                                             ("files", 2048, False, True, 0)):
            if src == "device":
                d_stage[: hi - lo].copy_(torch.from_numpy(canon[lo:hi]).cuda())
            d_view.fill_(0x3C)
            res = group.load(canon.size, leaf, bounds, rank_jobs, d_stage=d_stage, d_view=d_view,
                             h_stage=h if src == "host" else None, files=files if src == "files" else None,
                             read_threads=3, ring_slots=2, slot_bytes=1 << 12,
                             permutes=plan.permutes, view_bytes=plan.view_bytes, expected_root=want_root,
                             slab_bytes=256 if src == "host" else 0, window_bytes=window, peer_push=push,
                             all_gather=ag, push_nccl_share=share)
            got = d_view.cpu().numpy()[: plan.view_bytes]
            if res["root"] != want_root or got.size != want.size or not (got == want).all():
                log(f"rank {rank}: case {name} src={src} window={window} push={push} share={share} "
                    f"all_gather={ag} FAILED")
                failures += 1
    # Separate target tensors (bind_into, TCX_LOAD_TARGETS) over the NCCL exchange:
    # the Llama TP views with every tensor in its own allocation, guard bytes around.
    from tensorcast_b200.api import _TORCH_DTYPES
    from tensorcast_b200.binding import target_ranges, view_target_jobs
    canon, meta = oviews.canonical_bytes(llama)
    index = index_from_meta(meta, canon.size)
    sl = oviews.tp_slices(meta, world, rank)
    plan = plan_view(index, ViewSpec({n: [NarrowOp(*v)] for n, v in sl.items()}))
    guards, targets = [], {}
    for t in reversed(plan.tensors):
        g = torch.full((t.nbytes + 512,), 0xA5, dtype=torch.uint8, device="cuda")
        guards.append(g)
        targets[t.name] = g[256:256 + t.nbytes].view(_TORCH_DTYPES[t.dtype]).view(t.shape)
    base, ranges, vbytes = target_ranges(targets)
    jobs, _ = view_target_jobs(plan, targets, base)
    leaf = 1 << 16
    bounds = stage_bounds(canon.size, leaf, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    h = torch.empty(max(hi - lo, 1), dtype=torch.uint8, pin_memory=True)
    h.numpy()[: hi - lo] = canon[lo:hi]
    d_stage = torch.empty(max(hi - lo, 1), dtype=torch.uint8, device="cuda")
    want_root = oracle.tree_root(oracle.leaf_digests(canon, leaf))
    res = group.load(canon.size, leaf, bounds, gather(jobs), d_stage=d_stage, d_view=base,
                     h_stage=h, view_bytes=vbytes, expected_root=want_root, slab_bytes=256, window_bytes=4096,
                     target_ranges=ranges)
    want = oviews.materialize_view(canon, meta, sl, {}, None)
    same = all((targets[t.name].reshape(-1).view(torch.uint8).cpu().numpy() == want[t.offset:t.offset + t.nbytes]).all()
               for t in plan.tensors)
    guard_ok = all(bool((g[:256] == 0xA5).all()) and bool((g[-256:] == 0xA5).all()) for g in guards)
    if res["root"] != want_root or want.size != plan.view_bytes or not same or not guard_ok:
        log(f"rank {rank}: bind-into targets case FAILED")
        failures += 1
    return failures
