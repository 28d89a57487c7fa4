"""One rank of a multi-GPU collective-load parity check (launched by tests/test_multi_gpu.py
through torch.distributed.run; one process per GPU, NCCL).

Every rank builds the same seeded artifact bytes, plans its own view (tensor-parallel
narrows, a transpose, sometimes a subset), gathers every rank's view jobs, stages its
leaf-aligned share from pinned memory, and runs tcx_group_load. Its view must equal the
numpy oracle byte for byte and the Merkle root the CPU oracle's; exit status 0 = pass."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import datetime  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import oracle  # noqa: E402
from oracle import views as oviews  # noqa: E402
from tensorcast_b200.api import gather_rank_jobs  # noqa: E402
from tensorcast_b200.loader import Group, stage_bounds  # noqa: E402
from tensorcast_b200.synthetic import llama_shapes, tiny_llama  # noqa: E402
from tensorcast_b200.views import NarrowOp, TransposeOp, ViewSpec, plan_view  # noqa: E402
from viewtools import index_from_meta, random_tensors, random_view  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    group = Group.from_torch_distributed(local, timeout_ms=60_000)
    failures = 0
    try:
        cases = []
        # Llama-shaped TP-N views (+ one transposed o_proj) over a few MB.
        shapes = llama_shapes(tiny_llama(layers=4, hidden=256, heads=8, kv_heads=4, head_dim=32, ffn=512, vocab=1024))
        rng = np.random.default_rng(7)
        llama = {n: (rng.integers(0, 256, int(np.prod(s)) * 2, dtype=np.uint8), s, 2) for n, s in shapes.items()}
        cases.append(("llama", llama, 1 << 16))
        for seed in range(3):
            cases.append((f"random{seed}", random_tensors(100 + seed, n=24), int(np.random.default_rng(seed).choice([64, 512, 4096]))))
        for name, tensors, leaf in cases:
            canon, meta = oviews.canonical_bytes(tensors)
            index = index_from_meta(meta, canon.size)
            if name == "llama":
                sl = oviews.tp_slices(meta, world, rank)
                o = "model.layers.1.self_attn.o_proj.weight"
                sl.pop(o)
                spec = ViewSpec({n: [NarrowOp(*v)] for n, v in sl.items()})
                spec.tensors[o] = [TransposeOp(0, 1)]
                slices, transpose, subset = sl, {o: [(0, 1)]}, None
            else:
                slices, transpose, subset, spec = random_view(meta, np.random.default_rng(1000 * rank + leaf))
            plan = plan_view(index, spec, subset)
            rank_jobs = gather_rank_jobs(plan.jobs, world)
            bounds = stage_bounds(canon.size, leaf, world)
            lo, hi = bounds[rank], bounds[rank + 1]
            h = torch.empty(max(hi - lo, 1), dtype=torch.uint8, pin_memory=True)
            h.numpy()[: hi - lo] = canon[lo:hi]
            d_stage = torch.empty(max(hi - lo, 1), dtype=torch.uint8, device="cuda")
            d_view = torch.full((max(plan.view_bytes, 1),), 0x3C, dtype=torch.uint8, device="cuda")
            want_root = oracle.tree_root(oracle.leaf_digests(canon, leaf))
            for host, window, push, ag in ((True, 0, False, False), (False, 0, False, False),
                                           (False, 1000, False, False), (True, 4096, False, False),
                                           (True, 0, True, False), (False, 0, True, False),
                                           (True, 0, False, True), (False, 3000, False, True)):
                if not host:
                    d_stage[: hi - lo].copy_(torch.from_numpy(canon[lo:hi]).cuda())
                d_view.fill_(0x3C)
                res = group.load(canon.size, leaf, bounds, rank_jobs, d_stage=d_stage, d_view=d_view,
                                 h_stage=h if host else None, permutes=plan.permutes, view_bytes=plan.view_bytes,
                                 expected_root=want_root, slab_bytes=256, window_bytes=window, peer_push=push,
                                 all_gather=ag)
                want = oviews.materialize_view(canon, meta, slices, transpose, subset)
                got = d_view.cpu().numpy()[: plan.view_bytes]
                if res["root"] != want_root or got.size != want.size or not (got == want).all():
                    print(f"rank {rank}: case {name} host={host} window={window} push={push} all_gather={ag} FAILED",
                          flush=True)
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
        res = group.load(canon.size, leaf, bounds, gather_rank_jobs(jobs, world), d_stage=d_stage, d_view=base,
                         h_stage=h, view_bytes=vbytes, expected_root=want_root, slab_bytes=256, window_bytes=4096,
                         target_ranges=ranges)
        want = oviews.materialize_view(canon, meta, sl, {}, None)
        same = all((targets[t.name].reshape(-1).view(torch.uint8).cpu().numpy() == want[t.offset:t.offset + t.nbytes]).all()
                   for t in plan.tensors)
        guard_ok = all(bool((g[:256] == 0xA5).all()) and bool((g[-256:] == 0xA5).all()) for g in guards)
        if res["root"] != want_root or want.size != plan.view_bytes or not same or not guard_ok:
            print(f"rank {rank}: bind-into targets case FAILED", flush=True)
            failures += 1
        ok = torch.tensor([failures], device="cuda")
        dist.all_reduce(ok)
        failures = int(ok.item())
    finally:
        group.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(f"multi-GPU load parity: world={world} failures={failures}", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
