"""N>1 paths.

* GPU (marked gpu): tests/mp_load_worker.py on 2 (and, when present, 4) GPUs through
  torch.distributed.run + NCCL: every rank's view and the Merkle root against the oracles;
  tests/threads_load_worker.py: the same cases with the ranks as threads of one process
  (tcx_group_join, the reference daemon's model), plus the SDK path from those threads.
* CPU (gloo, world size 2): the host side of a collective load in two real processes:
  every rank's view jobs travel through gather_rank_jobs (all_gather_object), each rank
  computes its exchange schedule with the native planner, packs its share in numpy,
  the packed bytes travel over gloo send/recv, and each rank scatters what it received;
  both views must equal the numpy oracle's.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_collective_load_parity_multi_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "mp_load_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "failures=0" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_collective_load_parity_rank_threads(world):
    """The same loads with the ranks as threads of one process (tcx_group_join)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, os.path.join(HERE, "threads_load_worker.py"), str(world)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"world={world} failures=0 errors=0" in r.stdout


def test_in_process_job_gather_rounds():
    """The in-process all-gather the rank threads use for their view jobs: every thread gets
    every rank's bytes in rank order, over several rounds under one group id."""
    import threading
    from tensorcast_b200.api import _gather_in_process
    world, rounds = 3, 4
    got = {}

    def rank(r):
        for k in range(rounds):
            got[(r, k)] = _gather_in_process("g-test", world, r, f"{r}:{k}".encode())

    ts = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=30)
    for r in range(world):
        for k in range(rounds):
            assert got[(r, k)] == [f"{q}:{k}".encode() for q in range(world)]


def test_in_process_job_gather_times_out_without_peers():
    from tensorcast_b200.api import ArtifactError, _gather_in_process
    from tensorcast_b200 import api
    with pytest.raises(ArtifactError, match="timed out"):
        _gather_in_process("g-lonely", 2, 0, b"x", timeout_s=0.2)
    assert "g-lonely" not in api._RDV_TABLE


def _gloo_rank(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    from oracle import views as oviews
    from tensorcast_b200.api import gather_rank_jobs
    from tensorcast_b200.loader import plan_exchange, stage_bounds
    from tensorcast_b200.views import plan_view
    from viewtools import apply_jobs, apply_permutes, index_from_meta, random_tensors, random_view

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bad = 0
        for seed in range(4):
            canon, meta = oviews.canonical_bytes(random_tensors(50 + seed, n=16))
            index = index_from_meta(meta, canon.size)
            slices, transpose, subset, spec = random_view(meta, np.random.default_rng(rank * 97 + seed))
            plan = plan_view(index, spec, subset)
            rank_jobs = gather_rank_jobs(plan.jobs, world)
            leaf = 128
            bounds = stage_bounds(canon.size, leaf, world)
            x = plan_exchange(canon.size, leaf, bounds, rank_jobs, rank, plan.view_bytes)
            stage = canon[bounds[rank]:bounds[rank + 1]]
            send = np.zeros(int(x["send_offsets"][-1]), np.uint8)
            apply_jobs(stage, send, x["pack"])
            view = np.full(plan.view_bytes, 0xEE, np.uint8)
            for off, ln in x["gaps"]:
                view[int(off): int(off) + int(ln)] = 0
            apply_jobs(stage, view, x["local"])
            recv = np.zeros(int(x["recv_offsets"][-1]), np.uint8)
            peer = 1 - rank
            s0, s1 = int(x["send_offsets"][peer]), int(x["send_offsets"][peer + 1])
            rbuf = torch.zeros(int(x["recv_counts"][peer]), dtype=torch.uint8)
            reqs = []
            if s1 > s0:
                reqs.append(dist.isend(torch.from_numpy(send[s0:s1].copy()), peer))
            if rbuf.numel():
                reqs.append(dist.irecv(rbuf, peer))
            for r in reqs:
                r.wait()
            data = rbuf.numpy()
            if x["direct"][peer]:
                o = int(x["recv_view_off"][peer])
                view[o:o + data.size] = data
            else:
                o = int(x["recv_offsets"][peer])
                recv[o:o + data.size] = data
            apply_jobs(recv, view, x["scatter"])
            apply_permutes(view, plan.permutes)
            want = oviews.materialize_view(canon, meta, slices, transpose, subset)
            bad += int(not (view.size == want.size and (view == want).all()))
        q.put((rank, bad))
    finally:
        dist.destroy_process_group()


def test_collective_protocol_gloo_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(0, 0), (1, 0)], results
