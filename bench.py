#!/usr/bin/env python
"""Benchmark of the B200 realization hot path (TensorCast from_disk load + GPU SHA-256).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tcx|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Workload (the single-GPU load benchmark at N=1, its tensor-parallel form at N>1): a synthetic
Llama-3-8B-shaped bf16 safetensors artifact (seed 1, 16 060 522 496 payload bytes) in
tmpfs. Each rank stages its leaf-aligned 1/N of the canonical byte space, hashes the
leaves it staged (SHA-256, explicit 4 MiB leaves), the ranks exchange over NVLink the
bytes of each other's tensor-parallel view (N=1: the identity view), and every rank
ends with its view and the verified Merkle root of the whole artifact.

One JSON line on rank 0:
* value  - realized GB/s (artifact bytes / step) with the staged bytes already in HBM
           (device-timed, max over ranks);
* e2e    - the same metric through tcx_group_load from pinned host memory (H2D, hashing,
           exchange, view, 32-byte root read-back all inside the timed step);
* roofline - the SHA-256 leaf kernel against the measured compute bound of the
           compression (register-only probe) and the measured HBM bandwidth;
* cpu_baseline - the reference's CPU path (pread + OpenSSL SHA-256 per leaf + Merkle
           tree, single thread, source_hash.cc:19-61) restated in oracle/, on a sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Realized GB/s into 1/2/4/8 B200 (SHA-256 verified); GPU SHA-256 GB/s/GPU"
LEAF = 4 << 20
SEEDS = {"llama3-8b": 1, "llama3-70b": 2}  # the 8B and 70B benchmark artifacts


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["tcx", "reference"], default="tcx")
    ap.add_argument("--dir", default=os.environ.get("TCX_BENCH_DIR", "/dev/shm/tcx_bench"))
    ap.add_argument("--model", choices=["llama3-8b", "llama3-70b"], default="llama3-8b")
    ap.add_argument("--leaf", type=int, default=LEAF)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU baseline sample time")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip timing the reference's own GPU kernel")
    ap.add_argument("--no-c4", action="store_true", help="at N>1, skip the Llama-3-70B (config 4) leg")
    ap.add_argument("--c4-exchange", choices=["nccl", "push"], default="push",
                    help="shard exchange of the config-4 leg (push: copy-engine copies into the peers' views, "
                         "measured faster than NCCL send/recv on the 70B TP-2 load)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the extra legs after the main line (paged KV; bind_into at N>1; disk-dir hash at N=1)")
    ap.add_argument("--exchange", choices=["auto", "push", "nccl", "allgather"], default="auto",
                    help="N>1 shard exchange: push over peer memory (copy-engine copies into the peers' views "
                         "over NVLink) or NCCL send/recv of packed windows; auto = push; allgather = windowed "
                         "broadcast of every rank's staged bytes to all ranks (every rank sees every byte)")
    ap.add_argument("--push-nccl-share", default="auto",
                    help="with the push exchange, the share (0..1) of every pair's bytes sent by NCCL "
                         "send/recv beside the copy-engine copies; auto = the share measured best for the "
                         "number of ranks on the exchange-bound 70B leg, none on the hash-bound 8B load")
    ap.add_argument("--stage", choices=["mapped", "pinned"], default="pinned",
                    help="host staging of each rank's range: the tmpfs file pages mapped and page-locked in place "
                         "(no second host copy), or a pinned copy read with parallel preads")
    ap.add_argument("--workload", choices=["artifact", "kv", "disk-hash"], default="artifact",
                    help="artifact: the collective from-disk load (default); kv: the paged-KV benchmark, paged KV "
                         "gather + per-sequence hash, 8 sequence shards dealt to the ranks; disk-hash: "
                         "compute_data_multihash_from_disk_dir of the artifact's directory on one GPU, against "
                         "the reference's single-core CPU path")
    ap.add_argument("--kv-pages", type=int, default=65536,
                    help="pool pages of the paged-KV workload (config 5: 65536); smaller pools make the few-GB "
                         "case used for ncu captures")
    ap.add_argument("--copy-only", metavar="ROWS:COLS:TP",
                    help="only time the view kernels on a bf16 [ROWS, COLS] tensor: the dim-0 and dim-1 "
                         "tensor-parallel shards of rank 0 of TP (copy jobs) and a full transpose")
    ap.add_argument("--hash-only", metavar="BYTES:LEAF",
                    help="only time the SHA-256 leaf kernel on BYTES of seeded device data (e.g. 512M:128K); "
                         "the small case used for ncu captures")
    return ap.parse_args()


def exchange_mode(args) -> str:
    # auto: the copy-engine push for both artifacts (with the local extraction on its own
    # stream it measured faster than NCCL send/recv on the 70B TP-2 load: 127 against 154 ms)
    return "push" if args.exchange == "auto" else args.exchange


# Share of every pair's bytes that the push exchange sends over NCCL, by number of ranks, for
# loads whose exchange is the long leg (the 70B TP-N load at 2 and 4 ranks). Measured on B200
# (70B TP-N, device-resident, mean of 3 loads, max over ranks):
#  * 2 ranks: the copy engines alone already deliver about the peer-copy rate (transfer 47.9 ms;
#    a 20 / 35 / 50 % NCCL share 48.5 / 49.7 / 54.1 ms);
#  * 4 ranks: the copy engines reach about 390 GB/s per GPU in the all-to-all (transfer 78.2 ms,
#    step 83.1 ms); a 30 % share 63.9 ms (step 70.5 ms, now hash-bound), 45 % 65.1, 60 % 70.6.
# Where the leaf hash is the long leg (the 8B load at every N) the split only takes SM time from
# the hash (70.3 against 69.0 ms at 4 ranks), so those loads use none.
AUTO_PUSH_NCCL_SHARE_EXCHANGE_BOUND = {2: 0.0, 4: 0.3}


def push_share(args, world: int, exchange_bound: bool = False) -> float:
    if args.push_nccl_share != "auto":
        return min(1.0, max(0.0, float(args.push_nccl_share)))
    return AUTO_PUSH_NCCL_SHARE_EXCHANGE_BOUND.get(world, 0.0) if exchange_bound else 0.0


def _size(x: str) -> int:
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    return int(float(x[:-1]) * mult[x[-1].upper()]) if x[-1].upper() in mult else int(x)


def run_hash_only(args) -> None:
    import torch
    import tensorcast_b200 as tcx
    nbytes, leaf = (_size(v) for v in args.hash_only.split(":"))
    g = torch.Generator(device="cuda").manual_seed(0)
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda", generator=g)
    n = (nbytes + leaf - 1) // leaf
    out = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        tcx.sha256_leaves(src, leaf, out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        tcx.sha256_leaves(src, leaf, out)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"mode": "hash-only", "bytes": nbytes, "leaf": leaf, "leaves": n, "ms": round(ms, 3),
                      "gbs": round(nbytes / ms / 1e6, 2)}), flush=True)


def run_copy_only(args) -> None:
    """HBM-bound view kernels alone: algorithmic bytes = bytes read + bytes written."""
    import ctypes
    import numpy as np
    import torch
    from tensorcast_b200 import _native
    from tensorcast_b200.views import JOB_DTYPE
    rows, cols, tp = (int(v) for v in args.copy_only.split(":"))
    es = 2
    g = torch.Generator(device="cuda").manual_seed(0)
    src = torch.randint(0, 256, (rows * cols * es,), dtype=torch.uint8, device="cuda", generator=g)
    L = _native.lib()
    s = torch.cuda.current_stream()
    res = {"mode": "copy-only", "rows": rows, "cols": cols, "tp": tp}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(max(args.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(args.steps):
            fn()
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / args.steps

    for name, job in (("dim0_shard", (0, 0, cols * es * rows // tp, cols * es * rows // tp, cols * es * rows // tp, 1)),
                      ("dim1_shard", (0, 0, cols * es, cols * es // tp, cols * es // tp, rows))):
        jobs = torch.from_numpy(np.array([job], dtype=JOB_DTYPE).view(np.uint8)).cuda()
        nbytes = job[4] * job[5]
        dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        sb = int(L.tcx_copy_jobs_scratch_bytes(1))
        scratch = torch.empty(sb, dtype=torch.uint8, device="cuda")
        ms = timed(lambda: _native.call("tcx_copy_jobs", src.data_ptr(), dst.data_ptr(), jobs.data_ptr(), 1,
                                        scratch.data_ptr(), sb, s.cuda_stream))
        res[name] = {"bytes_moved": 2 * nbytes, "ms": round(ms, 4), "gbs": round(2 * nbytes / ms / 1e6, 1)}
    out = torch.empty_like(src)
    # the same bytes as [rows, cols] bf16, [rows, 2*cols] 1-byte and [rows, cols/2] 4-byte elements
    for key, esize, ncols in (("transpose", es, cols), ("transpose_1byte", 1, cols * es),
                              ("transpose_4byte", 4, cols * es // 4)):
        pj = _native.PermuteJob(0, 0, esize, 2)
        pj.shape[0], pj.shape[1], pj.perm[0], pj.perm[1] = rows, ncols, 1, 0
        ms = timed(lambda: _native.call("tcx_permute", src.data_ptr(), out.data_ptr(), ctypes.byref(pj), s.cuda_stream))
        res[key] = {"bytes_moved": 2 * src.numel(), "ms": round(ms, 4), "gbs": round(2 * src.numel() / ms / 1e6, 1)}
    res["hbm_gbs"] = measured_hbm()
    print(json.dumps(res), flush=True)


def log(*a):
    print("[bench]", *a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# Artifact
# ---------------------------------------------------------------------------
def artifact_path(args) -> str:
    return os.path.join(args.dir, f"{args.model}-seed{SEEDS[args.model]}.safetensors")


TRANSPOSED_O_PROJ = "model.layers.0.self_attn.o_proj.weight"


def model_shapes(model: str) -> dict:
    """Benchmark shapes: Llama-3-8B (single-GPU and TP-8 loads) or Llama-3-70B (the 70B collective load, whose layer-0 o_proj is
    stored as [in, out] and read through a transpose view)."""
    from tensorcast_b200.synthetic import LLAMA3_70B, LLAMA3_8B, llama_shapes
    if model == "llama3-8b":
        return llama_shapes(LLAMA3_8B)
    return llama_shapes(LLAMA3_70B, transposed=(TRANSPOSED_O_PROJ,))


def ensure_artifact(args, rank: int, local_rank: int, world: int = 1) -> str:
    """Writes the artifact once (marker file): rank 0 alone, or every rank its share of the
    tensors when several ranks start together; the other ranks wait for the marker."""
    from tensorcast_b200.synthetic import artifact_bytes, write_safetensors, write_safetensors_parallel
    shapes = model_shapes(args.model)
    path = artifact_path(args)
    marker = path + ".done"
    if not os.path.exists(marker) and (rank == 0 or world > 1):
        import torch
        os.makedirs(args.dir, exist_ok=True)
        if rank == 0:
            need = artifact_bytes(shapes) + (64 << 20)
            st = os.statvfs(args.dir)
            if st.f_bavail * st.f_frsize < need:
                raise SystemExit(f"not enough space in {args.dir} for the {need / 1e9:.1f} GB artifact "
                                 f"(set TCX_BENCH_DIR)")
        t0 = time.time()
        dev = f"cuda:{local_rank}" if torch.cuda.is_available() else "cpu"
        if world > 1:
            info = write_safetensors_parallel(path, shapes, SEEDS[args.model], world, rank, device=dev)
        else:
            info = write_safetensors(path, shapes, SEEDS[args.model], device=dev)
        if rank == 0:
            with open(marker, "w") as f:
                json.dump(info, f)
            log(f"wrote {info['total_bytes'] / 1e9:.2f} GB artifact in {time.time() - t0:.1f}s ({dev}, "
                f"{world} writer(s))")
    t0 = time.time()
    while not os.path.exists(marker):
        if time.time() - t0 > 900:
            raise SystemExit("timed out waiting for rank 0 to write the artifact")
        time.sleep(0.5)
    return path


def tp_slices(index, world: int, rank: int) -> dict:
    """Tensor-parallel sharding of the benchmark: q/k/v/gate/up, embed and lm_head along dim 0; o/down along dim 1."""
    out = {}
    for name, e in index.entries.items():
        if any(k in name for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "embed_tokens", "lm_head")):
            d = 0
        elif any(k in name for k in ("o_proj", "down_proj")):
            d = 1
        else:
            continue
        ln = e.shape[d] // world
        out[name] = (d, slice(rank * ln, (rank + 1) * ln))
    return out


# ---------------------------------------------------------------------------
# Clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device: int):
        self.device, self.proc, self.rows = device, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + ",".join(self.FIELDS), "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(self.FIELDS):
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower().startswith("active")})
        pw = [float(r[3]) for r in self.rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU hashing path, restated in oracle/)
# ---------------------------------------------------------------------------
def cpu_reference_sample(path: str, payload_off: int, total: int, leaf: int, target_s: float,
                         max_bytes: int | None = None, threads: int = 1) -> dict:
    """pread of a leaf-aligned sample of the canonical bytes + OpenSSL SHA-256 per leaf
    (source_hash.cc:38-58) + Merkle tree + multihash, timed on the host. threads=1 is the
    reference's own single-core path; more threads spread the preads and the leaves over
    that many host threads (the same per-leaf work)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import oracle

    def read(buf, nbytes):
        mv = memoryview(buf)
        fd = os.open(path, os.O_RDONLY)
        try:
            def part(lo, hi):
                got = lo
                while got < hi:
                    n = os.preadv(fd, [mv[got:hi]], payload_off + got)
                    if n <= 0:
                        raise IOError("short read")
                    got += n
            if threads <= 1:
                part(0, nbytes)
            else:
                step = max(leaf, (nbytes // threads + leaf - 1) // leaf * leaf)
                with ThreadPoolExecutor(threads) as ex:
                    list(ex.map(lambda lo: part(lo, min(nbytes, lo + step)), range(0, nbytes, step)))
        finally:
            os.close(fd)

    def run(nbytes):
        buf = np.empty(nbytes, np.uint8)
        t0 = time.perf_counter()
        read(buf, nbytes)
        d = oracle.leaf_digests(buf, leaf, openssl=True, threads=threads)
        oracle.multihash(oracle.tree_root(d))
        return time.perf_counter() - t0

    probe = min(total, 64 * leaf * max(1, threads))
    dt = run(probe)
    rate = probe / dt
    nbytes = min(total, max(probe, int(rate * target_s) // leaf * leaf))
    if max_bytes:
        nbytes = min(nbytes, max_bytes)
    dt = run(nbytes)
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"first {nbytes // leaf} leaves ({nbytes / 1e9:.2f} GB) of the artifact: pread from tmpfs + "
                      f"OpenSSL EVP SHA-256 per {leaf >> 20} MiB leaf + Merkle tree, {threads} thread(s)",
            "seconds": round(dt, 2), "host_nproc": os.cpu_count()}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = ensure_artifact(args, 0, int(os.environ.get("LOCAL_RANK", "0")))
    from tensorcast_b200.artifact import build_canonical_index, build_source_index, canonical_segments
    index = build_canonical_index(build_source_index(path))
    segs = canonical_segments(index, 0, index.total_bytes)
    payload_off = segs[0][1]
    if len(segs) != 1:
        raise SystemExit("canonical bytes are not one contiguous payload range")
    per_step = max(args.cpu_seconds / max(args.steps, 1), 2.0)
    threads = max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1))
    cap = 8 << 30  # host memory for one sample
    for _ in range(args.warmup):
        cpu_reference_sample(path, payload_off, index.total_bytes, args.leaf, min(per_step, 2.0), cap, threads)
    vals = [cpu_reference_sample(path, payload_off, index.total_bytes, args.leaf, per_step, cap, threads)
            for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in vals)
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(statistics.median(x["seconds"] for x in vals) * 1e3, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"{args.model} safetensors from tmpfs, SHA-256 {args.leaf >> 20} MiB leaves, "
                                   f"CPU realization sample (reference CPU hashing path on {threads} host threads)",
                       "artifact_bytes": index.total_bytes, "leaf_bytes": args.leaf},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": vals[0]["sample"]},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# tcx arm
# ---------------------------------------------------------------------------
def main() -> None:
    args = parse_args()
    if args.hash_only:
        run_hash_only(args)
        return
    if args.copy_only:
        run_copy_only(args)
        return
    if args.workload == "kv":
        run_kv(args)
        return
    if args.workload == "disk-hash":
        run_disk_hash(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"note: WORLD_SIZE={world} differs from --gpus {args.gpus}; using WORLD_SIZE")
    torch.cuda.set_device(local)
    try:
        from tensorcast_b200.loader import bind_device_cpus
        n_local_cpus = bind_device_cpus(local)
    except Exception as e:  # noqa: BLE001
        n_local_cpus = 0
        log(f"CPU binding unavailable: {e}")
    path = ensure_artifact(args, rank, local, world)
    if world > 1:
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    import tensorcast_b200 as tcx
    from tensorcast_b200 import _native
    from tensorcast_b200.artifact import build_canonical_index, build_source_index, canonical_segments, pad_ranges
    from tensorcast_b200.loader import Group, read_segments, stage_bounds
    from tensorcast_b200.views import build_view_spec, plan_view

    index = build_canonical_index(build_source_index(path))
    T, L = index.total_bytes, args.leaf
    bounds = stage_bounds(T, L, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    whole = canonical_segments(index, 0, T)
    canonical_is_payload = len(whole) == 1 and whole[0][3] == T
    # Every rank's view: identity at N=1, the tensor-parallel shards otherwise.
    plans = []
    transposed = TRANSPOSED_O_PROJ if args.model == "llama3-70b" else None
    for r in range(world):
        slices = {} if world == 1 else tp_slices(index, world, r)
        tr = None
        if transposed:
            slices.pop(transposed, None)
            tr = {transposed: [(0, 1)]}
        spec = None if not slices and not tr else build_view_spec(index, slices=slices, transpose=tr)
        plans.append(plan_view(index, spec))
    mine = plans[rank]
    rank_jobs = [p.jobs for p in plans]

    # This rank's staged range as file segments: the from-file loads read them inside the
    # timed step (tcx_group_load_files). Reader threads: the CPUs this rank may use,
    # shared evenly by the ranks of this host.
    files_mine = canonical_segments(index, lo, hi)
    affinity = tuple(sorted(os.sched_getaffinity(0)))
    sharing = 1
    if world > 1:
        import socket
        everyone = [None] * world
        dist.all_gather_object(everyone, (socket.gethostname(), affinity))
        sharing = sum(1 for x in everyone if x == (socket.gethostname(), affinity))
    read_threads = max(2, min(32, len(affinity) // sharing))
    # Staged bytes in page-locked host memory as well (setup), for the from-pinned-memory
    # form of e2e and the host-to-device bound: the file's own tmpfs pages mapped and
    # registered in place when asked, else a pinned copy assembled with parallel preads.
    from tensorcast_b200.loader import FileMapping
    stage_kind, h_stage, t_pin = "pinned copy", None, 0.0
    t0 = time.perf_counter()
    if args.stage == "mapped" and canonical_is_payload:
        try:
            h_stage = FileMapping(path, whole[0][1] + lo, hi - lo, register=True)
            stage_kind = "mapped tmpfs pages, page-locked in place"
        except Exception as e:  # noqa: BLE001
            log(f"file registration unavailable ({e}); staging through a pinned copy")
    t_map = time.perf_counter() - t0
    if h_stage is None:
        t0 = time.perf_counter()
        h_stage = torch.empty(hi - lo, dtype=torch.uint8, pin_memory=True)
        t_pin = time.perf_counter() - t0
        read_segments(files_mine, h_stage.data_ptr(), threads=read_threads)  # first touch of the pinned pages
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        read_segments(files_mine, h_stage.data_ptr(), threads=read_threads)
        t_read = time.perf_counter() - t0
        for off, ln in pad_ranges(index, lo, hi):
            h_stage[off:off + ln].zero_()
    else:
        t_read = t_map
    d_stage = torch.empty(hi - lo, dtype=torch.uint8, device="cuda")
    identity = world == 1 and mine.is_identity
    d_view = d_stage if identity else torch.empty(max(mine.view_bytes, 1), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    group = Group.from_torch_distributed(local) if world > 1 else Group(1, 0, local)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def load(host: bool, expected=None, from_files: bool = False):
        return group.load(T, L, bounds, rank_jobs, d_stage=d_stage, d_view=d_view,
                          h_stage=h_stage if host and not from_files else None,
                          files=files_mine if from_files else None, read_threads=read_threads,
                          permutes=mine.permutes, view_bytes=mine.view_bytes, expected_root=expected,
                          peer_push=exchange_mode(args) == "push" and world > 1,
                          push_nccl_share=push_share(args, world) if exchange_mode(args) == "push" else 0.0,
                          all_gather=exchange_mode(args) == "allgather" and world > 1)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # First load (from the files, so it also fills d_stage for the device-resident steps)
    # establishes the root; rank 0 checks it against the CPU oracle over the whole file.
    first = load(True, from_files=True)
    root = first["root"]
    parity = {}
    if rank == 0:
        from oracle import oracle
        mm = np.memmap(path, dtype=np.uint8, mode="r", offset=whole[0][1], shape=(T,)) if canonical_is_payload else None
        if mm is not None:
            t0 = time.perf_counter()
            threads = os.cpu_count() or 8
            cpu_root = oracle.tree_root(oracle.leaf_digests(mm, L, openssl=True, threads=threads))
            parity = {"root_matches_cpu_oracle": cpu_root == root, "oracle_threads": threads,
                      "oracle_seconds": round(time.perf_counter() - t0, 1), "multihash": first["multihash"]}
            if cpu_root != root:
                raise SystemExit(f"PARITY FAILURE: GPU root {root.hex()} != CPU oracle {cpu_root.hex()}")
    # Views: every byte of every rank's view against numpy slicing of the file.
    view_ok, view_checked, view_tensors = verify_view_full(path, index, mine, d_view, world, rank, transposed)
    straddling = straddling_tensors(index, bounds)
    if world > 1:
        ok = torch.tensor([1 if view_ok else 0, view_checked, view_tensors], dtype=torch.float64, device="cuda")
        mn = ok.clone()
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        dist.all_reduce(ok, op=dist.ReduceOp.SUM)
        view_ok, view_checked, view_tensors = bool(mn[0].item()), int(ok[1].item()), int(ok[2].item())
    if not view_ok:
        raise SystemExit("PARITY FAILURE: view bytes differ from numpy slicing of the artifact")

    # Hash-kernel roofline (device-resident, alone, CUDA events on the launching stream).
    hk = hash_kernel_roofline(d_stage, hi - lo, L, rank)
    # The reference's own GPU kernel on the same bytes (rank 0 of a one-GPU run).
    ref_gpu = reference_gpu_kernel(d_stage, hi - lo, L, hk) if world == 1 and not args.no_ref_gpu else None

    # value: device-resident loads.
    for _ in range(args.warmup):
        load(False, root)
    with ClockSampler(local) as clk:
        barrier()
        n0 = _native.lib().tcx_kernel_launch_count()
        w0 = time.perf_counter()
        steps = [load(False, root) for _ in range(args.steps)]
        barrier()
        wall = (time.perf_counter() - w0) / args.steps * 1e3
        launches = _native.lib().tcx_kernel_launch_count() - n0
    dev_ms = [r["total_ms"] for r in steps]
    ms = max_over_ranks(statistics.mean(dev_ms))
    hash_ms = max_over_ranks(statistics.mean(r["hash_ms"] for r in steps))
    exch_ms = max_over_ranks(statistics.mean(r["exchange_ms"] for r in steps))
    xfer_ms = max_over_ranks(statistics.mean(r["transfer_ms"] for r in steps))
    wall = max_over_ranks(wall)

    # e2e (headline): from the files through tcx_group_load_files -- preads into the
    # pinned ring, H2D, hash, exchange, view and the 32-byte root read back, all inside
    # each step -- timed with events on this stream around the K steps, max over ranks.
    cur = torch.cuda.current_stream()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.warmup):
        load(True, root, from_files=True)
    barrier()
    n0 = _native.lib().tcx_kernel_launch_count()
    w0 = time.perf_counter()
    f0.record(cur)
    file_res = [load(True, root, from_files=True) for _ in range(args.steps)]
    f1.record(cur)
    f1.synchronize()
    file_wall = (time.perf_counter() - w0) / args.steps * 1e3
    barrier()
    file_launches = _native.lib().tcx_kernel_launch_count() - n0
    file_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps)
    file_wall = max_over_ranks(file_wall)
    file_read_ms = max_over_ranks(statistics.mean(r["stage_read_ms"] for r in file_res))
    file_h2d_ms = max_over_ranks(statistics.mean(r["h2d_ms"] for r in file_res))

    # e2e from pinned host memory (the staged range already read into pinned memory).
    for _ in range(args.warmup):
        load(True, root)
    barrier()
    n0 = _native.lib().tcx_kernel_launch_count()
    e2e_res = [load(True, root) for _ in range(args.steps)]
    barrier()
    e2e_launches = _native.lib().tcx_kernel_launch_count() - n0
    e2e_ms = max_over_ranks(statistics.mean(r["total_ms"] for r in e2e_res))
    h2d_ms = max_over_ranks(statistics.mean(r["h2d_ms"] for r in e2e_res))
    peer = max_over_ranks(float(e2e_res[-1]["peer_recv_bytes"]))
    read_gbs = None
    if stage_kind == "pinned copy" and t_read > 0:
        read_gbs = round(T / max_over_ranks(t_read) / 1e9, 2)

    # e2e bound: this run's own host-to-device rate, a plain pinned -> device copy of each
    # rank's staged range on all ranks at once (the same bytes d_stage already holds).
    h2d_peak = None
    h2d_solo, read_solo = [0.0] * world, [0.0] * world
    if isinstance(h_stage, torch.Tensor):
        n = min(hi - lo, 4 << 30)
        s = torch.cuda.current_stream()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = 0.0
        for _ in range(3):
            barrier()
            c0.record(s)
            d_stage[:n].copy_(h_stage[:n], non_blocking=True)
            c1.record(s)
            c1.synchronize()
            t = max_over_ranks(c0.elapsed_time(c1))
            best = max(best, n * world / t / 1e6)
        h2d_peak = round(best, 2)
        if world > 1:
            # Each GPU alone (the others idle at a barrier), to tell a per-link limit from a
            # shared host-side one, and the same for the preads of each rank's range.
            for r in range(world):
                barrier()
                if r == rank:
                    c0.record(s)
                    d_stage[:n].copy_(h_stage[:n], non_blocking=True)
                    c1.record(s)
                    c1.synchronize()
                    h2d_solo[r] = n / c0.elapsed_time(c1) / 1e6
                    t0 = time.perf_counter()
                    read_segments(files_mine, h_stage.data_ptr(), threads=read_threads)
                    read_solo[r] = (hi - lo) / (time.perf_counter() - t0) / 1e9
            barrier()
            sv = torch.tensor(h2d_solo + read_solo, dtype=torch.float64, device="cuda")
            dist.all_reduce(sv, op=dist.ReduceOp.SUM)
            h2d_solo = [round(float(x), 2) for x in sv[:world].tolist()]
            read_solo = [round(float(x), 2) for x in sv[world:].tolist()]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and canonical_is_payload:
        cpu = cpu_reference_sample(path, whole[0][1], T, L, args.cpu_seconds)

    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(T / ms / 1e6, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
            "config": {
                "workload": (f"{args.model}-shaped bf16 safetensors (seed {SEEDS[args.model]}), {T} B, identity view"
                             if world == 1 else
                             f"{args.model}-shaped bf16 safetensors (seed {SEEDS[args.model]}), {T} B, TP-{world} views "
                             f"(q/k/v/gate/up/embed/lm_head dim 0, o/down dim 1)"
                             + (f"; {transposed} stored [in, out] and read whole through a transpose view"
                                if transposed else "")),
                "artifact_bytes": T, "leaf_bytes": L, "leaves": first["leaves"],
                "exchange": {"push": "push over peer memory (copy-engine 2-D copies into the peers' views over NVLink)",
                             "nccl": "NCCL send/recv of packed windows",
                             "allgather": "windowed all-gather (ncclBroadcast per root) + extraction"}[exchange_mode(args)]
                if world > 1 else "none",
                "view_bytes_per_rank": mine.view_bytes, "parallelism": f"tp{world}",
                "l2": "inputs (staged bytes) far larger than the 126 MB L2; no flush needed",
                "timing": "device events per step (tcx_group_load), mean over steps, max over ranks"},
            "sha256_gbs_per_gpu": hk["achieved"],
            "roofline": hk,
            "e2e": {"value": round(T / file_ms / 1e6, 2), "unit": "GB/s", "ms_per_step": round(file_ms, 3),
                    "from": f"the safetensors file in tmpfs (page-cache resident): {read_threads} reader threads per "
                            "rank pread leaf pieces into small pinned buffers and queue each group's H2D copy at "
                            "once; streamed hash, exchange, view, 32-byte root read back, all inside each step "
                            "(tcx_group_load_files)",
                    "h2d_bytes_per_step": T, "d2h_bytes_per_step": 32 * world,
                    "stage_read_ms": round(file_read_ms, 3), "h2d_ms": round(file_h2d_ms, 3),
                    "wall_ms_per_step": round(file_wall, 3), "gpu_launches": int(file_launches),
                    "read_threads_per_rank": read_threads,
                    "bound": {"kind": "aggregate host-to-device copy (and the host pread rate beside it)",
                              "peak_gbs": h2d_peak,
                              "frac": round(T / file_ms / 1e6 / h2d_peak, 4) if h2d_peak else None,
                              "read_gbs": read_gbs,
                              "topology": gpu_topology(world) if world > 1 else None,
                              "h2d_gbs_per_gpu_alone": h2d_solo if world > 1 else None,
                              "read_gbs_per_rank_alone": read_solo if world > 1 else None,
                              "h2d_gbs_per_gpu_all_at_once": round(h2d_peak / world, 2) if h2d_peak else None,
                              "read_gbs_per_rank_all_at_once": round(read_gbs / world, 2) if read_gbs else None,
                              "frac_of_min_h2d_read": round(T / file_ms / 1e6 / min(h2d_peak, read_gbs), 4)
                              if h2d_peak and read_gbs else None,
                              "source": "measured in this run: pinned -> device copy of each rank's staged range, "
                                        "all ranks at once, best of 3, max over ranks; read_gbs: parallel preads of "
                                        "each rank's range from the file into pinned memory (same threads), "
                                        "all ranks at once"},
                    "from_pinned": {
                        "value": round(T / e2e_ms / 1e6, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                        "h2d_ms": round(h2d_ms, 3), "h2d_gbs_per_gpu": round((hi - lo) / h2d_ms / 1e6, 2),
                        "gpu_launches": int(e2e_launches),
                        "frac_of_h2d": round(T / e2e_ms / 1e6 / h2d_peak, 4) if h2d_peak else None,
                        "note": "the staged range already in pinned host memory (read before the step)"}},
            "gpu_launches": int(launches),
            "wall_ms_per_step": round(wall, 3),
            "phases_ms": {"hash": round(hash_ms, 3), "exchange_and_view": round(exch_ms, 3),
                          "note": "device-resident steps; hashing and the exchange run concurrently"},
            "peer_recv_bytes_per_rank": int(peer),
            "setup": {"host_stage": stage_kind, "stage_prep_s": round(t_read + t_pin, 2),
                      "host_nproc": os.cpu_count(), "affinity_cpus": len(os.sched_getaffinity(0)),
                      "canonical_is_payload": canonical_is_payload, "local_cpus_bound": n_local_cpus},
            "parity": dict(parity, view_full_ok=view_ok, view_bytes_checked=int(view_checked),
                           view_tensors_checked=int(view_tensors), tensors_straddling_stage_bounds=straddling,
                           view_check="every byte of every rank's view == numpy slicing of the file"),
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if ref_gpu is not None:
            line["reference_gpu_kernel"] = ref_gpu
        if world > 1:
            # The shard exchange of the device-resident steps (it runs beside the hash).
            line["exchange"] = exchange_summary(exchange_mode(args), peer, exch_ms, xfer_ms, push_share(args, world))

    # Extra legs (driver-visible evidence of the other benchmark rows), after the main
    # workload's buffers are released: paged KV (config 5) on every N, the collective
    # bind_into at N > 1, the disk-directory hash at N = 1.
    extras = {}
    if not args.no_extras:
        del d_view, d_stage, h_stage, first, file_res, e2e_res, steps
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        barrier()
        torch._C._host_emptyCache()  # release the pinned staging copy to the host
        # The main group goes first (all ranks at once): it also closes its peer-view
        # mappings, so the views freed above are returned to their devices.
        group.close()
        torch.cuda.empty_cache()
        def leg(name, fn):
            # A leg that raises is recorded and the rest still run (the main line is
            # printed in any case); device memory left by it is released first.
            try:
                extras[name] = fn()
            except Exception as e:  # noqa: BLE001
                extras[name] = {"error": f"{type(e).__name__}: {e}"[:400]}
                log(f"{name} leg failed: {e}")
            torch.cuda.synchronize()
            torch.cuda.empty_cache()

        if world > 1:
            leg("bind_into", lambda: bind_into_check(args, path, index, world, rank, local))
            if args.model == "llama3-8b" and not args.no_c4:
                def c4():
                    g4 = Group.from_torch_distributed(local)
                    try:
                        return c4_leg(args, g4, world, rank, local, read_threads, args.c4_exchange)
                    finally:
                        g4.close()
                leg("c4", c4)
        leg("kv", lambda: kv_measure(args, world, rank, local))
        if world == 1:
            leg("disk_hash", lambda: measure_disk_hash(args, min(args.steps, 5), 1))
    bad = []
    if rank == 0:
        line.update({k: v for k, v in extras.items() if v is not None})
        print(json.dumps(line), flush=True)
        bad = [k for k, v in extras.items() if isinstance(v, dict) and
               (v.get("ok") is False or v.get("matches_cpu_oracle") is False or
                v.get("parity", {}).get("first_and_last_shard_sequences_match_oracle") is False)]
    group.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if bad:
        raise SystemExit(f"PARITY FAILURE in {bad}")


def kv_measure(args, world: int, rank: int, local: int):
    """The paged-KV benchmark: 64 planes (32 layers x K/V) of 65536 pages [16, 8, 128] bf16 (seed 3),
    sequences of 64-4096 tokens drawn in order until the pool is full, pages at a seeded
    permutation; the sequences are dealt to 8 shards and rank r processes shards r, r+N, ...
    (each shard's pool holds its own pages in their global random order). A step gathers
    every sequence of the rank's shards contiguously and hashes each with 2 MiB leaves into
    a per-sequence root; value = gathered bytes of all ranks / step time (max over ranks)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from tensorcast_b200 import _native, kvcache
    from oracle import kv as okv

    w = kvcache.workload(seed=3, pool_pages=getattr(args, "kv_pages", 65536))
    shards = [w.shard(8, k, local_pool=True) for k in range(rank, 8, world)]
    pools, runners = [], []
    for k, sh in zip(range(rank, 8, world), shards):
        pools.append(kvcache.make_pool(sh, seed=3 * 100 + k))
    # Output buffers reused by the rank's shards in turn: two when they fit, so that the
    # gather and the (chain-latency bound) hash of one shard overlap with the next
    # shard's on a second stream.
    out_max = max(kvcache.plan(sh).out_bytes for sh in shards)
    torch.cuda.synchronize()
    free, _ = torch.cuda.mem_get_info()
    n_buf = 2 if len(shards) > 1 and free > 2 * out_max + (4 << 30) else 1
    shared = [torch.empty(out_max, dtype=torch.uint8, device="cuda") for _ in range(n_buf)]
    streams = [torch.cuda.Stream() for _ in range(n_buf)]
    for i, sh in enumerate(shards):
        runners.append(kvcache.KvGatherHash(sh, out=shared[i % n_buf]))
    torch.cuda.synchronize()

    def step():
        cur = torch.cuda.current_stream()
        start = cur.record_event()
        for st in streams:
            st.wait_event(start)
        for i, (r, pool) in enumerate(zip(runners, pools)):
            r.run(pool, stream=streams[i % n_buf].cuda_stream)
        for st in streams:
            cur.wait_stream(st)

    # parity: two sequences of the first shard against the numpy gather + OpenSSL tree hash
    runners[0].run(pools[0])
    torch.cuda.synchronize()
    runners[0].check_status()
    mh = runners[0].multihashes()
    host_pool = None
    ok = True
    for i in (0, shards[0].n_seq - 1):
        sh = shards[0]
        slots = sh.page_table[sh.page_offsets[i]:sh.page_offsets[i + 1]]
        if host_pool is None:
            host_pool = pools[0].cpu().numpy()
        want = okv.gather_sequence(host_pool, sh.planes, sh.pool_pages, sh.page_tokens, sh.token_bytes, slots,
                                   int(sh.seq_tokens[i]))
        ok &= bool((runners[0].sequence(i).cpu().numpy() == want).all())
        ok &= mh[i] == okv.sequence_multihash(want, kvcache.KV_LEAF)
    del host_pool
    for _ in range(args.warmup):
        step()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        n0 = _native.lib().tcx_kernel_launch_count()
        e0.record(s)
        for _ in range(args.steps):
            step()
        e1.record(s)
        e1.synchronize()
        launches = _native.lib().tcx_kernel_launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    # the pipelined path: the last shard's outputs and roots after the timed steps
    last, sh_last = runners[-1], shards[-1]
    last.check_status()
    mh_last = last.multihashes()
    host_pool = pools[-1].cpu().numpy()
    for i in (0, sh_last.n_seq - 1):
        slots = sh_last.page_table[sh_last.page_offsets[i]:sh_last.page_offsets[i + 1]]
        want = okv.gather_sequence(host_pool, sh_last.planes, sh_last.pool_pages, sh_last.page_tokens,
                                   sh_last.token_bytes, slots, int(sh_last.seq_tokens[i]))
        ok &= bool((last.sequence(i).cpu().numpy() == want).all())
        ok &= mh_last[i] == okv.sequence_multihash(want, kvcache.KV_LEAF)
    del host_pool
    mine = sum(r.gathered_bytes for r in runners)
    t = torch.tensor([ms, float(mine), 1.0 if ok else 0.0], dtype=torch.float64, device="cuda")
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        mn = t.clone()
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        ms, total, ok = float(mx[0]), float(sm[1]), bool(mn[2] > 0)
    else:
        total = float(mine)
    del runners, pools, shared
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"value": round(total / ms / 1e6, 2), "unit": "GB/s", "ms_per_step": round(ms, 3),
            "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"paged KV: 64 planes x {w.pool_pages} pages [16, 8, 128] bf16, seed 3, "
                                   f"{w.n_seq} sequences (64-4096 tokens), 2 MiB leaves, 8 sequence shards "
                                   "dealt to the ranks",
                       "gathered_bytes": int(total), "sequences": w.n_seq,
                       "pipeline": f"{n_buf} output buffer(s) / stream(s) per rank"},
            "parity": {"first_and_last_shard_sequences_match_oracle": ok},
            "gpu_launches": int(launches), "clocks": clk.summary()}


def run_kv(args) -> None:
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    out = kv_measure(args, world, rank, local)
    if rank == 0:
        line = {"metric": "Paged-KV gather + per-sequence SHA-256 GB/s (config 5)", "n_gpus": world,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u32",
                "data": "synthetic"}
        line.update(out)
        print(json.dumps(line), flush=True)
        if not out["parity"]["first_and_last_shard_sequences_match_oracle"]:
            raise SystemExit("PARITY FAILURE: paged-KV gather or hash differs from the oracle")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measure_disk_hash(args, steps: int, warmup: int) -> dict:
    """compute_data_multihash_from_disk_dir (disk_dir_hash.cc:47-104) of a directory holding
    the artifact, on this rank's GPU: preads into pinned slots, H2D and the leaf kernel per
    1 GiB group of 4 MiB leaves, Merkle root on the GPU; wall-clock timed (the call is
    synchronous), checked against the CPU oracle over the same payload bytes."""
    import numpy as np
    from oracle import oracle
    from tensorcast_b200.disk_hash import compute_data_multihash_from_disk_dir
    path = artifact_path(args)
    d = os.path.join(args.dir, f"dirhash-{args.model}")
    os.makedirs(d, exist_ok=True)
    link = os.path.join(d, "model.safetensors")
    if not os.path.islink(link):
        os.symlink(path, link)
    with open(path + ".done") as f:
        info = json.load(f)
    T = info["total_bytes"]
    got = None
    for _ in range(warmup):
        got = compute_data_multihash_from_disk_dir(d)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        got = compute_data_multihash_from_disk_dir(d)
        times.append(time.perf_counter() - t0)
    raw = np.memmap(path, dtype=np.uint8, mode="r", offset=info["payload_offset"], shape=(T,))
    want = oracle.multihash(oracle.tree_root(oracle.leaf_digests(raw, LEAF, openssl=True,
                                                                 threads=min(32, os.cpu_count() or 1))))
    ms = statistics.median(times) * 1e3
    return {"value": round(T / ms / 1e6, 2), "unit": "GB/s", "ms_per_call": round(ms, 1), "steps": steps,
            "config": {"workload": f"compute_data_multihash_from_disk_dir of a directory holding the {args.model} "
                                   f"safetensors file ({T} B payload, 4 MiB leaves, page-cache-hot tmpfs)",
                       "timing": "wall clock of the synchronous call"},
            "multihash": got, "matches_cpu_oracle": got == want}


def run_disk_hash(args) -> None:
    import torch
    if int(os.environ.get("RANK", "0")) != 0:
        return
    torch.cuda.set_device(0)
    path = ensure_artifact(args, 0, 0)
    out = measure_disk_hash(args, args.steps, args.warmup)
    with open(path + ".done") as f:
        info = json.load(f)
    cpu = None if args.no_cpu_baseline else cpu_reference_sample(path, info["payload_offset"], info["total_bytes"],
                                                                 LEAF, args.cpu_seconds)
    line = {"metric": "compute_data_multihash_from_disk_dir GB/s (tmpfs -> GPU SHA-256)", "n_gpus": 1,
            "warmup": args.warmup, "higher_is_better": True, "cpu_baseline": cpu}
    line.update(out)
    print(json.dumps(line), flush=True)
    if not out["matches_cpu_oracle"]:
        raise SystemExit("disk-dir multihash differs from the CPU oracle")




def verify_view_full(path, index, plan, d_view, world, rank, transposed=None):
    """Compares every tensor of this rank's view, byte for byte, with numpy slicing of the
    file (the tensor-parallel rule of tp_slices; the transposed tensor read whole and
    transposed). Returns (ok, bytes checked, tensors checked)."""
    import numpy as np
    import torch
    from concurrent.futures import ThreadPoolExecutor
    from tensorcast_b200.artifact import ELEMENT_SIZE
    slices = {} if world == 1 else tp_slices(index, world, rank)
    udt = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}
    torch.cuda.synchronize()

    def check(t):
        st, e = index.sources[t.name], index.entries[t.name]
        es = ELEMENT_SIZE[e.dtype]
        arr = np.memmap(path, dtype=udt[es], mode="r", offset=st.file_offset, shape=tuple(st.shape))
        if t.name == transposed:
            arr = arr.T
        elif t.name in slices:
            d, sl = slices[t.name]
            arr = arr[sl] if d == 0 else arr[:, sl]
        want = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        got = d_view[t.offset:t.offset + t.nbytes].cpu().numpy()
        return bool(got.size == want.size and np.array_equal(got, want)), int(t.nbytes)

    with ThreadPoolExecutor(max(2, min(16, len(os.sched_getaffinity(0))))) as ex:
        res = list(ex.map(check, plan.tensors))
    return all(r[0] for r in res), sum(r[1] for r in res), len(res)


def exchange_summary(mode: str, recv: float, phase_ms: float, xfer_ms: float, nccl_share: float = 0.0) -> dict:
    """The shard exchange of the device-resident steps, per rank: bytes received over the
    transfer itself (pushes or NCCL rounds, device events) as a fraction of NVLink 5 (900 GB/s
    per direction) and of the measured 770 GB/s peer copy; the phase also holds the local
    extraction and runs beside the leaf hash."""
    gbs = recv / xfer_ms / 1e6 if xfer_ms > 0 else 0.0
    if mode == "push" and nccl_share > 0:
        mode = f"push + {nccl_share:g} of each pair's bytes over NCCL"
    return {"mode": mode, "recv_bytes_per_rank": int(recv), "transfer_ms": round(xfer_ms, 3),
            "gbs_per_rank": round(gbs, 1), "frac_of_nvlink_900": round(gbs / 900.0, 4),
            "frac_of_measured_peer_copy_770": round(gbs / 770.0, 4), "exchange_and_view_ms": round(phase_ms, 3),
            "note": "received bytes per rank / the device time of the transfer (max over ranks); it runs beside the "
                    "leaf hash and the local extraction"}


def gpu_topology(world: int):
    """Where the N GPUs sit (queries only): PCI bus ids, the GPU-to-GPU link types and the CPU /
    NUMA affinity columns of `nvidia-smi topo -m`, so that GPUs sharing a host bridge or a
    socket can be told apart when the per-GPU H2D rates differ."""
    out = {}
    try:
        r = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id", "--format=csv,noheader"],
                           capture_output=True, text=True, timeout=30)
        ids = [ln.split(",")[1].strip() for ln in r.stdout.splitlines() if "," in ln]
        out["pci_bus_ids"] = ids[:world]
        r = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True, timeout=30)
        import re
        text = re.sub(r"\x1b\[[0-9;]*m", "", r.stdout)  # the header is underlined with escape codes
        lines = [ln for ln in text.splitlines() if ln.strip()]
        head = [h.strip() for h in lines[0].split("\t")] if lines else []
        rows = {}
        for ln in lines[1:]:
            cols = [c.strip() for c in ln.split("\t")]
            if cols and cols[0].startswith("GPU") and cols[0][3:].isdigit() and int(cols[0][3:]) < world:
                named = dict(zip(head[1:], cols[1:]))
                rows[cols[0]] = {"gpus": [named.get(f"GPU{j}", "?") for j in range(world)],
                                 "cpu_affinity": named.get("CPU Affinity"), "numa": named.get("NUMA Affinity"),
                                 "nics": {k: v for k, v in named.items() if k.startswith("NIC")}}
        out["topo"] = rows
    except (OSError, subprocess.SubprocessError, IndexError, ValueError) as e:
        out["error"] = str(e)
    return out


def host_mem_available() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def c4_leg(args, group, world: int, rank: int, local: int, read_threads: int, exchange: str = "nccl"):
    """BASELINE config 4 at N > 1: the Llama-3-70B-shaped artifact (141.1 GB, seed 2) with
    TP-N views plus the layer-0 o_proj stored [in, out] and read through a transpose view,
    over the NCCL shard exchange. Runs when the host can hold the file in tmpfs and every
    GPU its share and view; otherwise returns a skip reason. Parity: the root against the
    CPU oracle over the whole file and every byte of every rank's view against numpy
    slicing of the file. value: device-resident steps; e2e: from the file, as the main line."""
    import copy
    import numpy as np
    import torch
    import torch.distributed as dist
    from tensorcast_b200.artifact import build_canonical_index, build_source_index, canonical_segments
    from tensorcast_b200.loader import stage_bounds
    from tensorcast_b200.synthetic import artifact_bytes
    from tensorcast_b200.views import build_view_spec, plan_view
    a70 = copy.copy(args)
    a70.model = "llama3-70b"
    shapes = model_shapes(a70.model)
    need = artifact_bytes(shapes)
    path = artifact_path(a70)
    exists = os.path.exists(path + ".done")
    st = os.statvfs(args.dir) if os.path.isdir(args.dir) else None
    shm_free = st.f_bavail * st.f_frsize if st else 0
    host_ok = (exists or shm_free > need + (4 << 30)) and \
        host_mem_available() > (0 if exists else need) + world * (3 << 30) + (48 << 30)
    gpu_ok = torch.cuda.mem_get_info()[0] > 2.3 * need / world
    flags = torch.tensor([1.0 if host_ok else 0.0, 1.0 if gpu_ok else 0.0], dtype=torch.float64, device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if flags.min().item() < 1:
        return {"skipped": f"needs {need / 1e9:.1f} GB of tmpfs and host memory for the file "
                           f"(host ok: {bool(flags[0].item())}) and ~{2.3 * need / world / 1e9:.0f} GB free per GPU "
                           f"(gpu ok: {bool(flags[1].item())})"} if rank == 0 else None
    t0 = time.perf_counter()
    ensure_artifact(a70, rank, local, world)
    gen_s = time.perf_counter() - t0
    index = build_canonical_index(build_source_index(path))
    T, L = index.total_bytes, args.leaf
    bounds = stage_bounds(T, L, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    plans = []
    for r in range(world):
        slices = tp_slices(index, world, r)
        slices.pop(TRANSPOSED_O_PROJ, None)
        plans.append(plan_view(index, build_view_spec(index, slices=slices,
                                                      transpose={TRANSPOSED_O_PROJ: [(0, 1)]})))
    mine = plans[rank]
    rank_jobs = [p.jobs for p in plans]
    files = canonical_segments(index, lo, hi)
    d_stage = torch.empty(hi - lo, dtype=torch.uint8, device="cuda")
    d_view = torch.empty(max(mine.view_bytes, 1), dtype=torch.uint8, device="cuda")

    def load(from_files: bool, expected=None):
        return group.load(T, L, bounds, rank_jobs, d_stage=d_stage, d_view=d_view,
                          files=files if from_files else None, read_threads=read_threads,
                          permutes=mine.permutes, view_bytes=mine.view_bytes, expected_root=expected,
                          peer_push=exchange == "push",
                          push_nccl_share=push_share(args, world, exchange_bound=True) if exchange == "push" else 0.0)

    def mx(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    first = load(True)
    root = first["root"]
    root_ok = True
    if rank == 0:
        from oracle import oracle
        whole = canonical_segments(index, 0, T)
        if len(whole) == 1 and whole[0][3] == T:
            mm = np.memmap(path, dtype=np.uint8, mode="r", offset=whole[0][1], shape=(T,))
            root_ok = oracle.tree_root(oracle.leaf_digests(mm, L, openssl=True, threads=os.cpu_count() or 8)) == root
            del mm
    view_ok, checked, n_t = verify_view_full(path, index, mine, d_view, world, rank, TRANSPOSED_O_PROJ)
    agg = torch.tensor([1.0 if view_ok else 0.0, 1.0 if root_ok else 0.0, checked, n_t], dtype=torch.float64,
                       device="cuda")
    mn = agg.clone()
    dist.all_reduce(mn, op=dist.ReduceOp.MIN)
    dist.all_reduce(agg, op=dist.ReduceOp.SUM)
    # value: device-resident steps
    load(False, root)
    dist.barrier()
    torch.cuda.synchronize()
    res = [load(False, root) for _ in range(2)]
    ms = mx(statistics.mean(r["total_ms"] for r in res))
    hash_ms = mx(statistics.mean(r["hash_ms"] for r in res))
    exch_ms = mx(statistics.mean(r["exchange_ms"] for r in res))
    xfer_ms = mx(statistics.mean(r["transfer_ms"] for r in res))
    recv = mx(float(res[-1]["peer_recv_bytes"]))
    # e2e: from the file
    cur = torch.cuda.current_stream()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    load(True, root)
    dist.barrier()
    torch.cuda.synchronize()
    f0.record(cur)
    fres = [load(True, root) for _ in range(2)]
    f1.record(cur)
    f1.synchronize()
    file_ms = mx(f0.elapsed_time(f1) / 2)
    read_ms = mx(statistics.mean(r["stage_read_ms"] for r in fres))
    del d_stage, d_view
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"workload": f"llama3-70b-shaped bf16 safetensors (seed 2), {T} B, TP-{world} views + {TRANSPOSED_O_PROJ} "
                        "stored [in, out] read whole through a transpose view; "
                        + ("copy-engine push" if exchange == "push" else "NCCL send/recv shard exchange"),
            "artifact_bytes": T, "leaves": first["leaves"], "view_bytes_per_rank": mine.view_bytes,
            "value": round(T / ms / 1e6, 2), "ms_per_step": round(ms, 3), "steps": 2, "warmup": 1,
            "phases_ms": {"hash": round(hash_ms, 3), "exchange_and_view": round(exch_ms, 3)},
            "e2e": {"value": round(T / file_ms / 1e6, 2), "ms_per_step": round(file_ms, 3),
                    "stage_read_ms": round(read_ms, 3), "steps": 2, "warmup": 1,
                    "from": "the file in tmpfs, tcx_group_load_files on every rank"},
            "exchange": exchange_summary(exchange, recv, exch_ms, xfer_ms,
                                         push_share(args, world, exchange_bound=True) if exchange == "push" else 0.0),
            "parity": {"root_matches_cpu_oracle": bool(mn[1].item() > 0), "view_full_ok": bool(mn[0].item() > 0),
                       "view_bytes_checked": int(agg[2].item()), "view_tensors_checked": int(agg[3].item()),
                       "multihash": first["multihash"]},
            "ok": bool(mn[0].item() > 0 and mn[1].item() > 0),
            "artifact_write_s": round(gen_s, 1)}


def bind_into_check(args, path, index, world, rank, local) -> dict:
    """The collective bind_into of the SDK (Artifact.view(...).bind_into(targets, ctx=...),
    the reference's mapped-target load, collective_disk_loader.cc:5818-6293): every rank's
    tensor-parallel view straight into one separate CUDA tensor per tensor, through the
    NCCL shard exchange; every target compared byte for byte with numpy slicing of the file.
    Returns the result on rank 0 (all ranks take part)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from tensorcast_b200 import api
    from tensorcast_b200.artifact import ELEMENT_SIZE
    slices = tp_slices(index, world, rank)
    view_slices = {n: (sl if d == 0 else (1, sl)) for n, (d, sl) in slices.items()}
    art = api.from_disk(path).view(slices=view_slices)
    udt = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}
    dts = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16, "torch.float32": torch.float32}
    targets = {}
    for name, e in index.entries.items():
        shape = list(e.shape)
        if name in slices:
            d, sl = slices[name]
            shape[d] = sl.stop - sl.start
        targets[name] = torch.empty(shape, dtype=dts.get(e.dtype, torch.bfloat16), device=f"cuda:{local}")
    ctx = api.CallContext(collective=api.CollectiveLoadGroup("bench-bind-into", world, rank))
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    art.bind_into(targets, ctx=ctx)
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    bad, checked = 0, 0
    for name, t in targets.items():
        st, e = index.sources[name], index.entries[name]
        arr = np.memmap(path, dtype=udt[ELEMENT_SIZE[e.dtype]], mode="r", offset=st.file_offset, shape=tuple(st.shape))
        if name in slices:
            d, sl = slices[name]
            arr = arr[sl] if d == 0 else arr[:, sl]
        want = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        got = t.reshape(-1).view(torch.uint8).cpu().numpy()
        bad += 0 if np.array_equal(got, want) else 1
        checked += got.size
    r = torch.tensor([bad, checked, len(targets), secs], dtype=torch.float64, device="cuda")
    mx = r.clone()
    dist.all_reduce(r, op=dist.ReduceOp.SUM)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    del targets
    # Every rank releases the SDK's group here, at the same point (its NCCL finalize
    # involves the peers).
    for g in list(api._GROUPS.values()):
        g.close()
    api._GROUPS.clear()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"ok": int(r[0].item()) == 0, "targets_checked": int(r[2].item()), "bytes_checked": int(r[1].item()),
            "seconds_max_over_ranks": round(float(mx[3].item()), 3),
            "what": "SDK Artifact.view(TP-N slices).bind_into(one CUDA tensor per tensor, ctx=CollectiveLoadGroup) "
                    "from the file: every target == numpy slicing of the file"}


def straddling_tensors(index, bounds) -> int:
    """Tensors whose canonical bytes cross a rank's stage boundary (their pieces come from two ranks)."""
    inner = bounds[1:-1]
    return sum(1 for e in index.entries.values() if any(e.offset < b < e.offset + e.size for b in inner))


def reference_gpu_kernel(d_stage, nbytes: int, leaf: int, hk: dict):
    """Times the reference's own GPU kernel (tensorcast_sha256_leaf_kernel, its source text
    compiled with NVRTC for compute_100 by oracle/ref_gpu_build.py and launched with the
    reference's configuration by oracle/_ref/libref_gpu.so) beside the product kernel on the
    same bytes: the staged artifact at the bench's leaf size, and BASELINE config 1 (1 GiB of
    seed-0 bytes) at the reference GPU policy's 512 KiB leaves, whose digests must equal the
    committed golden ones. A baseline leg, like cpu_baseline."""
    import ctypes
    import numpy as np
    import torch
    import tensorcast_b200 as tcx
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libref_gpu.so")
    ptx = os.path.join(ROOT, "oracle", "_ref", "tensorcast_sha256_compute_100.ptx")
    if not (os.path.exists(lib_path) and os.path.exists(ptx)):
        return {"unavailable": "oracle/_ref not built (make -C oracle ref needs the reference source tree)"}
    lib = ctypes.CDLL(lib_path)
    lib.ref_gpu_last_error.restype = ctypes.c_char_p
    lib.ref_gpu_sha256_leaves.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p,
                                          ctypes.c_uint32, ctypes.c_void_p]
    torch.cuda.synchronize()
    if lib.ref_gpu_load(ptx.encode(), torch.cuda.current_device()) != 0:
        return {"unavailable": "reference kernel load failed: " + lib.ref_gpu_last_error().decode()}
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0.record(s)
            fn()
            e1.record(s)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    def ref_run(src, total, lf, out):
        n = (total + lf - 1) // lf
        rc = lib.ref_gpu_sha256_leaves(src.data_ptr(), total, lf, out.data_ptr(), n, s.cuda_stream)
        if rc != 0:
            raise RuntimeError(lib.ref_gpu_last_error().decode())

    out = {"kernel": "tensorcast_sha256_leaf_kernel: the reference's source text (core/common/artifact_hash_gpu.cc:"
                     "193-412) compiled by NVRTC for compute_100 with its own options and JIT-loaded by the driver; "
                     "launch 512 threads x min(ceil(leaves/512), 8*SMs) (:771-781)", "cases": {}}
    # (1) the staged artifact at the bench's leaf size
    n = (nbytes + leaf - 1) // leaf
    ref_d = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
    ours = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
    ms = timed(lambda: ref_run(d_stage, nbytes, leaf, ref_d), 1)
    tcx.sha256_leaves(d_stage, leaf, ours, nbytes=nbytes, stream=s)
    torch.cuda.synchronize()
    blocks = leaf // 64 + 1
    out["cases"]["artifact"] = {"bytes": nbytes, "leaf_bytes": leaf, "leaves": n, "ms": round(ms, 3),
                                "gbs": round(nbytes / ms / 1e6, 2), "us_per_block": round(ms * 1e3 / blocks, 3),
                                "tcx_ms": hk["kernel_ms"],
                                "tcx_us_per_block": round(hk["kernel_ms"] * 1e3 / blocks, 4),
                                "speedup_tcx_vs_reference": round(ms / hk["kernel_ms"], 2),
                                "digests_equal_tcx": bool(torch.equal(ref_d, ours))}
    del ref_d, ours
    # (2) BASELINE config 1 at the reference GPU policy's leaf: 1 GiB of seed-0 bytes, 512 KiB leaves
    golden = os.path.join(ROOT, "tests", "golden", "c1_seed0_1gib_leaf512kib.digests.bin")
    c1 = torch.from_numpy(np.random.default_rng(0).integers(0, 256, size=1 << 30, dtype=np.uint8)).cuda()
    lf, total = 512 << 10, 1 << 30
    n = total // lf
    ref_d = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
    ours = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
    ms = timed(lambda: ref_run(c1, total, lf, ref_d), 3)
    t_ms = timed(lambda: tcx.sha256_leaves(c1, lf, ours, stream=s), 5)
    want = np.fromfile(golden, dtype=np.uint8).reshape(-1, 32) if os.path.exists(golden) else None
    blocks = lf // 64 + 1
    out["cases"]["c1_1GiB_512KiB"] = {
        "bytes": total, "leaf_bytes": lf, "leaves": n, "ms": round(ms, 3), "gbs": round(total / ms / 1e6, 2),
        "us_per_block": round(ms * 1e3 / blocks, 3), "tcx_ms": round(t_ms, 3),
        "tcx_gbs": round(total / t_ms / 1e6, 2), "speedup_tcx_vs_reference": round(ms / t_ms, 2),
        "reference_digests_equal_golden": None if want is None else bool((ref_d.cpu().numpy() == want).all()),
        "tcx_digests_equal_golden": None if want is None else bool((ours.cpu().numpy() == want).all())}
    del c1, ref_d, ours
    torch.cuda.synchronize()
    return out


def hash_kernel_roofline(d_stage, nbytes: int, leaf: int, rank: int) -> dict:
    """Times the SHA-256 leaf kernel alone over the staged bytes and the register-only probes."""
    import torch
    import tensorcast_b200 as tcx
    from tensorcast_b200 import _native
    n = (nbytes + leaf - 1) // leaf
    out = torch.empty((n, 32), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0.record(s)
            fn()
            e1.record(s)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    ms = timed(lambda: tcx.sha256_leaves(d_stage, leaf, out, nbytes=nbytes, stream=s))
    achieved = nbytes / ms / 1e6
    # Compute bound: 64 chains per SMSP x 592 SMSPs, 1024 blocks each.
    probe_n, probe_b = 148 * 4 * 64, 1024
    pout = torch.empty((probe_n, 32), dtype=torch.uint8, device="cuda")
    pms = timed(lambda: _native.call("tcx_sha256_compute_probe", probe_n, probe_b, pout.data_ptr(), s.cuda_stream))
    compute = probe_n * probe_b * 64 / pms / 1e6
    # Chain latency of the leaf kernel itself: 32 chains (one consumer warp) of 4096 blocks each.
    lb = 4096 * 64
    lout = torch.empty((32, 32), dtype=torch.uint8, device="cuda")
    lsrc = d_stage[: 32 * lb] if d_stage.numel() >= 32 * lb else torch.zeros(32 * lb, dtype=torch.uint8, device="cuda")
    lms = timed(lambda: tcx.sha256_leaves(lsrc, lb, lout, nbytes=32 * lb - 64, stream=s), reps=2)
    t_block_us = lms * 1e3 / 4096
    chain = n * 64 / (t_block_us * 1e-6) / 1e9
    hbm = measured_hbm()
    peak = min(compute, hbm["gbs"])
    traffic = profiled_traffic(nbytes)
    return {"bound": "int_alu" if compute < hbm["gbs"] else "hbm", "achieved": round(achieved, 2),
            "peak": round(peak, 2), "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": traffic, "kernel": "sha256_leaf (ws/plain auto)", "leaves": n,
            "algorithmic_bytes": nbytes, "kernel_ms": round(ms, 3),
            "compute_bound_gbs": round(compute, 2), "compute_bound_source": "measured: register-only SHA-256 probe, "
            f"{probe_n} chains x {probe_b} blocks", "hbm_gbs": hbm["gbs"], "hbm_source": hbm["source"],
            "frac_of_hbm": round(achieved / hbm["gbs"], 4), "chain_bound_gbs": round(chain, 2),
            "t_block_us_one_chain_per_lane": round(t_block_us, 4), "frac_of_chain_bound": round(achieved / chain, 4)}


def measured_hbm() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return {"gbs": float(json.load(f)["hbm_gbs"]), "source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}
    except Exception:
        return {"gbs": 6650.0, "source": "profiling recipe fallback 6.65 TB/s (of fallback)"}


def profiled_traffic(nbytes: int):
    """DRAM bytes of one launch, scaled from the committed ncu capture of the leaf kernel."""
    p = os.path.join(ROOT, "profiles", "sha256_leaf_traffic.txt")
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("dram_bytes_per_hashed_byte:"):
                    return round(float(line.split(":", 1)[1]) * nbytes)
    except OSError:
        pass
    return None


if __name__ == "__main__":
    main()
