"""A multi-GPU collective-load parity check with the ranks as threads of ONE process (the
reference daemon's model: N rank threads, one per GPU, that find each other by group id;
launched by tests/test_multi_gpu.py in a fresh process).

Each rank thread joins with tcx_group_join (Group.join), gathers every rank's view jobs
through the in-process rendezvous, and runs the same cases as the one-process-per-GPU
worker (tests/load_cases.py: every exchange mode, the peer push writing through the
sibling threads' own pointers, staging from pinned memory, files or the device, the
bind-into targets). Then the SDK path: from_disk(...).view(...).tensor_dict(ctx=
CallContext(collective=CollectiveLoadGroup(group_id, N, r))) from every thread, against
the safetensors reader. Exit status 0 = pass."""
import os
import sys
import tempfile
import threading
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import torch  # noqa: E402

from load_cases import run_cases  # noqa: E402
from tensorcast_b200 import api  # noqa: E402
from tensorcast_b200.api import gather_rank_jobs  # noqa: E402
from tensorcast_b200.loader import Group  # noqa: E402
from tensorcast_b200.synthetic import llama_shapes, tiny_llama, write_safetensors  # noqa: E402


def sdk_case(path: str, world: int, rank: int) -> int:
    from safetensors.torch import load_file
    ref = load_file(path)
    slices = {}
    for name, t in ref.items():
        if any(k in name for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "embed", "lm_head")):
            n = t.shape[0] // world
            slices[name] = slice(rank * n, (rank + 1) * n)
        elif any(k in name for k in ("o_proj", "down_proj")):
            n = t.shape[1] // world
            slices[name] = (1, slice(rank * n, (rank + 1) * n))
    ctx = api.CallContext(collective=api.CollectiveLoadGroup("sdk-threads", world, rank))
    got = api.from_disk(path).view(slices=slices).tensor_dict(device=f"cuda:{rank}", ctx=ctx)
    bad = 0
    for name, t in ref.items():
        want = t
        if name in slices:
            s = slices[name]
            want = t[s] if isinstance(s, slice) else t[:, s[1]]
        if not torch.equal(got[name].cpu(), want.contiguous()):
            print(f"rank {rank}: SDK tensor {name} FAILED", flush=True)
            bad += 1
    return bad


def main() -> int:
    world = int(sys.argv[1])
    if torch.cuda.device_count() < world:
        print(f"needs {world} GPUs", flush=True)
        return 2
    failures = [0] * world
    errors = []
    with tempfile.TemporaryDirectory() as tmp:
        art = os.path.join(tmp, "model.safetensors")
        write_safetensors(art, llama_shapes(tiny_llama(layers=2, hidden=128, ffn=256, vocab=512)), 9, device="cpu")

        def rank_thread(r: int) -> None:
            try:
                torch.cuda.set_device(r)
                group = Group.join("threads-parity", world, r, r, timeout_ms=60_000)
                try:
                    d = os.path.join(tmp, f"r{r}")
                    os.makedirs(d)
                    failures[r] = run_cases(group, world, r,
                                            lambda jobs: gather_rank_jobs(jobs, world, r, "threads-parity-jobs"), d,
                                            log=lambda m: print(m, flush=True))
                finally:
                    group.close()
                failures[r] += sdk_case(art, world, r)
            except Exception:  # noqa: BLE001
                errors.append(f"rank {r}: " + traceback.format_exc())

        threads = [threading.Thread(target=rank_thread, args=(r,), daemon=True) for r in range(world)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=500)
        if any(t.is_alive() for t in threads):
            errors.append("a rank thread did not finish")
    for e in errors:
        print(e, flush=True)
    print(f"threads load parity: world={world} failures={sum(failures)} errors={len(errors)}", flush=True)
    return 0 if sum(failures) == 0 and not errors else 1


if __name__ == "__main__":
    sys.exit(main())
