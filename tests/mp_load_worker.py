"""One rank of a multi-GPU collective-load parity check (launched by tests/test_multi_gpu.py
through torch.distributed.run; one process per GPU, NCCL).

Every rank builds the same seeded artifact bytes, plans its own view (tensor-parallel
narrows, a transpose, sometimes a subset), gathers every rank's view jobs, stages its
leaf-aligned share (from pinned memory, from a file, or already on the device), and runs
the load in every exchange mode (tests/load_cases.py). Its view must equal the numpy
oracle byte for byte and the Merkle root the CPU oracle's; exit status 0 = pass."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import datetime  # noqa: E402
import tempfile  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from load_cases import run_cases  # noqa: E402
from tensorcast_b200.api import gather_rank_jobs  # noqa: E402
from tensorcast_b200.loader import Group  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    group = Group.from_torch_distributed(local, timeout_ms=60_000)
    failures = 0
    try:
        with tempfile.TemporaryDirectory() as tmp:
            failures = run_cases(group, world, rank, lambda jobs: gather_rank_jobs(jobs, world), tmp,
                                 log=lambda m: print(m, flush=True))
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
