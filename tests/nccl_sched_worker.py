"""One rank of tests/test_gpu_sched_ranks.py: the branch scheduler with one
shard per process and GPU.  The default group is gloo (the rendezvous); the
records travel to rank 0 over an NCCL group, which creates its communicator
at the final gather.  Rank 0 writes every lane's records and retirement
reason to SCHED_OUT (an .npz file)."""
from __future__ import annotations

import datetime
import importlib
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.dirname(HERE), HERE]

import sched_gpu_setup as G  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    records_group = dist.new_group(backend="nccl", timeout=datetime.timedelta(seconds=60))
    pp = importlib.import_module("pop2-bezier_b200")
    res = G.scheduler(pp).run_rank(dist, dev, group=records_group)
    if rank == 0:
        np.savez(os.environ["SCHED_OUT"], **{f"lane{ln}": r.records for ln, r in res.items()},
                 reasons=np.array([res[ln].reason for ln in range(len(G.COSTS))]))
    else:
        assert res is None
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
