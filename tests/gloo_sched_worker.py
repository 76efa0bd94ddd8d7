"""One rank of the branch-scheduler test (run by tests/test_sched_gloo.py as
a child process, gloo backend on 127.0.0.1, no GPU).

Every rank runs BranchScheduler.run_rank over the same lanes with the CPU
stand-ins of tests/sched_standins.py: its LPT shard of the lanes goes through
the primitive cycle with no collective, and one gather brings every lane's
records to rank 0, which checks each lane against the records its own stream
must produce (seed + lane, draw p*9+f) and its retirement reason.
Exit status 0 = agreement."""
from __future__ import annotations

import datetime
import importlib
import os
import sys

import numpy as np
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, HERE]

import sched_standins as S  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    costs = [int(x) for x in os.environ["SCHED_COSTS"].split(",")]
    budgets = [int(x) for x in os.environ["SCHED_BUDGETS"].split(",")]
    seed = int(os.environ["SCHED_SEED"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    sched = importlib.import_module("pop2-bezier_b200").sched
    w = S.small_windows(sched)
    rows = max(len(m) for m in sched.ShardPlan.make(costs, world).members)

    def make_model(shard, lanes, device):
        return S.RecordingModel(rows, w)

    bs = sched.BranchScheduler(make_model, costs, seed, budgets, w,
                               make_streams=lambda sd, lanes, r, dev: S.HostStreams(sched, sd, lanes, r, dev),
                               sampler=S.window_sampler)
    res = bs.run_rank(dist, "cpu")
    status = 0
    if rank == 0:
        assert sorted(res) == list(range(len(costs)))
        for lane, r in res.items():
            want, why = S.expected_records(sched, w, seed, lane, budgets[lane])
            if not (np.array_equal(r.records, want) and r.reason == why):
                print(f"lane {lane}: got {r.records.tolist()} {r.reason}, want {want.tolist()} {why}", flush=True)
                status = 1
    else:
        assert res is None
    dist.barrier()
    dist.destroy_process_group()
    return status


if __name__ == "__main__":
    sys.exit(main())
