"""One rank of the branch-shard test (run by tests/test_shards_gloo.py as a
child process, gloo backend on 127.0.0.1, no GPU).

Every rank builds the same seeded batch of independent branches, decodes the
branches its LPT shard owns (the CPU checker stands in for the device kernel:
this exercises the host-side sharding and the final gather, not the
arithmetic), and gathers the outputs to rank 0, which compares them with the
whole batch decoded in one piece.  Exit status 0 = agreement.
"""
from __future__ import annotations

import datetime
import importlib
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    lengths = [int(x) for x in os.environ["SHARD_LENGTHS"].split(",")]
    fail_rank = int(os.environ.get("SHARD_FAIL_RANK", "-1"))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    pp = importlib.import_module("pop2-bezier_b200")
    import oracle

    heads, d, cap = 2, 64, max(lengths)
    branches, rows = len(lengths), len(lengths) * heads
    g = np.random.Generator(np.random.PCG64(7))
    k = g.integers(0, 256, (rows, cap, d), dtype=np.uint8)
    v = g.integers(0, 256, (rows, cap, d), dtype=np.uint8)
    ks = g.uniform(0.005, 0.03, (rows, cap)).astype(np.float32)
    vs = g.uniform(0.005, 0.03, (rows, cap)).astype(np.float32)
    q = g.standard_normal((rows, d), dtype=np.float32)
    lens = np.asarray(lengths, np.uint32)

    shards = pp.kv_cache.BranchShards(lengths, world, rank)
    if rank == fail_rank:
        raise SystemExit(3)  # leaves before the gather: the others must end with an error, not wait for good
    mine_rows = np.asarray([b * heads + h for b in shards.mine for h in range(heads)], np.int64)
    if len(mine_rows):
        part = oracle.attention(q[mine_rows], k[mine_rows], v[mine_rows], ks[mine_rows], vs[mine_rows],
                                lens[shards.mine], heads)
    else:
        part = np.zeros((0, d), np.float32)
    out = torch.from_numpy(part).reshape(len(shards.mine), heads, d)
    try:
        full = shards.gather(dist, out)
    except Exception as e:  # a peer left: reported, not waited on
        print(f"rank {rank}: gather failed: {type(e).__name__}", flush=True)
        return 4
    status = 0
    if rank == 0:
        want = oracle.attention(q, k, v, ks, vs, lens, heads).reshape(branches, heads, d)
        if not np.array_equal(full.numpy(), want):
            print("rank 0: gathered outputs differ from the whole-batch decode", flush=True)
            status = 1
    dist.destroy_process_group()
    return status


if __name__ == "__main__":
    sys.exit(main())
