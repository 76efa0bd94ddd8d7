"""Branch sharding across ranks (host logic of the multi-GPU path), as gloo
processes on the CPU: the LPT shards of a ragged batch, decoded rank by rank
and gathered to rank 0, equal the batch decoded in one piece; a rank that
leaves before the gather makes the others fail within the group timeout."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "gloo_shard_worker.py")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, lengths: list[int], fail_rank: int = -1) -> list[tuple[int, str]]:
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   SHARD_LENGTHS=",".join(map(str, lengths)), SHARD_FAIL_RANK=str(fail_rank),
                   CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    out = []
    for p in procs:
        try:
            text, _ = p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            text, _ = p.communicate()
        out.append((p.returncode, text))
    return out


@pytest.mark.parametrize("world,lengths", [
    (2, [64, 1, 30, 50, 7]),           # ragged: the LPT shards hold 1 and 4 branches
    (2, [40, 40, 40, 40]),             # equal: 2 + 2
    (3, [12, 5]),                      # more ranks than branches: one shard is empty
])
def test_sharded_decode_gathers_to_whole_batch(world, lengths):
    res = _run(world, lengths)
    for r, (rc, text) in enumerate(res):
        assert rc == 0, f"rank {r} exited {rc}:\n{text}"


def test_rank_leaving_before_gather_fails_the_others():
    res = _run(2, [64, 1, 30, 50, 7], fail_rank=1)
    assert res[1][0] == 3
    assert res[0][0] != 0, "rank 0 completed a gather its peer never joined"
