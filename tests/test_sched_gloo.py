"""The branch scheduler over ranks (one shard per rank, gloo on the CPU):
lanes split by LPT over 2 and 3 ranks produce, after the final gather on
rank 0, exactly the records each lane's own stream (seed + lane) dictates,
with the same retirement, whatever rank ran them."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "gloo_sched_worker.py")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,costs,budgets", [
    (2, [4000, 300, 2500, 2600, 10, 900, 7000], [5, 1, 8, 3, 12, 2, 6]),
    (3, [100, 200], [4, 7]),  # more ranks than lanes: one rank holds none
])
def test_sharded_lanes_match_their_streams(world, costs, budgets):
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   SCHED_COSTS=",".join(map(str, costs)), SCHED_BUDGETS=",".join(map(str, budgets)),
                   SCHED_SEED="77", CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    for r, p in enumerate(procs):
        try:
            text, _ = p.communicate(timeout=180)
        except subprocess.TimeoutExpired:
            p.kill()
            text, _ = p.communicate()
        assert p.returncode == 0, f"rank {r} exited {p.returncode}:\n{text}"
