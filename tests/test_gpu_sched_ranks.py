"""The branch scheduler with one shard per GPU (two processes, two B200s):
the lanes split by LPT over two ranks, each on its own GPU, and gathered to
rank 0 over NCCL, must give every lane the records and retirement that one
shard on one GPU gives.  Skipped on a box with fewer than two GPUs."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

import sched_gpu_setup as G

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_on_two_gpus_match_one_shard(pp, cuda, tmp_path):
    one = G.scheduler(pp).run([cuda])
    torch.cuda.synchronize()
    out = tmp_path / "ranks.npz"
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), GLOO_SOCKET_IFNAME="lo", SCHED_OUT=str(out))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "nccl_sched_worker.py")], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    for r, p in enumerate(procs):
        try:
            text, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            p.kill()
            text, _ = p.communicate()
        assert p.returncode == 0, f"rank {r} exited {p.returncode}:\n{text}"
    got = np.load(out)
    for lane in range(len(G.COSTS)):
        assert str(got["reasons"][lane]) == one[lane].reason, lane
        np.testing.assert_array_equal(got[f"lane{lane}"], one[lane].records, err_msg=f"lane {lane}")
