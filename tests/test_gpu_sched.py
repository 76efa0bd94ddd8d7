"""The branch scheduler on the B200: the device lane streams against their
host form, and a run of independent lanes split over two shards (two
streams, two host threads) against the same lanes in one shard, which must
agree bit for bit (records and retirement), with the synthetic decoder,
int8 KV appends (partial and commit queries), attention and the device
sampler all on the device."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import sched_gpu_setup as G

pytestmark = pytest.mark.gpu


def test_device_streams_match_host_and_skip_inactive_rows(pp, cuda):
    sched = pp.sched
    lanes = [3, 0, 17]
    st = sched.DeviceLaneStreams(99, lanes, 5, cuda)
    masks = [[1, 1, 1, 0, 0], [1, 0, 1, 0, 0], [0, 0, 1, 0, 0], [1, 1, 1, 0, 0]]
    draws = [0] * 5
    for m in masks:
        got = st.draw(torch.tensor(m, dtype=torch.int32, device=cuda)).cpu().numpy()
        for r in range(5):
            if m[r]:
                want = sched.lane_uniform(sched.parallel_seed(99, lanes[r]), draws[r])
                assert got[r] == np.float32(want), (r, got[r], want)
                draws[r] += 1
            else:
                assert got[r] == 0.0
    assert st.draws.cpu().tolist() == draws


def test_two_shards_match_one_shard_bit_for_bit(pp, cuda):
    budgets = G.BUDGETS
    one = G.scheduler(pp).run([cuda])
    two = G.scheduler(pp).run([cuda, cuda])
    assert sorted(one) == sorted(two) == list(range(8))
    for lane in range(8):
        a, b = one[lane], two[lane]
        assert a.reason == b.reason, lane
        np.testing.assert_array_equal(a.records, b.records, err_msg=f"lane {lane}")
        assert len(a.records) <= budgets[lane]
        assert a.reason == "end" or len(a.records) == budgets[lane]
        w = pp.sched.default_windows()
        for f, (s, c) in enumerate(w.windows):
            assert ((a.records[:, f] >= s) & (a.records[:, f] < s + c)).all()
