"""The branch scheduler's host logic on the CPU: lane seeds and streams, the
reference's primitive cycle (one commit for the start record, then per
primitive eight partial queries and one commit, inference/batch.rs:415-494),
retirement of finished lanes, which then draw nothing, and the LPT plan."""
from __future__ import annotations

import numpy as np

import sched_standins as S


def _splitmix_uniform(seed: int, n: int) -> float:
    """SplitMix64 (Steele, Lea and Flood 2014) restated in Python: output n
    of the generator seeded `seed`, top 24 bits / 2^24."""
    m = (1 << 64) - 1
    z = (seed + (n + 1) * 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    z ^= z >> 31
    return (z >> 40) / 16777216.0


def test_lane_seed_and_stream_values(pp):
    sched = pp.sched
    assert sched.parallel_seed(7, 3) == 10
    assert sched.parallel_seed((1 << 64) - 2, 5) == 3  # wraps like u64::wrapping_add
    for seed in (0, 1, 12345, (1 << 64) - 1):
        for n in (0, 1, 2, 99, 1 << 40):
            assert sched.lane_uniform(seed, n) == _splitmix_uniform(seed, n)
    u = [sched.lane_uniform(sched.parallel_seed(42, 0), n) for n in range(20000)]
    assert 0.0 <= min(u) and max(u) < 1.0 and abs(np.mean(u) - 0.5) < 0.01


def test_primitive_cycle_retirement_and_records(pp):
    sched = pp.sched
    w = S.small_windows(sched)
    lanes, budgets, seed, rows = [5, 0, 9, 2], [6, 1, 9, 4], 1234, 6
    model = S.RecordingModel(rows, w)
    streams = S.HostStreams(sched, seed, lanes, rows, "cpu")
    runner = sched.ShardRunner(model, lanes, seed, budgets, w, streams=streams, sampler=S.window_sampler)
    res = runner.run()
    assert [r.lane for r in res] == lanes
    for r, b in zip(res, budgets):
        want, why = S.expected_records(sched, w, seed, r.lane, b)
        np.testing.assert_array_equal(r.records, want)
        assert r.reason == why
        # a lane draws 9 uniforms per primitive it generated, then no more
        assert streams.draws[lanes.index(r.lane)] == 9 * len(want)
    assert streams.draws[4] == streams.draws[5] == 0  # rows without a lane never draw
    log = model.log
    assert log[0] == (True, 0, (1, 1, 1, 1, 0, 0))
    body = log[1:]
    assert len(body) % 9 == 0
    for p in range(len(body) // 9):
        cyc = body[9 * p: 9 * p + 9]
        assert [c[:2] for c in cyc] == [(False, f) for f in range(1, 9)] + [(True, 0)]
        assert len({c[2] for c in cyc}) == 1  # one ready set for the whole primitive
    # the ready set shrinks exactly when lanes finish
    generated = {r.lane: len(r.records) for r in res}
    for p in range(len(body) // 9):
        act = body[9 * p][2]
        assert act[:4] == tuple(int(generated[ln] > p) for ln in lanes)


def test_lpt_plan_balances_context_lengths(pp):
    costs = [8000, 300, 5000, 2900, 100, 4000]
    plan = pp.sched.ShardPlan.make(costs, 2)
    loads = [sum(costs[b] for b in m) for m in plan.members]
    assert sorted(sum(plan.members, [])) == list(range(6))
    # longest first onto the lightest shard: 8000 | 5000, 4000 | 2900 | 300, 100
    assert loads == [10900, 9400]
    assert max(loads) <= 4 / 3 * max(sum(costs) / 2, max(costs))  # LPT's bound
