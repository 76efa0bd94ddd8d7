"""CPU stand-ins for the branch scheduler's device parts, used by the host
logic tests (tests/test_sched_cpu.py and the gloo ranks of
tests/test_sched_gloo.py).  They replace the model, the lane streams and the
sampler so that the primitive cycle, the lane seeding, retirement and the
gather can be checked without a GPU; none of them is the product.

The sampler stand-in maps a uniform u onto the field window as
start + floor(u * count), so every sampled token shows the exact draw that
produced it."""
from __future__ import annotations

import numpy as np
import torch

FIELDS = 9


def small_windows(sched):
    """Nine small windows; field 0 has 4 tokens and token 3 ends a lane."""
    sizes = [4, 5, 6, 7, 8, 9, 10, 11, 12]
    out, s = [], 0
    for n in sizes:
        out.append((s, n))
        s += n
    return sched.FieldWindows(out, end_token=3)


class RecordingModel:
    """Checks every query against the reference's cycle and returns zero
    logits: partial query f sees fields < f sampled and fields >= f empty on
    every active row; commits carry complete records."""

    def __init__(self, rows: int, windows):
        self.rows, self.windows = rows, windows
        self.device = torch.device("cpu")
        self.log = []  # (commit, field, active rows)

    def query(self, rec, active, commit, field):
        on = active.bool()
        r = rec[on]
        if commit:
            if len(self.log):  # every query after the start record commits a complete record
                assert (r >= 0).all(), "commit of an incomplete record"
            assert field == 0
        else:
            assert 1 <= field < FIELDS
            assert (r[:, :field] >= 0).all() and (r[:, field:] == -1).all(), f"partial query {field} record"
        self.log.append((bool(commit), int(field), tuple(int(x) for x in active.tolist())))
        return torch.zeros(self.rows, self.windows.windows[field][1])


class HostStreams:
    """The lane streams on the host through pp_b200_sched_uniform."""

    def __init__(self, sched, seed, lanes, rows, device):
        self.sched = sched
        self.seeds = [sched.parallel_seed(seed, ln) for ln in lanes] + [0] * (rows - len(lanes))
        self.draws = [0] * rows

    def draw(self, active):
        out = torch.zeros(len(self.draws), dtype=torch.float32)
        for r, a in enumerate(active.tolist()):
            if a:
                out[r] = self.sched.lane_uniform(self.seeds[r], self.draws[r])
                self.draws[r] += 1
        return out


def window_sampler(raw, uniforms, bounds, start):
    count = bounds[:, 1].to(torch.float64)
    col = torch.clamp(torch.floor(uniforms.to(torch.float64) * count), max=count - 1)
    return (start + col).to(torch.int32)


def expected_records(sched, windows, seed: int, lane: int, budget: int):
    """The records a lane must produce with the stand-ins: draw p*9+f of its
    stream picks field f of primitive p; it stops at the end token or its
    budget."""
    s = sched.parallel_seed(seed, lane)
    recs = []
    for p in range(budget):
        row = []
        for f, (start, count) in enumerate(windows.windows):
            u = sched.lane_uniform(s, p * FIELDS + f)
            row.append(start + min(int(np.floor(np.float64(u) * count)), count - 1))
        recs.append(row)
        if row[0] == windows.end_token:
            return np.asarray(recs, np.int64), "end"
    return np.asarray(recs, np.int64), "limit"
