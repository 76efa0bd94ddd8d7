"""Branch scheduler: independent generation lanes sharded over GPUs.

The reference runs parallel generation on one device
(NativeEngine::generate_parallel, app/src/inference/batch.rs:241-558): every
lane owns its KV cache and a random stream seeded `seed + lane`
(parallel_seed, batch.rs:9-11); for each primitive (a record of nine
attributes) the ready lanes are stacked into one batch, field 0 is sampled
from the head the previous commit produced, fields 1..8 each take one
partial query (commit = false: the current record with the fields sampled so
far, the rest as placeholders, batch.rs:415-469), and one commit query appends
the finished record to every ready lane's cache and yields the next
primitive's head (commit = true, batch.rs:485-494).  A lane that finishes
(its end token, or its primitive budget) drops out of `ready` and draws no
more random numbers.

Here the same cycle runs per shard:
  * LPT partition of the lanes over shards by their context length
    (pp_b200_sched_partition);
  * one device and one stream per shard, one host thread per shard in one
    process (BranchScheduler.run), or one shard per rank of a process group
    (BranchScheduler.run_rank) with the records gathered to rank 0 by one
    NCCL gather at the end and no collective during generation;
  * per-lane random streams on the device (pp_b200_sched_uniforms): draw n of
    lane i is the n-th output of SplitMix64 seeded `seed + i`, whatever shard
    or batch row holds the lane;
  * the model's per-query work (embedding, decoder step, output head) and the
    Rényi sampler stay on the device; the host reads the batch's records once
    per primitive, to retire lanes and report records.
A retired lane keeps its batch row: its attention reads no history (length 0)
and its row rides along in the projections, whose cost is the weight stream
and not the row count, so nothing is compacted or copied.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _native as N
from . import decoder as D
from . import int8_kv_ops as ops
from . import kv_cache
from . import sampling

FIELDS = 9
PARTIAL = -1  # a field not predicted yet (the reference's learnable empty attribute)
MASK64 = (1 << 64) - 1


def parallel_seed(base: int, lane: int) -> int:
    """inference/batch.rs:9-11: lane `lane` of a generation seeded `base`."""
    return int(N.lib.pp_b200_sched_lane_seed(base & MASK64, lane & MASK64))


def lane_uniform(lane_seed: int, draw: int) -> float:
    """Draw `draw` of the lane stream (the host form of the device streams)."""
    return float(N.lib.pp_b200_sched_uniform(lane_seed & MASK64, draw & MASK64))


@dataclass
class FieldWindows:
    """The legal token window (start, count) of each of the nine fields in
    the model's output vocabulary, and the field-0 token that ends a lane."""
    windows: list[tuple[int, int]]
    end_token: int

    def __post_init__(self):
        if len(self.windows) != FIELDS:
            raise N.PreconditionError(f"{FIELDS} field windows required")
        s, c = self.windows[0]
        if not s <= self.end_token < s + c:
            raise N.PreconditionError("the end token must lie in field 0's window")

    @property
    def vocab(self) -> int:
        return max(s + c for s, c in self.windows)


def default_windows() -> FieldWindows:
    """Nine attribute windows in the spirit of the reference's record (x, y,
    angle, width, height, shape, red, green, blue; docs/architecture.md):
    half-pixel coordinates, third-degree angles, quarter-pixel sizes, 128
    colour levels; field 0 also holds the end token."""
    sizes = [1025, 1024, 1080, 1024, 1024, 4, 128, 128, 128]
    out, s = [], 0
    for n in sizes:
        out.append((s, n))
        s += n
    return FieldWindows(out, end_token=1024)


@dataclass
class LaneResult:
    lane: int
    records: np.ndarray  # int64 [generated, 9]
    reason: str          # "end" (sampled the end token) or "limit" (primitive budget)


class DeviceLaneStreams:
    """Per-row random streams on the device (pp_b200_sched_uniforms): row r
    holds lane lanes[r]; rows past the shard's lanes never draw."""

    def __init__(self, seed: int, lanes: list[int], rows: int, device):
        seeds = [parallel_seed(seed, ln) for ln in lanes] + [0] * (rows - len(lanes))
        self.seeds = torch.tensor(np.asarray(seeds, dtype=np.uint64).view(np.int64), device=device)
        self.draws = torch.zeros(rows, dtype=torch.int64, device=device)
        self.out = torch.empty(rows, dtype=torch.float32, device=device)

    def draw(self, active: torch.Tensor) -> torch.Tensor:
        N.check(N.lib.pp_b200_sched_uniforms(ops._ptr(self.seeds), ops._ptr(self.draws), ops._ptr(active),
                                             active.numel(), ops._ptr(self.out), ops._stream(self.out)))
        return self.out


def device_sampler(alpha: float):
    """The Rényi sampler of the reference's device path (CFG 1): raw holds
    one field's logits, `start` is the field's first token id."""
    def sample(raw: torch.Tensor, uniforms: torch.Tensor, bounds: torch.Tensor, start: int) -> torch.Tensor:
        tok, _, _ = sampling.renyi_sample(raw, uniforms, bounds, alpha, 1.0, 1, start)
        return tok.view(-1)
    return sample


class ShardRunner:
    """The primitive cycle of one shard.

    model: rows (batch rows, >= len(lanes)), device, and
      query(records int32 [rows, 9], active int32 [rows], commit, field)
        -> f32 [rows, count of field's window]
      (the reference's forward_records_batched_for for the stacked rows with
      OutputScope::Field(field), or NextPrimitive = field 0 when committing;
      commit appends the record to the active rows' caches).
      An optional `status_word()` returns the model's device status bits.
    lanes: global lane ids, one per batch row from row 0.
    max_primitives: per lane (same order as lanes).
    streams / sampler: the device lane streams and sampler by default."""

    def __init__(self, model, lanes: list[int], seed: int, max_primitives: list[int], windows: FieldWindows, *,
                 alpha: float = 4.0, streams=None, sampler=None):
        if len(lanes) > model.rows:
            raise N.PreconditionError(f"{len(lanes)} lanes for a batch of {model.rows} rows")
        if len(max_primitives) != len(lanes) or any(p < 1 for p in max_primitives):
            raise N.PreconditionError("every lane needs a primitive budget of at least one")
        self.model, self.lanes, self.windows = model, list(lanes), windows
        self.max_primitives = list(max_primitives)
        dev = model.device
        self.streams = streams or DeviceLaneStreams(seed, self.lanes, model.rows, dev)
        self.sampler = sampler or device_sampler(alpha)
        self.bounds = [torch.tensor([[0, c]] * model.rows, dtype=torch.int32, device=dev) for _, c in windows.windows]
        self.queries = 0

    def run(self) -> list[LaneResult]:
        m, n, rows = self.model, len(self.lanes), self.model.rows
        dev = m.device
        ready = [i < n for i in range(rows)]
        active = torch.tensor(ready, dtype=torch.int32, device=dev)
        rec = torch.zeros((rows, FIELDS), dtype=torch.int32, device=dev)  # the start record
        out: list[list[np.ndarray]] = [[] for _ in range(n)]
        reason = [""] * n
        if n == 0:
            return []
        head = m.query(rec, active, True, 0)  # commits the start record; head of the first primitive
        self.queries += 1
        partial = torch.full((rows, FIELDS), PARTIAL, dtype=torch.int32, device=dev)
        while any(ready):
            on = active.bool()
            rec = torch.where(on[:, None], partial, rec)
            for f in range(FIELDS):
                if f:
                    raw = m.query(rec, active, False, f)
                    self.queries += 1
                else:
                    raw = head
                u = self.streams.draw(active)
                tok = self.sampler(raw, u, self.bounds[f], self.windows.windows[f][0])
                rec[:, f] = torch.where(on, tok.to(torch.int32), rec[:, f])
            head = m.query(rec, active, True, 0)
            self.queries += 1
            host = rec.cpu().numpy()  # the one host read per primitive
            changed = False
            for i in range(n):
                if not ready[i]:
                    continue
                out[i].append(host[i].astype(np.int64))
                if int(host[i, 0]) == self.windows.end_token:
                    reason[i], ready[i], changed = "end", False, True
                elif len(out[i]) >= self.max_primitives[i]:
                    reason[i], ready[i], changed = "limit", False, True
            if changed:
                active = torch.tensor(ready, dtype=torch.int32, device=dev)
        status = m.status_word() if hasattr(m, "status_word") else 0
        if status:
            raise N.InvalidOutputError(f"generation device status: {N.status_message(status)}")
        return [LaneResult(self.lanes[i], np.stack(out[i]), reason[i]) for i in range(n)]


class SyntheticPrimitiveModel:
    """A random-weight primitive model on the synthetic decoder: a record's
    input is the sum of its nine field embeddings (fields not predicted yet
    use a per-field empty embedding, docs/architecture.md), one decode step
    of the decoder (history in int8 arenas; reference-mode attention over the
    history plus the current token), and one output head over the attribute
    vocabulary.  Row r holds lane lanes[r]; its history is drawn from a stream
    seeded by the lane, so a lane computes the same whichever shard holds it.

    split_tokens > 0 makes every row's attention independent of the other
    rows (fixed splits instead of the stream-K balance); with the same `rows`
    on every shard, the projections also see one shape, and a lane's results
    are then bit-identical whatever shard or batch holds it."""

    def __init__(self, cfg: D.DecoderConfig, rows: int, lanes: list[int], past: list[int], capacity: int, device,
                 windows: FieldWindows, *, seed: int = 0, split_tokens: int = 0):
        if len(lanes) > rows or len(past) != len(lanes):
            raise N.PreconditionError("model rows must hold every lane, with one history length per lane")
        self.rows, self.device, self.cfg, self.windows = rows, torch.device(device), cfg, windows
        self.vocab = windows.vocab
        if capacity < max(past, default=0) + 2:
            raise N.PreconditionError("the arena needs room for the start record and at least one primitive")
        self.decoder = D.SyntheticDecoder(cfg, branches=rows, capacity=capacity, device=self.device, seed=seed,
                                          split_tokens=split_tokens)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + 1)
        self.embed = (torch.randn(self.vocab + FIELDS, cfg.width, device=self.device, generator=g) * 0.02
                      ).to(torch.bfloat16)
        self.head = (torch.randn(self.vocab, cfg.width, device=self.device, generator=g) / cfg.width ** 0.5
                     ).to(torch.bfloat16)
        self.empty = self.vocab + torch.arange(FIELDS, device=self.device, dtype=torch.int32)
        self.past = torch.zeros(rows, dtype=torch.int32, device=self.device)
        self.past[: len(past)] = torch.tensor(past, dtype=torch.int32, device=self.device)
        self._fill_lane_history(lanes, seed)

    def _fill_lane_history(self, lanes: list[int], seed: int) -> None:
        heads = self.cfg.heads
        for r, lane in enumerate(lanes):
            g = torch.Generator(device=self.device)
            g.manual_seed((seed * 1000003 + lane) & 0x7FFFFFFFFFFFFFFF)
            for a in self.decoder.arenas:
                rs = slice(r * heads, (r + 1) * heads)
                a.k[rs].random_(0, 256, generator=g)
                a.v[rs].random_(0, 256, generator=g)
                a.k_scale[rs].uniform_(0.005, 0.05, generator=g)
                a.v_scale[rs].uniform_(0.005, 0.05, generator=g)

    def query(self, rec: torch.Tensor, active: torch.Tensor, commit: bool, field: int) -> torch.Tensor:
        idx = torch.where(rec < 0, self.empty[None, :], rec)
        x = self.embed[idx.long()].float().sum(1).to(torch.bfloat16)
        lengths = torch.where(active.bool(), self.past, torch.zeros_like(self.past))
        h = self.decoder.step(x, self.past, commit=commit, lengths=lengths)
        start, count = self.windows.windows[field]
        raw = torch.matmul(h, self.head[start:start + count].t()).float()
        if commit:
            self.past += active
        return raw

    def status_word(self) -> int:
        return ops.read_status(self.decoder.status)


@dataclass
class ShardPlan:
    """The LPT partition of the lanes (by context length) over shards."""
    shard_of: list[int]
    members: list[list[int]] = field(default_factory=list)

    @classmethod
    def make(cls, costs: list[int], shards: int) -> "ShardPlan":
        shard_of, _ = kv_cache.partition_branches(costs, shards)
        return cls(shard_of, [[b for b, s in enumerate(shard_of) if s == r] for r in range(shards)])


class BranchScheduler:
    """Runs `lanes` independent generation lanes over shards.

    make_model(shard, lanes, device) builds a shard's model for its lanes
    (one batch row per lane, from row 0); costs[lane] is the lane's context
    length, the LPT key; max_primitives[lane] its primitive budget."""

    def __init__(self, make_model, costs: list[int], seed: int, max_primitives: list[int],
                 windows: FieldWindows | None = None, *, alpha: float = 4.0, make_streams=None, sampler=None):
        if not costs or len(max_primitives) != len(costs):
            raise N.PreconditionError("one context length and one primitive budget per lane")
        self.make_model, self.costs, self.seed = make_model, list(costs), seed
        self.max_primitives = list(max_primitives)
        self.windows = windows or default_windows()
        self.alpha = alpha
        # make_streams(seed, lanes, rows, device) and sampler(raw, uniforms, bounds, start) replace the device
        # streams and sampler (the host-logic tests run the cycle on the CPU with stand-ins)
        self.make_streams, self.sampler = make_streams, sampler

    def _runner(self, shard: int, lanes: list[int], device) -> ShardRunner:
        model = self.make_model(shard, lanes, device)
        streams = self.make_streams(self.seed, lanes, model.rows, device) if self.make_streams else None
        return ShardRunner(model, lanes, self.seed, [self.max_primitives[ln] for ln in lanes], self.windows,
                           alpha=self.alpha, streams=streams, sampler=self.sampler)

    def run(self, devices: list) -> dict[int, LaneResult]:
        """One process: shard s on devices[s] with its own stream and host
        thread (several shards may share a device, each on its own stream)."""
        plan = ShardPlan.make(self.costs, len(devices))
        results: dict[int, LaneResult] = {}
        errors: list[BaseException] = []
        runners = [self._runner(s, plan.members[s], devices[s]) if plan.members[s] else None
                   for s in range(len(devices))]
        torch.cuda.synchronize()

        def work(s: int):
            try:
                dev = torch.device(devices[s])
                torch.cuda.set_device(dev)
                with torch.cuda.stream(torch.cuda.Stream(dev)):
                    for r in runners[s].run():
                        results[r.lane] = r
                    torch.cuda.current_stream(dev).synchronize()
            except BaseException as e:  # reported after every shard has stopped
                errors.append(e)

        threads = [threading.Thread(target=work, args=(s,)) for s in range(len(devices)) if runners[s]]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return results

    def run_rank(self, dist, device, group=None) -> dict[int, LaneResult] | None:
        """One shard per rank of an initialised process group: this rank runs
        its LPT shard with no collective until the end, then one gather (over
        `group`, the default group when None) brings every lane's records
        (padded to the largest budget) to rank 0, which returns all lanes; the
        other ranks return None.  An NCCL communicator that exists while the
        shards generate slows CUDA-graph steps by ~5 % on B200; a caller that
        replays graphs creates the NCCL group after generation and passes it."""
        world, rank = dist.get_world_size(), dist.get_rank()
        shards = kv_cache.BranchShards(self.costs, world, rank)
        mine = shards.mine
        res = self._runner(rank, mine, device).run() if mine else []
        width = max(self.max_primitives)
        dev = torch.device(device)
        packed = torch.full((len(mine), width + 1, FIELDS), -1, dtype=torch.int64, device=dev)
        for i, r in enumerate(res):
            packed[i, 0, 0] = len(r.records)
            packed[i, 0, 1] = 1 if r.reason == "end" else 0
            packed[i, 1:1 + len(r.records)] = torch.from_numpy(r.records).to(dev)
        full = shards.gather(dist, packed, group=group)
        if full is None:
            return None
        out = {}
        for lane in range(len(self.costs)):
            row = full[lane].cpu().numpy()
            n = int(row[0, 0])
            out[lane] = LaneResult(lane, row[1:1 + n].copy(), "end" if row[0, 1] == 1 else "limit")
        return out
