"""Benchmark of the int8 historical-KV decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg1|cfg2|cfg3|cfg4|prefill|encode|float]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1, one rank per GPU)

Workload cfg1 (the one the headline metric is quoted
on): per GPU 32 independent branches x 16 heads, head_dim 128, context 4096,
one int8 K/V cache per layer for 24 layers (24 x 553.6 MB, each larger than
L2).  One step = one decode token for every branch: for each of the 24 layer
caches, a bf16 query per head -> fused int8 decode attention -> bf16 output.
Weak scaling: every rank owns 32 branches (its shard of 32*N); no collective
runs in the step; outputs are gathered to rank 0 over NCCL after timing.

Prints one JSON line (rank 0).  `value` is the aggregate attention HBM
throughput (algorithmic bytes / device time, max over ranks); `e2e` is the
same metric through the public Python API with the queries copied from
pinned host memory and the outputs read back every step.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import importlib
import json
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: branches per GPU, heads, head_dim, context, layers, description
    "cfg1": dict(branches=32, heads=16, d=128, ctx=4096, layers=24,
                 desc="BASELINE config 1: 32 branches x 16 heads x d128, context 4096, 24 layer caches, bf16 q/out"),
    "cfg4": dict(branches=8, heads=16, d=128, ctx=16384, layers=4, dist="student_t",
                 desc="BASELINE config 4: 8 branches x 16 heads x d128, context 16384, 4 layer caches, K/V "
                      "Student-t(3) x 0.7 with 1% of channels x 8"),
    # the full synthetic decoder step (per GPU: 16 branches; the box: 128 branches on 8 GPUs)
    "cfg3": dict(branches=16, heads=16, d=128, ctx=2048, layers=24, width=2048, ffn=5632,
                 desc="BASELINE config 3: synthetic decoder (24 layers, width 2048, 16x128 heads, SwiGLU 5632, "
                      "RMSNorm, RoPE 10000, random bf16 weights, int8 KV), 16 branches per GPU at context 2048"),
    # bulk encode: one layer's K and V quantized to int8 codes + scales (int8_kv_ops::quantize, row a2)
    "encode": dict(branches=32, heads=16, d=128, ctx=4096, layers=1, kv="bf16",
                   desc="encode: one cfg1 layer's K and V (512 rows x 4096 x d128, bf16 in) quantized per (token, "
                        "head) to int8 codes + f32 scales"),
    # the prefill path: one layer's whole int8 history back to bf16 (int8_cache.rs:363-371)
    "prefill": dict(branches=32, heads=16, d=128, ctx=4096, layers=1,
                    desc="prefill dequant: one cfg1 layer's int8 K and V (512 rows x 4096 x d128) to bf16"),
    # the float-KV path (fused_attention.rs): bf16 K/V at the reference kernel's head_dim 64, f32 q/out
    "float": dict(branches=32, heads=16, d=64, ctx=4096, layers=24, kv="bf16",
                  desc="float-KV decode attention: 32 branches x 16 heads x d64, bf16 K/V, context 4096, "
                       "24 layer caches, f32 q/out (the reference's F32 query and output)"),
    # the reference model's own regime (docs/architecture.md: 24 heads x 64, context 1024): reference
    # mode (history of `ctx - 1` int8 tokens + the current token as f32 scratch), f32 q/out as the
    # reference's op, 8 branches (CFG 1: one row per branch), the model's 35 layer caches
    "deployed": dict(branches=8, heads=24, d=64, ctx=1024, layers=35, refmode=True,
                     desc="the reference model's shape: 8 branches x 24 heads x d64, 1023 int8 history tokens + "
                          "the current token as f32 scratch (capacity 1024), f32 q/out, 35 layer caches"),
    # BASELINE config 0 as one call per step; 64 distinct copies of the layer are rotated so that each call
    # reads its 2.2 MB from HBM rather than L2 (64 x 2.2 MB > 126 MB)
    "cfg0": dict(branches=1, heads=16, d=64, ctx=1024, layers=64, refmode=True, per_step_calls=1,
                 desc="BASELINE config 0: 1 branch x 16 heads x d64, context 1024 (1023 int8 history tokens + the "
                      "current token as f32 scratch), f32 q/out; one call per step over 64 rotated copies"),
    # the device sampler after the output heads (fused_sampling.rs): 16 logical rows with CFG (2 physical
    # rows each) over a 2048-choice head, the whole head legal; 64 calls per step over rotated heads
    "sample": dict(branches=16, heads=1, d=0, ctx=2048, layers=64, guidance=2, alpha=4.0, cfg=1.5,
                   desc="Renyi sampling with CFG: 16 rows x 2 (CFG) x 2048 choices, alpha 4, cfg 1.5, one call "
                        "per head, 64 heads per step"),
    # ctx: mean initial context (the CPU sample's length); lengths are drawn per branch from U[lo, hi]
    "cfg2": dict(branches=64, heads=16, d=128, ctx=4224, layers=1, lo=256, hi=8192, max_steps=256,
                 desc="BASELINE config 2: 64 branches x 16 heads x d128, initial contexts U[256, 8192], per step "
                      "quantize+append one bf16 N(0, 0.5^2) K/V token per branch, then decode; one layer"),
}


def bytes_per_call(w) -> int:
    rows = w["branches"] * w["heads"]
    return rows * w["ctx"] * (2 * w["d"] + 8) + rows * w["d"] * 2 + rows * w["d"] * 2


def bytes_per_call_refmode(w) -> int:
    """Reference mode: ctx - 1 history tokens per row, the f32 scratch K and V,
    f32 q and out."""
    rows = w["branches"] * w["heads"]
    return rows * (w["ctx"] - 1) * (2 * w["d"] + 8) + rows * w["d"] * 4 * 4


def load_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def pipelined_e2e_ms(n: int, h2d, compute, d2h, stream, dev) -> float:
    """Device time of `n` end-to-end steps with the host copies on their own streams.

    Every step still copies its inputs in from pinned host memory and its
    outputs back, all inside the timed region; what changes from the serial
    loop is that step s+1's (and s+2's) host->device copies and step s-1's
    device->host copy run on the copy engines while step s computes, the way a
    serving loop overlaps them.  Two buffer slots alternate: `h2d(s, slot)`
    fills slot `slot` with step s's inputs, `compute(s, slot)` runs step s
    from it into that slot's outputs, `d2h(s, slot)` reads them back.  Events
    order each slot's reuse (inputs are overwritten only after the compute that
    read them, outputs only after the copy that read them)."""
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, done, out_read = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    up.wait_event(s0)
    down.wait_event(s0)
    for j in range(min(2, n)):
        with torch.cuda.stream(up):
            h2d(j, j)
        in_ready[j].record(up)
    for s in range(n):
        slot = s % 2
        stream.wait_event(in_ready[slot])
        if s >= 2:
            stream.wait_event(out_read[slot])
        compute(s, slot)
        done[slot].record(stream)
        down.wait_event(done[slot])
        with torch.cuda.stream(down):
            d2h(s, slot)
        out_read[slot].record(down)
        if s + 2 < n:
            up.wait_event(done[slot])
            with torch.cuda.stream(up):
                h2d(s + 2, slot)
            in_ready[slot].record(up)
    stream.wait_stream(down)
    stream.wait_stream(up)
    s1.record(stream)
    torch.cuda.synchronize()
    return s0.elapsed_time(s1)


class ClockSampler:
    """Samples SM clock, power and clock-event reasons with NVML during the timed region."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x1: "gpu_idle"}

    def __init__(self, device_index: int):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            uuid = getattr(torch.cuda.get_device_properties(device_index), "uuid", None)
            h = None
            if uuid is not None:
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
                except Exception:
                    h = None
            self.h = h or pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        if self.nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


def attention_config(args, w, world: int) -> dict:
    """The `config` object of the cfg1 / cfg4 attention lines (both arms)."""
    return {"workload": args.workload, "desc": w["desc"], "branches_per_gpu": w["branches"], "heads": w["heads"],
            "head_dim": w["d"], "context": w["ctx"], "layers": w["layers"], "split_tokens": args.split,
            "max_ctas": args.max_ctas,
            "parallelism": f"branch shards x{world} (no collective in the step)",
            "l2": "inputs larger than L2 (each layer cache > 126 MB), no flush"}


_DATA_GROUP = None


def data_group(pg):
    """The NCCL group of all ranks that carries the outputs' final gather over
    NVLink, created at its first use, after every timed region (the default
    group is gloo: barriers and timing reductions on host tensors)."""
    global _DATA_GROUP
    if _DATA_GROUP is None:
        _DATA_GROUP = pg.new_group(backend="nccl")
    return _DATA_GROUP


def per_rank(pg, dev, ms_local: float, steps: int, clocks: "ClockSampler") -> list:
    """Every rank's own device time per step and its median SM clock during
    the timed region, gathered to every rank (one all_gather, outside the
    timed region).  time x clock per rank separates a slower clock (shared
    power budget) from a rank that did more work or waited on its host."""
    c = clocks.summary()
    mine = torch.tensor([ms_local / max(1, steps), float(c["sm_mhz"] or 0.0), float(clocks.reasons)],
                        dtype=torch.float64)
    if pg is None:
        rows = [mine]
    else:
        rows = [torch.empty_like(mine) for _ in range(pg.get_world_size())]
        pg.all_gather(rows, mine)
    out = []
    for r, t in enumerate(rows):
        ms, mhz, bits = (float(x) for x in t.tolist())
        names = [n for bit, n in ClockSampler.REASONS.items() if int(bits) & bit and n != "gpu_idle"]
        out.append({"rank": r, "ms_per_step": ms, "sm_mhz": mhz or None, "reasons": names})
    return out


def cpu_reference(w, steps: int, warmup: int, sample_branches: int, threads: int, budget_s: float) -> dict:
    """The reference arithmetic restated on the CPU (oracle/), timed on a
    bounded sample of the same workload: `sample_branches` branches of one
    layer per step, all host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    rows = sample_branches * w["heads"]
    g = np.random.Generator(np.random.PCG64(1))
    k = g.integers(-127, 128, (rows, w["ctx"], w["d"]), dtype=np.int8).view(np.uint8)
    v = g.integers(-127, 128, (rows, w["ctx"], w["d"]), dtype=np.int8).view(np.uint8)
    ks = g.uniform(0.005, 0.03, (rows, w["ctx"])).astype(np.float32)
    vs = g.uniform(0.005, 0.03, (rows, w["ctx"])).astype(np.float32)
    q = oracle.bf16_round(g.standard_normal((rows, w["d"]), dtype=np.float32))
    sk = sv = None
    if w.get("refmode"):  # history of ctx - 1 tokens plus the f32 scratch token
        q = g.standard_normal((rows, w["d"]), dtype=np.float32)
        sk = g.standard_normal((rows, w["d"]), dtype=np.float32)
        sv = g.standard_normal((rows, w["d"]), dtype=np.float32)
    lens = np.full(sample_branches, w["ctx"] - (1 if w.get("refmode") else 0), np.uint32)
    per_call = (bytes_per_call_refmode(dict(w, branches=sample_branches)) if w.get("refmode") else
                rows * w["ctx"] * (2 * w["d"] + 8) + rows * w["d"] * 4)
    for _ in range(max(0, warmup)):
        oracle.attention(q, k, v, ks, vs, lens, w["heads"], sk=sk, sv=sv, threads=threads)
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        oracle.attention(q, k, v, ks, vs, lens, w["heads"], sk=sk, sv=sv, threads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    mean = sum(times) / len(times)
    return {"value": per_call / mean / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{sample_branches} branches x {w['heads']} heads x ctx {w['ctx']} x d{w['d']} of one layer "
                      f"per step, {len(times)} timed steps, oracle/int8kv_oracle.c (reference arithmetic restated)"}


def cpu_encode_reference(w, steps: int, warmup: int, sample_branches: int, threads: int, budget_s: float) -> dict:
    """The reference quantizer restated on the CPU (oracle/int8kv_oracle.c:
    int8_kv_ops.rs:13-21, one thread), timed on a bounded sample: the K of
    `sample_branches` branches of one layer per step."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    rows, L, D = sample_branches * w["heads"], w["ctx"], w["d"]
    g = np.random.Generator(np.random.PCG64(1))
    x = g.standard_normal((rows * L, D), dtype=np.float32)
    bf16 = w.get("kv", "bf16") == "bf16"
    if bf16:
        x = (x.view(np.uint32) >> 16).astype(np.uint16)
    per_call = rows * L * D * ((2 if bf16 else 4) + 1) + rows * L * 4
    for _ in range(max(0, warmup)):
        oracle.quantize(x, D)
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        oracle.quantize(x, D)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    mean = sum(times) / len(times)
    return {"value": per_call / mean / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"K of {sample_branches} branches x {w['heads']} heads x ctx {L} x d{D} "
                      f"({'bf16' if bf16 else 'f32'} in) per step, {len(times)} timed steps, one thread, "
                      f"oracle/int8kv_oracle.c (reference quantizer restated)"}


def cpu_float_reference(w, steps: int, warmup: int, sample_branches: int, threads: int, budget_s: float) -> dict:
    """The float-KV attention arithmetic restated on the CPU
    (oracle/float_attn_oracle.c), timed on a bounded sample: `sample_branches`
    branches of one layer per step, all host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    rows, L, D = sample_branches * w["heads"], w["ctx"], w["d"]
    g = np.random.Generator(np.random.PCG64(1))
    k = g.standard_normal((rows, L, D), dtype=np.float32)
    v = g.standard_normal((rows, L, D), dtype=np.float32)
    if w.get("kv", "bf16") == "bf16":
        k = (k.view(np.uint32) >> 16).astype(np.uint16)
        v = (v.view(np.uint32) >> 16).astype(np.uint16)
    q = g.standard_normal((rows, D), dtype=np.float32)
    elem = 2 if w.get("kv", "bf16") == "bf16" else 4
    per_call = rows * L * 2 * D * elem + rows * D * 8
    for _ in range(max(0, warmup)):
        oracle.float_attention(q, k, v, None, w["heads"], threads=threads)
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        oracle.float_attention(q, k, v, None, w["heads"], threads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    mean = sum(times) / len(times)
    return {"value": per_call / mean / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{sample_branches} branches x {w['heads']} heads x ctx {L} x d{D} {w.get('kv', 'bf16')} K/V of "
                      f"one layer per step, {len(times)} timed steps, oracle/float_attn_oracle.c (the reference "
                      f"kernel's arithmetic restated)"}


def run_reference_arm(args, w) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    ref = {"float": cpu_float_reference, "encode": cpu_encode_reference}.get(args.workload, cpu_reference)
    cb = ref(w, args.steps, args.warmup, sample_branches=1, threads=threads, budget_s=120.0)
    n = args.gpus
    line = {
        "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
        "impl": "reference", "value": cb["value"], "unit": "GB/s", "n_gpus": n, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"float": "bf16 KV, f32 accumulate", "encode": w.get("kv", "bf16") + " in, int8 codes + f32 scales out"}
        .get(args.workload, "int8 KV, f32 accumulate"),
        "data": "synthetic (seeded)",
        # the same workload description as this repository's arm (what was sampled is in cpu_baseline)
        "config": attention_config(args, w, n) if args.workload in ("cfg1", "cfg4") else
                  refmode_config(args, w, n) if w.get("refmode") else
                  {"workload": args.workload, "desc": w["desc"], "branches_per_gpu": w["branches"],
                   "heads": w["heads"], "head_dim": w["d"], "context": w["ctx"], "layers": w["layers"],
                   "parallelism": "replicas only (host cores)"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Candle CPU path cannot be built (no Rust toolchain); timed: its arithmetic restated in C",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_cfg2(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """ragged quantize+append then decode, one layer.

    Per GPU 64 branches with initial contexts drawn from U[256, 8192]
    (seeded); a step appends one bf16 K/V token per branch (pp_b200_quant_append
    at each branch's own offset), re-plans the ragged lengths and runs the
    decode attention over every branch's whole history.  Steps replay the same
    256 precomputed tokens, so warm-up steps rewrite identical values.
    Branches are sharded over ranks by LPT on their initial length."""
    ops, N = pp.int8_kv_ops, pp._native
    H, D = w["heads"], w["d"]
    steps = min(args.steps, w["max_steps"])
    g = np.random.Generator(np.random.PCG64(2))
    all_lens = g.integers(w["lo"], w["hi"] + 1, w["branches"] * world).astype(np.int64)
    shards = pp.kv_cache.BranchShards([int(x) for x in all_lens], world, rank)
    init = all_lens[shards.mine]
    B = len(init)
    rows = B * H
    cap = int(init.max()) + w["max_steps"]
    arena = pp.kv_cache.Int8KvArena.zeros(B, H, D, cap, dev)
    tg = torch.Generator(device=dev)
    tg.manual_seed(2 + rank)
    arena.k.random_(0, 256, generator=tg)
    arena.v.random_(0, 256, generator=tg)
    arena.k_scale.uniform_(0.005, 0.05, generator=tg)
    arena.v_scale.uniform_(0.005, 0.05, generator=tg)
    # per step s: append offsets init + s, attention lengths init + s + 1
    base = torch.tensor(init, dtype=torch.int32, device=dev)
    offs = torch.stack([base + s for s in range(steps)]).contiguous()
    lens = (offs + 1).contiguous()
    k_new = (torch.randn(steps, rows, D, device=dev, generator=tg) * 0.5).to(torch.bfloat16)
    v_new = (torch.randn(steps, rows, D, device=dev, generator=tg) * 0.5).to(torch.bfloat16)
    qs = torch.randn(steps, rows, D, device=dev, generator=tg).to(torch.bfloat16)
    outs = torch.empty(steps, rows, D, dtype=torch.bfloat16, device=dev)
    a = arena.struct()
    params = ops.attn_params(split_tokens=args.split, q_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
    ws = ops.new_workspace(a, params, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    lib = N.lib
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    ws_p, st_p = P(ws), P(status)

    def step(s: int, q=None, kn=None, vn=None, out=None):
        q = qs[s] if q is None else q
        kn = k_new[s] if kn is None else kn
        vn = v_new[s] if vn is None else vn
        out = outs[s] if out is None else out
        N.check(lib.pp_b200_quant_append(C.byref(a), P(kn), P(vn), N.DTYPE_BF16, P(offs[s]), 1, st_p, sp))
        N.check(lib.pp_b200_decode_attention(C.byref(a), C.byref(params), P(q), None, None, P(lens[s]), P(out),
                                             ws_p, ws.numel(), st_p, sp))

    for s in range(min(args.warmup, steps)):
        step(s)
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise SystemExit(f"device status after warm-up: {N.status_message(int(status.item()))}")

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64)
        if pg is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for s in range(steps):
            step(s)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_local = start.elapsed_time(end)
    ranks = per_rank(pg, dev, ms_local, steps, clocks)
    ms_step = max_over_ranks(ms_local) / steps

    # bytes: attention reads every branch's whole history once, plus q, out and the append
    hist = float(sum((init + s + 1).sum() for s in range(steps))) / steps  # mean tokens per branch-row set
    attn_bytes = hist * H * (2 * D + 8) + rows * D * 2 * 2
    append_bytes = rows * (2 * D * 2 + 2 * D + 8)
    per_step = attn_bytes + append_bytes
    peak, peak_kind = load_peaks()
    value = world * per_step / (ms_step * 1e-3) / 1e9
    achieved = per_step / (ms_local / steps * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        q_h = qs.cpu().pin_memory()
        k_h = k_new.cpu().pin_memory()
        v_h = v_new.cpu().pin_memory()
        o_h = torch.empty(outs.shape, dtype=outs.dtype).pin_memory()
        q_d, k_d, v_d = torch.empty_like(qs[0]), torch.empty_like(k_new[0]), torch.empty_like(v_new[0])
        o_d = torch.empty_like(outs[0])
        e_steps = min(steps, 64)

        def e2e_step(s):
            q_d.copy_(q_h[s], non_blocking=True)
            k_d.copy_(k_h[s], non_blocking=True)
            v_d.copy_(v_h[s], non_blocking=True)
            arena.append(k_d, v_d, offs[s])
            ops.decode_attention(q_d, arena.k, arena.v, arena.k_scale, arena.v_scale, lens[s], H,
                                 out_dtype=torch.bfloat16, split_tokens=args.split, workspace=ws, out=o_d)
            o_h[s].copy_(o_d, non_blocking=True)

        for s in range(min(args.warmup, e_steps)):
            e2e_step(s)
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for s in range(e_steps):
            e2e_step(s)
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        serial_ms = max_over_ranks(s0.elapsed_time(s1) / e_steps)

        # the same steps with the host copies overlapped on copy streams (two slots)
        q2, k2, v2, o2 = ([torch.empty_like(t[0]) for _ in range(2)] for t in (qs, k_new, v_new, outs))

        def up(s, j):
            q2[j].copy_(q_h[s], non_blocking=True)
            k2[j].copy_(k_h[s], non_blocking=True)
            v2[j].copy_(v_h[s], non_blocking=True)

        def run(s, j):
            arena.append(k2[j], v2[j], offs[s])
            ops.decode_attention(q2[j], arena.k, arena.v, arena.k_scale, arena.v_scale, lens[s], H,
                                 out_dtype=torch.bfloat16, split_tokens=args.split, workspace=ws, out=o2[j])

        def down(s, j):
            o_h[s].copy_(o2[j], non_blocking=True)

        pipelined_e2e_ms(min(args.warmup, e_steps), up, run, down, stream, dev)
        barrier()
        e_ms = max_over_ranks(pipelined_e2e_ms(e_steps, up, run, down, stream, dev) / e_steps)
        barrier()
        e2e = {"value": world * per_step / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": 3 * rows * D * 2, "d2h_bytes_per_step": rows * D * 2, "ms_per_step": e_ms,
               "tokens_per_s": world * B / (e_ms * 1e-3), "copies": "overlapped on two copy streams",
               "serial_value": world * per_step / (serial_ms * 1e-3) / 1e9, "serial_ms_per_step": serial_ms}

    if pg is not None:
        shards.gather(pg, outs[steps - 1].view(B, H, D).contiguous(), group=data_group(pg))

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(w, steps=3, warmup=1, sample_branches=1, threads=os.cpu_count() or 1, budget_s=20.0)

    if rank == 0:
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 KV (bf16-rounded dequant), bf16 K/V in, bf16 q/out, f32 accumulate",
            "data": "synthetic (seeded)",
            "config": {"workload": "cfg2", "desc": w["desc"], "branches_per_gpu": B, "heads": H, "head_dim": D,
                       "capacity": cap, "mean_context": hist / B, "split_tokens": args.split,
                       "parallelism": f"branch shards x{world} by LPT on context (no collective in the step)",
                       "l2": "history read per step > 126 MB L2, no flush"},
            "tokens_per_s": world * B / (ms_step * 1e-3),
            "percent_of_peak": 100.0 * value / (world * peak),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind, "per_launch_bytes": per_step,
                         "per_launch_ms": ms_local / steps,
                         "timed": "timed region / steps: append + plan + attention per step (CUDA events)"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None,
            "e2e": e2e,
            "gpu_launches": steps * (4 if args.split else 3),  # append, plan, attention (+ combine)
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0



def run_cfg3(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """the whole decode step of a synthetic 1B-class decoder.

    Per GPU 16 branches whose int8 caches already hold 2048 tokens (random
    codes and scales); a step decodes one token for every branch through all
    24 layers (RMSNorm, QKV projection, fused q/k RMSNorm + RoPE + int8 append,
    int8 decode attention over history + the new token, output projection,
    RMSNorm, gate/up projection, SwiGLU, down projection) and the final
    RMSNorm.  Projections are cuBLAS GEMMs; the rest are this library's
    kernels.  Each step appends at the next slot, so the context grows by one
    token per step.  Branches are independent: no collective in the step."""
    D = pp.decoder
    cfg = D.DecoderConfig(layers=w["layers"], width=w["width"], heads=w["heads"], head_dim=w["d"],
                          ffn_hidden=w["ffn"], max_context=w["ctx"] + args.warmup + args.steps + 8)
    B, L0 = w["branches"], w["ctx"]
    steps = args.steps
    model = D.SyntheticDecoder(cfg, branches=B, capacity=cfg.max_context, device=dev, seed=1234 + rank)
    model.fill_history(None, seed=99 + rank)
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    n_in = args.warmup + steps
    xs = (torch.randn(n_in, B, cfg.width, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    past = torch.stack([torch.full((B,), L0 + s, dtype=torch.int32, device=dev) for s in range(n_in)]).contiguous()
    stream = torch.cuda.current_stream(dev)
    outs = []
    for s in range(args.warmup):
        model.step(xs[s].clone(), past[s])
    torch.cuda.synchronize()
    if int(model.status.item()) != 0:
        raise SystemExit(f"device status after warm-up: {pp._native.status_message(int(model.status.item()))}")
    work = [xs[args.warmup + s].clone() for s in range(steps)]
    graph = None
    if not args.no_graph:
        # the whole step as one CUDA graph: the history length advances by one per replay
        past_live = past[args.warmup].clone()
        graph = model.capture(past_live, advance=True)
        past_live.copy_(past[args.warmup])
        torch.cuda.synchronize()

    def run_step(s: int) -> torch.Tensor:
        if graph is not None:
            return graph.replay(work[s])
        return model.step(work[s], past[args.warmup + s])

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64)
        if pg is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for s in range(steps):
            outs.append(run_step(s))
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_local = start.elapsed_time(end)
    ranks = per_rank(pg, dev, ms_local, steps, clocks)
    ms_step = max_over_ranks(ms_local) / steps
    tokens_per_s = world * B / (ms_step * 1e-3)

    # bytes a step must move: every weight once, every layer's history once, the new K/V
    rows = B * cfg.heads
    mean_hist = L0 + args.warmup + (steps - 1) / 2.0
    kv_bytes = cfg.layers * rows * mean_hist * (2 * cfg.head_dim + 8)
    per_step = model.weight_bytes() + kv_bytes
    peak, peak_kind = load_peaks()
    achieved = per_step / (ms_local / steps * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        x_h = xs[args.warmup:].cpu().pin_memory()
        o_h = torch.empty((steps, B, cfg.width), dtype=torch.bfloat16).pin_memory()
        x_d = torch.empty(B, cfg.width, dtype=torch.bfloat16, device=dev)
        e_steps = min(steps, 20)
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if graph is not None:
            graph.past.copy_(past[args.warmup])
        s0.record(stream)
        for s in range(e_steps):
            x_d.copy_(x_h[s], non_blocking=True)
            o_h[s].copy_(graph.replay(x_d) if graph is not None else model.step(x_d, past[args.warmup + s]),
                         non_blocking=True)
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(s0.elapsed_time(s1) / e_steps)
        e2e = {"value": world * B / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": B * cfg.width * 2,
               "d2h_bytes_per_step": B * cfg.width * 2, "ms_per_step": e_ms}

    if pg is not None:
        shards = pp.kv_cache.BranchShards([L0] * (B * world), world, rank)
        shards.gather(pg, outs[-1].contiguous(), group=data_group(pg))

    if rank == 0:
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 weights/activations, int8 KV, f32 accumulate", "data": "synthetic (seeded, random weights)",
            "config": {"workload": "cfg3", "desc": w["desc"], "branches_per_gpu": B, "layers": cfg.layers,
                       "width": cfg.width, "heads": cfg.heads, "head_dim": cfg.head_dim, "ffn_hidden": cfg.ffn_hidden,
                       "context": L0, "parameters": cfg.parameters(), "cuda_graph": graph is not None,
                       "projections": "cuBLAS (torch.matmul), outside this library's kernels",
                       "parallelism": f"branch shards x{world}, weights replicated (no collective in the step)",
                       "l2": "weights 2.5 GB + history 3.3 GB per step, larger than L2; no flush"},
            "tokens_per_s": tokens_per_s,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind, "per_launch_bytes": per_step,
                         "per_launch_ms": ms_local / steps,
                         "timed": "whole decode step (weights + int8 history bytes) per step, CUDA events"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None,
            "e2e": e2e,
            # plan; per layer 2 rmsnorm, qkv_rope_append, attention, swiglu (+ 4 decode-row GEMMs); final rmsnorm
            "gpu_launches": steps * (1 + cfg.layers * 5 + 1),
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0



def run_encode(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """Bulk encode (int8_kv_ops::quantize, int8_kv_ops.rs:11-27; the CUDA
    branch pp_i8_scale + pp_i8_pack, int8_kv.cu:8-18): one layer's K and V
    quantized per (token, head) row, bf16 (default) or f32 in; no collective."""
    rows, L, D = w["branches"] * w["heads"], w["ctx"], w["d"]
    n = rows * L
    t = torch.bfloat16 if w.get("kv", "bf16") == "bf16" else torch.float32
    elem = 2 if t == torch.bfloat16 else 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    xs = [torch.randn(n, D, device=dev, generator=gen).to(t) for _ in range(2)]
    codes = [torch.empty(n, D, dtype=torch.uint8, device=dev) for _ in range(2)]
    scales = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(2)]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    lib, N = pp._native.lib, pp._native
    P = lambda t_: C.c_void_p(t_.data_ptr())  # noqa: E731
    sp = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    dt = N.DTYPE_BF16 if t == torch.bfloat16 else N.DTYPE_F32

    def step():
        for j in range(2):
            N.check(lib.pp_b200_quantize(P(xs[j]), dt, n, D, P(codes[j]), P(scales[j]), P(status), sp))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise SystemExit(f"device status after warm-up: {N.status_message(int(status.item()))}")
    stream = torch.cuda.current_stream(dev)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    ms_local = e0.elapsed_time(e1) / args.steps
    ranks = per_rank(pg, dev, ms_local, 1, clocks)
    tt = torch.tensor([ms_local], dtype=torch.float64)
    if pg is not None:
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
    ms_step = float(tt.item())
    per_call = n * D * (elem + 1) + n * 4
    per_step = 2 * per_call
    peak, peak_kind = load_peaks()
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_encode_reference(w, steps=3, warmup=1, sample_branches=1, threads=1, budget_s=20.0)
    if rank == 0:
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": world * per_step / (ms_step * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": f"{'bf16' if elem == 2 else 'f32'} in, int8 codes + f32 scales out",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": "encode", "desc": w["desc"], "rows": rows, "context": L, "head_dim": D,
                       "input": "bf16" if elem == 2 else "f32",
                       "l2": f"{per_step / 1e9:.2f} GB per step, larger than L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": per_step / (ms_local * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": per_step / (ms_local * 1e-3) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                         "per_launch_bytes": per_call, "per_launch_ms": ms_local / 2,
                         "timed": "two quantize calls (K, V) per step, CUDA events"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None, "e2e": None, "gpu_launches": 2 * args.steps, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


def run_prefill(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """The prefill dequant path: one layer's int8 K and V histories back to
    bf16 (Int8LayerCache::prefill_prefix, int8_cache.rs:363-371), 1.6 GB of
    codes, scales and bf16 per step on each GPU; no collective."""
    ops = pp.int8_kv_ops
    rows, L, D = w["branches"] * w["heads"], w["ctx"], w["d"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(5 + rank)
    k = torch.randint(0, 256, (rows, L, D), dtype=torch.uint8, device=dev, generator=gen)
    v = torch.randint(0, 256, (rows, L, D), dtype=torch.uint8, device=dev, generator=gen)
    ks = torch.rand(rows, L, device=dev, generator=gen) * 0.05
    vs = torch.rand(rows, L, device=dev, generator=gen) * 0.05
    kb = torch.empty(rows, L, D, dtype=torch.bfloat16, device=dev)
    vb = torch.empty_like(kb)
    lib, N = pp._native.lib, pp._native
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    sp = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def step():
        for codes, sc, out in ((k, ks, kb), (v, vs, vb)):
            N.check(lib.pp_b200_dequantize(P(codes), P(sc), rows * L, D, 1, N.DTYPE_BF16, P(out), sp))

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.current_stream(dev)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    ms_local = e0.elapsed_time(e1) / args.steps
    ranks = per_rank(pg, dev, ms_local, 1, clocks)
    t = torch.tensor([ms_local], dtype=torch.float64)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_step = float(t.item())
    per_step = 2 * (rows * L * D * (1 + 2) + rows * L * 4)
    peak, peak_kind = load_peaks()
    if rank == 0:
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": world * per_step / (ms_step * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 codes -> bf16(i8 * scale)", "data": "synthetic (seeded)",
            "config": {"workload": "prefill", "desc": w["desc"], "rows": rows, "context": L, "head_dim": D,
                       "l2": "1.6 GB per step, larger than L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": per_step / (ms_local * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": per_step / (ms_local * 1e-3) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                         "per_launch_bytes": per_step / 2, "per_launch_ms": ms_local / 2,
                         "timed": "two dequantize calls (K, V) per step, CUDA events"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None, "e2e": None, "gpu_launches": 2 * args.steps, "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0



def run_float(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """The float-KV decode path (fused_attention::decode_attention): per step
    one plan, then one pp_b200_decode_attention_float per layer cache; branch
    shards per rank as the int8 path, no collective in the step."""
    fa, ops, N = pp.fused_attention, pp.int8_kv_ops, pp._native
    B, H, D, L, layers = w["branches"], w["heads"], w["d"], w["ctx"], w["layers"]
    rows = B * H
    kv_t = torch.bfloat16 if w.get("kv", "bf16") == "bf16" else torch.float32
    elem = 2 if kv_t == torch.bfloat16 else 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)
    caches = [(torch.randn(rows, L, D, device=dev, generator=gen).to(kv_t),
               torch.randn(rows, L, D, device=dev, generator=gen).to(kv_t)) for _ in range(layers)]
    lengths = torch.full((B,), L, dtype=torch.int32, device=dev)
    qs = torch.randn(layers, rows, D, device=dev, generator=gen)
    outs = torch.empty(layers, rows, D, device=dev)
    kvs = [fa.kv_struct(k, v, H) for k, v in caches]
    params = ops.attn_params(split_tokens=args.split)
    p_ready = ops.attn_params(split_tokens=args.split, plan_ready=True)
    p_pref = ops.attn_params(split_tokens=args.split, plan_ready=True, prefetch_history=not args.no_prefetch)
    ws = torch.empty(fa.workspace_bytes(kvs[0], params), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp, lib = C.c_void_p(stream.cuda_stream), N.lib
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    lens_p, ws_p, st_p = P(lengths), P(ws), P(status)
    q_ptrs = [P(qs[i]) for i in range(layers)]
    o_ptrs = [P(outs[i]) for i in range(layers)]
    kv_refs = [C.byref(g) for g in kvs]

    def step():
        N.check(lib.pp_b200_plan_ragged_float(kv_refs[0], C.byref(params), lens_p, ws_p, ws.numel(), sp))
        for i in range(layers):
            N.check(lib.pp_b200_decode_attention_float(kv_refs[i], C.byref(p_pref if i else p_ready), q_ptrs[i], D,
                                                       lens_p, o_ptrs[i], ws_p, ws.numel(), st_p, sp))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise SystemExit(f"device status after warm-up: {N.status_message(int(status.item()))}")

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64)
        if pg is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_local = e0.elapsed_time(e1)
    ranks = per_rank(pg, dev, ms_local, args.steps, clocks)
    ms_step = max_over_ranks(ms_local) / args.steps
    call_ms = ms_local / (args.steps * layers)
    per_call = rows * L * 2 * D * elem + rows * D * 4 + rows * D * 4
    peak, peak_kind = load_peaks()

    e2e = None
    if not args.no_e2e:
        q_host = qs.cpu().pin_memory()
        o_host = torch.empty(outs.shape, dtype=outs.dtype).pin_memory()
        q_dev = torch.empty_like(qs)

        def e2e_step():
            q_dev.copy_(q_host, non_blocking=True)
            fa.plan_ragged(caches[0][0], caches[0][1], lengths, H, ws, split_tokens=args.split)
            for i, (k, v) in enumerate(caches):
                fa.decode_attention(q_dev[i].unsqueeze(1), k, v, lengths, H, args.split, workspace=ws,
                                    plan_ready=True, prefetch_history=i > 0 and not args.no_prefetch,
                                    out=outs[i].unsqueeze(1))
            o_host.copy_(outs, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        e_steps = max(1, min(args.steps, 50))
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        serial_ms = max_over_ranks(s0.elapsed_time(s1) / e_steps)

        # the same steps with the host copies overlapped on copy streams (two slots)
        q2, o2 = [torch.empty_like(qs) for _ in range(2)], [torch.empty_like(outs) for _ in range(2)]

        def up(s, j):
            q2[j].copy_(q_host, non_blocking=True)

        def run(s, j):
            fa.plan_ragged(caches[0][0], caches[0][1], lengths, H, ws, split_tokens=args.split)
            for i, (k, v) in enumerate(caches):
                fa.decode_attention(q2[j][i].unsqueeze(1), k, v, lengths, H, args.split, workspace=ws,
                                    plan_ready=True, prefetch_history=i > 0 and not args.no_prefetch,
                                    out=o2[j][i].unsqueeze(1))

        def down(s, j):
            o_host.copy_(o2[j], non_blocking=True)

        pipelined_e2e_ms(max(1, args.warmup), up, run, down, stream, dev)
        barrier()
        e_ms = max_over_ranks(pipelined_e2e_ms(e_steps, up, run, down, stream, dev) / e_steps)
        barrier()
        e2e = {"value": world * layers * per_call / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": q_host.numel() * q_host.element_size(),
               "d2h_bytes_per_step": o_host.numel() * o_host.element_size(), "ms_per_step": e_ms,
               "tokens_per_s": world * B / (e_ms * 1e-3), "copies": "overlapped on two copy streams",
               "serial_value": world * layers * per_call / (serial_ms * 1e-3) / 1e9, "serial_ms_per_step": serial_ms}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_float_reference(w, steps=3, warmup=1, sample_branches=1, threads=os.cpu_count() or 1,
                                  budget_s=20.0)
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                traffic = json.load(f).get("float" if kv_t == torch.bfloat16 else "float_f32")
        except Exception:
            traffic = None
    if rank == 0:
        value = world * layers * per_call / (ms_step * 1e-3) / 1e9
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"{w.get('kv', 'bf16')} KV, f32 q/out, f32 accumulate", "data": "synthetic (seeded)",
            "config": {"workload": "float", "desc": w["desc"], "branches_per_gpu": B, "heads": H, "head_dim": D,
                       "context": L, "layers": layers, "kv_dtype": w.get("kv", "bf16"), "split_tokens": args.split,
                       "parallelism": f"branch shards x{world} (no collective in the step)",
                       "l2": "inputs larger than L2 (each layer cache > 126 MB), no flush"},
            "tokens_per_s": world * B / (ms_step * 1e-3),
            "percent_of_peak": 100.0 * value / (world * peak),
            "roofline": {"bound": "hbm", "achieved": per_call / (call_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": per_call / (call_ms * 1e-3) / 1e9 / peak, "traffic": traffic,
                         "peak_kind": peak_kind, "per_launch_bytes": per_call, "per_launch_ms": call_ms,
                         "timed": "timed region / attention calls (CUDA events on the launching stream): "
                                  "attn_kernel over float rows, with the plan amortised over the step"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None, "e2e": e2e,
            "gpu_launches": args.steps * (1 + (2 if args.split else 1) * layers),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def refmode_inputs(w, dev, seed: int):
    """Per-layer int8 caches (N(0,1) quantized per (token, head)), f32
    queries and f32 scratch K/V for every layer, and the per-branch history
    length ctx - 1 (the token at index ctx - 1 is the scratch token)."""
    from importlib import import_module

    ops = import_module("pop2-bezier_b200").int8_kv_ops
    rows, D, cap, layers = w["branches"] * w["heads"], w["d"], w["ctx"], w["layers"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    caches = []
    for _ in range(layers):
        k, ks = ops.quantize(torch.randn(rows, cap, D, device=dev, generator=gen), check_finite=False)
        v, vs = ops.quantize(torch.randn(rows, cap, D, device=dev, generator=gen), check_finite=False)
        caches.append((k, v, ks, vs))
    qs = torch.randn(layers, rows, D, device=dev, generator=gen)
    sks = torch.randn(layers, rows, D, device=dev, generator=gen)
    svs = torch.randn(layers, rows, D, device=dev, generator=gen)
    past = torch.full((w["branches"],), cap - 1, dtype=torch.int32, device=dev)
    return caches, qs, sks, svs, past


def refmode_plan(w):
    """(calls per step, layer copy of call i in step s): the deployed step is
    one call per layer cache; cfg0 is one call per step over rotated copies."""
    if w.get("per_step_calls"):
        return w["per_step_calls"], (lambda s, i: s % w["layers"])
    return w["layers"], (lambda s, i: i)


def run_refmode(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """Reference-mode attention at the reference model's own shapes (workloads
    `deployed` and `cfg0`): per call, ctx - 1 int8 history tokens per row plus
    the current token as f32 scratch, f32 q and out, the reference's head_dim
    64 and 1024-token capacity (int8_kv_ops.rs:44).  A step plans once (the
    lengths are shared by the step's calls) and runs its calls; layers after
    the first stream their history while the previous call finishes."""
    ops, N = pp.int8_kv_ops, pp._native
    H, D = w["heads"], w["d"]
    caches, qs, sks, svs, past = refmode_inputs(w, dev, 1234 + rank)
    calls, layer_of = refmode_plan(w)
    outs = torch.empty_like(qs)
    arenas = [ops.arena_struct(k, v, ks, vs, H) for (k, v, ks, vs) in caches]
    mk = lambda ready, pf: ops.attn_params(q_dtype=torch.float32, out_dtype=torch.float32, plan_ready=ready,  # noqa
                                           prefetch_history=pf and not args.no_prefetch, max_ctas=args.max_ctas)
    params, p_ready, p_pf = mk(False, False), mk(True, False), mk(True, True)
    ws = ops.new_workspace(arenas[0], params, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    lib = N.lib
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    ws_p, st_p, past_p = P(ws), P(status), P(past)

    def enqueue(s: int, sp):
        N.check(lib.pp_b200_plan_ragged(C.byref(arenas[layer_of(s, 0)]), C.byref(params), past_p, 1, ws_p,
                                        ws.numel(), sp))
        for i in range(calls):
            li = layer_of(s, i)
            N.check(lib.pp_b200_decode_attention(C.byref(arenas[li]), C.byref(p_pf if i else p_ready), P(qs[li]),
                                                 P(sks[li]), P(svs[li]), past_p, P(outs[li]), ws_p, ws.numel(),
                                                 st_p, sp))

    for s in range(args.warmup):
        enqueue(s, sp)
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise SystemExit(f"device status after warm-up: {N.status_message(int(status.item()))}")
    # a call moves a few MB in a few microseconds, less than a launch from Python costs: each step pattern is
    # recorded once as a CUDA graph (one per rotated copy for cfg0) and replayed, so the device never waits
    # for the host
    graphs = capture_steps(lambda s, sp_: enqueue(s, sp_), w, dev)

    def step(s: int):
        graphs[s % len(graphs)].replay()

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64)
        if pg is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for s in range(args.steps):
            step(s)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_local = start.elapsed_time(end)
    ranks = per_rank(pg, dev, ms_local, args.steps, clocks)
    ms_step = max_over_ranks(ms_local) / args.steps
    per_call = bytes_per_call_refmode(w)
    call_us = ms_local / (args.steps * calls) * 1e3
    value = world * calls * per_call / (ms_step * 1e-3) / 1e9
    peak, peak_kind = load_peaks()
    achieved = per_call / (call_us * 1e-6) / 1e9

    e2e = None
    if not args.no_e2e:
        # The public Python API with every call's q and scratch K/V copied in from pinned host memory and its
        # output read back, all inside the timed region.  A call's three inputs sit side by side in one pinned
        # block [3, rows, d] and go up as one copy on an upload stream, ahead of the calls; the calls wait for
        # their inputs in chunks of 1, 1, 2, 4, 8 ... calls, so that few waits break the chain of dependent
        # launches whose history reads start before the previous call ends.  Each output goes down on a
        # download stream once its call has finished.  The step (copies, plan, calls) is recorded as a CUDA
        # graph per step pattern and replayed.
        h_in = torch.stack((qs, sks, svs), dim=1).cpu().pin_memory()  # [layers, 3, rows, d]
        ho = torch.empty(outs.shape, dtype=outs.dtype).pin_memory()
        d_in = torch.empty((calls,) + tuple(h_in.shape[1:]), dtype=h_in.dtype, device=dev)
        up_s, dn_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(calls)]
        ev_done = [torch.cuda.Event() for _ in range(calls)]
        k0, v0, ks0, vs0 = caches[0]
        chunk_end = {}  # first call of a chunk -> one past its last call
        c0 = 0
        while c0 < calls:
            chunk_end[c0] = min(calls, max(1, 2 * c0))
            c0 = chunk_end[c0]

        def e2e_step(s: int):
            cur = torch.cuda.current_stream(dev)
            up_s.wait_stream(cur)
            dn_s.wait_stream(cur)
            with torch.cuda.stream(up_s):
                for i in range(calls):
                    d_in[i].copy_(h_in[layer_of(s, i)], non_blocking=True)
                    ev_in[i].record(up_s)
            ops.plan_ragged(k0, v0, ks0, vs0, past, H, ws, scratch=True, max_ctas=args.max_ctas)
            for i in range(calls):
                li = layer_of(s, i)
                if i in chunk_end:
                    cur.wait_event(ev_in[chunk_end[i] - 1])
                k, v, ks, vs = caches[li]
                ops.decode_attention(d_in[i, 0], k, v, ks, vs, past, H, scratch_k=d_in[i, 1], scratch_v=d_in[i, 2],
                                     out_dtype=torch.float32, workspace=ws, plan_ready=True, out=outs[li],
                                     max_ctas=args.max_ctas, prefetch_history=i > 0 and not args.no_prefetch)
                ev_done[i].record(cur)
                dn_s.wait_event(ev_done[i])
                with torch.cuda.stream(dn_s):
                    ho[li].copy_(outs[li], non_blocking=True)
            cur.wait_stream(up_s)
            cur.wait_stream(dn_s)

        for s in range(max(1, args.warmup)):
            e2e_step(s)
        e_steps = max(1, min(args.steps, 50))
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for s in range(e_steps):
            e2e_step(s)
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        eager_ms = max_over_ranks(s0.elapsed_time(s1) / e_steps)
        e_graphs = capture_steps(lambda s_, sp_: e2e_step(s_), w, dev)
        for s in range(max(1, args.warmup)):
            e_graphs[s % len(e_graphs)].replay()
        barrier()
        s0.record(stream)
        for s in range(e_steps):
            e_graphs[s % len(e_graphs)].replay()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(s0.elapsed_time(s1) / e_steps)
        del e_graphs
        ok = torch.equal(ho[layer_of(e_steps - 1, calls - 1)], outs[layer_of(e_steps - 1, calls - 1)].cpu())
        e2e = {"value": world * calls * per_call / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": calls * h_in[0].numel() * 4, "d2h_bytes_per_step": calls * qs[0].numel() * 4,
               "ms_per_step": e_ms, "us_per_call": e_ms * 1e3 / calls, "read_back_matches": ok,
               "copies": "one packed upload per call on an upload stream (calls wait in chunks of 1, 1, 2, 4 ... "
                         "calls), one download per call on a download stream, both overlapping the calls; "
                         "the step replayed as a CUDA graph",
               "eager_value": world * calls * per_call / (eager_ms * 1e-3) / 1e9, "eager_ms_per_step": eager_ms}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(w, steps=20, warmup=2, sample_branches=w["branches"], threads=os.cpu_count() or 1,
                            budget_s=10.0)

    if rank == 0:
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "us_per_call": call_us, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 KV (bf16-rounded dequant), f32 scratch token, f32 q/out, f32 accumulate",
            "data": "synthetic (seeded)",
            "config": refmode_config(args, w, world),
            "tokens_per_s": world * w["branches"] / (ms_step * 1e-3) if not w.get("per_step_calls") else None,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind, "per_launch_bytes": per_call,
                         "per_launch_ms": call_us * 1e-3,
                         "timed": "timed region / attention calls (CUDA events), the step's plan charged to its calls"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None,
            "e2e": e2e,
            "gpu_launches": args.steps * (1 + calls),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def capture_steps(enqueue, w, dev) -> list:
    """One CUDA graph per distinct step of a reference-mode workload: a single
    graph for `deployed` (every step is the same plan + 35 calls), one per
    rotated layer copy for cfg0.  enqueue(s, stream_pointer) issues step s."""
    n = w["layers"] if w.get("per_step_calls") else 1
    graphs = []
    for s in range(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            enqueue(s, C.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
        graphs.append(g)
    torch.cuda.synchronize()
    return graphs


def refmode_config(args, w, world: int) -> dict:
    return {"workload": args.workload, "desc": w["desc"], "branches_per_gpu": w["branches"], "heads": w["heads"],
            "head_dim": w["d"], "capacity": w["ctx"], "history": w["ctx"] - 1, "layers": w["layers"],
            "calls_per_step": refmode_plan(w)[0], "mode": "reference (f32 scratch token)", "cuda_graph": True,
            "max_ctas": args.max_ctas,
            "parallelism": f"branch shards x{world} (no collective in the step)",
            "l2": "the rotated layer caches together exceed L2; no flush"}


def run_reference_kernels(args, w) -> int:
    """The reference's own CUDA kernels (pp_i8_attention + pp_i8_merge,
    app/src/model/int8_kv.cu, compiled from the reference sources into
    oracle/_ref/ with its NVRTC options) on the same inputs and steps as
    run_refmode, launched with the reference's geometry (int8_kv_ops.rs:
    143-161: grid (rows, ceil((capacity+1)/split)), 128 threads, split 128,
    then a 64-thread merge per row).  Partials and outputs are allocated once
    (the reference allocates them per call)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref_runner

    if not ref_runner.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/int8_kv_ref.cubin was not built "
                          "(the reference tree was absent when build() ran)"}), flush=True)
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    caches, qs, sks, svs, past = refmode_inputs(w, dev, 1234)
    kern = ref_runner.RefInt8Kernels()
    rows, D, cap = w["branches"] * w["heads"], w["d"], w["ctx"]
    split = 128
    splits = (cap + 1 + split - 1) // split
    partial = torch.empty(rows * splits * 66, dtype=torch.float32, device=dev)
    outs = torch.empty_like(qs)
    calls, layer_of = refmode_plan(w)

    def enqueue(s: int, sp=None):
        for i in range(calls):
            li = layer_of(s, i)
            k, v, ks, vs = caches[li]
            kern._launch("pp_i8_attention", (rows, splits), 128, (split + 128) * 4,
                         [qs[li], k, v, ks, vs, sks[li], svs[li], past, partial, C.c_uint32(w["heads"]),
                          C.c_uint32(cap), C.c_uint32(split), C.c_uint32(splits)])
            kern._launch("pp_i8_merge", (rows, 1), 64, 0, [partial, outs[li], C.c_uint32(splits)])

    for s in range(args.warmup):
        enqueue(s)
    torch.cuda.synchronize()
    # recorded as CUDA graphs exactly as this repository's arm is (the reference launches from Rust, where a
    # launch costs the host less than from Python)
    graphs = capture_steps(enqueue, w, dev)

    def step(s: int):
        graphs[s % len(graphs)].replay()
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        start.record(stream)
        for s in range(args.steps):
            step(s)
        end.record(stream)
        torch.cuda.synchronize()
    ms_step = start.elapsed_time(end) / args.steps
    per_call = bytes_per_call_refmode(w)
    value = calls * per_call / (ms_step * 1e-3) / 1e9
    line = {
        "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
        "impl": "reference", "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "us_per_call": ms_step * 1e3 / calls,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 KV (bf16-rounded dequant), f32 scratch token, f32 q/out, f32 accumulate",
        "data": "synthetic (seeded)", "config": refmode_config(args, w, 1), "clocks": clocks.summary(),
        "reference_kernels": "pp_i8_attention + pp_i8_merge (app/src/model/int8_kv.cu) compiled for sm_100a with "
                             "fmad=false, prec_div=true; launch geometry of int8_kv_ops.rs:143-161, split 128; "
                             "each step pattern replayed as a CUDA graph",
        "gpu_launches": args.steps * 2 * calls,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def sample_inputs(w, dev, seed: int):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    B, n, calls = w["branches"], w["ctx"], w["layers"]
    raw = torch.randn(calls, B * w["guidance"], n, device=dev, generator=g) * 3
    uni = torch.rand(calls, B, device=dev, generator=g)
    bounds = torch.tensor([[0, n]] * B, dtype=torch.int32, device=dev)
    return raw, uni, bounds


def run_sample(args, w, pp, pg, world: int, rank: int, local: int, dev) -> int:
    """The device Rényi sampler (pp_b200_renyi_sample): 64 calls per step,
    each over its own head, recorded once as a CUDA graph and replayed (a
    call takes microseconds, less than a launch from Python)."""
    raw, uni, bounds = sample_inputs(w, dev, 5 + rank)
    B, n, calls = w["branches"], w["ctx"], w["layers"]
    out = torch.empty(calls, 3, B, dtype=torch.int32, device=dev)
    N, ops = pp._native, pp.int8_kv_ops

    def enqueue(sp):
        for i in range(calls):
            N.check(N.lib.pp_b200_renyi_sample(ops._ptr(raw[i]), ops._ptr(uni[i]), ops._ptr(bounds), ops._ptr(out[i]),
                                               B, n, w["guidance"], w["alpha"], w["cfg"], 0, sp))

    stream = torch.cuda.current_stream(dev)
    enqueue(C.c_void_p(stream.cuda_stream))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        enqueue(C.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if pg is not None:
        pg.barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
    ms_local = start.elapsed_time(end)
    ranks = per_rank(pg, dev, ms_local, args.steps, clocks)
    t = torch.tensor([ms_local], dtype=torch.float64)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    per_call = raw[0].numel() * 4 + uni[0].numel() * 4 + bounds.numel() * 4 + out[0].numel() * 4
    us = ms_local / (args.steps * calls) * 1e3
    peak, peak_kind = load_peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": world * calls * B / (ms_step * 1e-3), "unit": "sampled rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "us_per_call": us,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 logits",
            "data": "synthetic (seeded)", "config": sample_config(args, w, world),
            "roofline": {"bound": "latency", "achieved": per_call / (us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": per_call / (us * 1e-6) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                         "per_launch_bytes": per_call, "per_launch_ms": us * 1e-3,
                         "timed": "64 sampler calls per step in one CUDA graph, CUDA events"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None,
            "e2e": None, "gpu_launches": args.steps * calls, "cpu_baseline": None}), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def sample_config(args, w, world: int) -> dict:
    return {"workload": "sample", "desc": w["desc"], "rows_per_gpu": w["branches"], "guidance": w["guidance"],
            "choices": w["ctx"], "alpha": w["alpha"], "cfg": w["cfg"], "calls_per_step": w["layers"],
            "cuda_graph": True, "parallelism": f"replicas x{world}"}


def run_reference_sampler(args, w) -> int:
    """The reference's own pp_renyi_sample (app/src/inference/renyi_sample.cu,
    compiled from the reference sources into oracle/_ref/) on the inputs and
    steps of run_sample, launched as fused_sampling.rs:147-162 does (one
    256-thread block per row, padded * 8 + 256 * 16 shared bytes) and
    recorded in a CUDA graph the same way."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref_runner

    if not os.path.exists(ref_runner.RENYI_CUBIN):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/renyi_ref.cubin was not built"}), flush=True)
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    raw, uni, bounds = sample_inputs(w, dev, 5)
    B, n, calls = w["branches"], w["ctx"], w["layers"]
    kern = ref_runner.RefRenyiKernel()
    padded = 1
    while padded < n:
        padded <<= 1
    out = torch.zeros(calls, 3 * B, dtype=torch.int32, device=dev)

    def enqueue():
        for i in range(calls):
            kern._launch("pp_renyi_sample", (B, 1), 256, padded * 8 + 256 * 16,
                         [raw[i], uni[i], bounds, out[i], C.c_uint32(B), C.c_uint32(n), C.c_uint32(w["guidance"]),
                          C.c_float(w["alpha"]), C.c_float(w["cfg"]), C.c_uint32(0), C.c_uint32(padded)])

    enqueue()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        enqueue()
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            g.replay()
        end.record(stream)
        torch.cuda.synchronize()
    ms_step = start.elapsed_time(end) / args.steps
    print(json.dumps({
        "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200", "impl": "reference",
        "value": calls * B / (ms_step * 1e-3), "unit": "sampled rows/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "us_per_call": ms_step * 1e3 / calls,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 logits",
        "data": "synthetic (seeded)", "config": sample_config(args, w, 1), "clocks": clocks.summary(),
        "reference_kernels": "pp_renyi_sample (app/src/inference/renyi_sample.cu) compiled for sm_100a with "
                             "fmad=false, prec_div=true; launch of fused_sampling.rs:147-162",
        "gpu_launches": args.steps * calls,
        "e2e": {"value": calls * B / (ms_step * 1e-3), "unit": "sampled rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg1")
    ap.add_argument("--layers", type=int, default=0, help="override the number of layer caches")
    ap.add_argument("--head-dim", type=int, choices=[64, 128], default=0,
                    help="override the head size (64: the reference model's own)")
    ap.add_argument("--split", type=int, default=0, help="fixed split size in tokens (0: automatic)")
    ap.add_argument("--max-ctas", type=int, default=0,
                    help="attention CTAs per call (0: one per SM); fewer leaves SMs on which the next call's "
                         "CTAs start streaming while this call drains")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="cfg3: launch the step eagerly instead of as a CUDA graph")
    ap.add_argument("--no-prefetch", action="store_true", help="never stream history before the previous kernel ends")
    ap.add_argument("--kv-dtype", choices=["bf16", "f32"], default=None,
                    help="float workload: K/V element type; encode: input element type")
    ap.add_argument("--ref-kernels", action="store_true",
                    help="with --impl reference and a reference-mode workload (deployed, cfg0): time the reference's "
                         "own CUDA kernels (oracle/_ref) on the GPU instead of its arithmetic on the host cores")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.workload])
    if args.layers:
        w["layers"] = args.layers
    if args.kv_dtype:
        w["kv"] = args.kv_dtype
    if args.head_dim:
        if args.workload == "cfg3":
            raise SystemExit("--head-dim does not apply to the decoder workload")
        w["d"] = args.head_dim
        w["desc"] += f" (head_dim overridden to {args.head_dim})"
    if args.ref_kernels and (args.impl != "reference" or not (w.get("refmode") or args.workload == "sample")):
        raise SystemExit("--ref-kernels needs --impl reference and a workload the reference has kernels for "
                         "(deployed, cfg0, sample)")
    if args.impl == "reference":
        if args.ref_kernels:
            return run_reference_sampler(args, w) if args.workload == "sample" else run_reference_kernels(args, w)
        if args.workload == "sample":
            print(json.dumps({"impl": "reference", "unavailable": "the reference samples on the GPU only "
                              "(fused_sampling.rs); run with --ref-kernels"}), flush=True)
            return 0
        return run_reference_arm(args, w)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist

        # Barriers and the timing reductions go over gloo with host tensors; NCCL carries the outputs' final
        # gather, over a group created after the timed regions (data_group).  While an NCCL communicator of
        # two or more ranks exists, a CUDA-graph decoder step (cfg3) runs ~5 % slower on every rank of a B200
        # box, with or without cuMem buffers and P2P/SHM transports; with only gloo it runs as fast as one
        # process alone.  All ranks are on this node, so gloo uses the loopback interface.
        if os.environ.get("MASTER_ADDR", "127.0.0.1") in ("127.0.0.1", "localhost"):
            os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        pg = dist

    pp = importlib.import_module("pop2-bezier_b200")
    ops = pp.int8_kv_ops
    N = pp._native
    if args.workload == "cfg2":
        return run_cfg2(args, w, pp, pg, world, rank, local, dev)
    if args.workload == "cfg3":
        return run_cfg3(args, w, pp, pg, world, rank, local, dev)
    if args.workload == "prefill":
        return run_prefill(args, w, pp, pg, world, rank, local, dev)
    if args.workload == "encode":
        return run_encode(args, w, pp, pg, world, rank, local, dev)
    if args.workload == "float":
        return run_float(args, w, pp, pg, world, rank, local, dev)
    if w.get("refmode"):
        return run_refmode(args, w, pp, pg, world, rank, local, dev)
    if args.workload == "sample":
        return run_sample(args, w, pp, pg, world, rank, local, dev)

    # ---- branch shard of this rank (independent branches, no collective)
    total_branches = w["branches"] * world
    shards = pp.kv_cache.BranchShards([w["ctx"]] * total_branches, world, rank)
    mine = shards.mine
    B, H, D, L, layers = len(mine), w["heads"], w["d"], w["ctx"], w["layers"]
    rows = B * H

    # ---- per-layer int8 caches, generated on the device as in config 0:
    # K/V ~ N(0,1) f32, quantized per (token, head) by our quantizer.
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    caches = []
    def draw():
        x = torch.randn(rows, L, D, device=dev, generator=gen)
        if w.get("dist") == "student_t":
            # Student-t(3) = z / sqrt(chi2(3) / 3), times 0.7; 1 % of the channels (at least one) x 8
            chi = torch.zeros_like(x)
            for _ in range(3):
                chi.add_(torch.randn(rows, L, D, device=dev, generator=gen).square_())
            x.div_(chi.div_(3).sqrt_()).mul_(0.7)
            del chi
            loud = torch.rand(D, device=dev, generator=gen) < 0.01
            loud[int(torch.randint(0, D, (1,), device=dev, generator=gen))] = True
            x[:, :, loud] *= 8
        return x

    for _ in range(layers):
        kv = []
        for _ in range(2):
            x = draw()
            kv.append(ops.quantize(x, check_finite=False))
            del x
        caches.append((kv[0][0], kv[1][0], kv[0][1], kv[1][1]))
    lengths = torch.full((B,), L, dtype=torch.int32, device=dev)
    qs = torch.randn(layers, rows, D, device=dev, generator=gen).to(torch.bfloat16)
    outs = torch.empty(layers, rows, D, dtype=torch.bfloat16, device=dev)
    arenas = [ops.arena_struct(k, v, ks, vs, H) for (k, v, ks, vs) in caches]
    params = ops.attn_params(split_tokens=args.split, q_dtype=torch.bfloat16, out_dtype=torch.bfloat16,
                             max_ctas=args.max_ctas)
    params_ready = ops.attn_params(split_tokens=args.split, q_dtype=torch.bfloat16, out_dtype=torch.bfloat16,
                                   plan_ready=True, max_ctas=args.max_ctas)
    # layers after the first follow another layer's attention, which writes neither this
    # layer's history nor the plan: they may stream history while it finishes
    params_prefetch = ops.attn_params(split_tokens=args.split, q_dtype=torch.bfloat16, out_dtype=torch.bfloat16,
                                      plan_ready=True, prefetch_history=not args.no_prefetch, max_ctas=args.max_ctas)
    ws = ops.new_workspace(arenas[0], params, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    lib = N.lib
    lens_p, ws_p, st_p = C.c_void_p(lengths.data_ptr()), C.c_void_p(ws.data_ptr()), C.c_void_p(status.data_ptr())
    q_ptrs = [C.c_void_p(qs[i].data_ptr()) for i in range(layers)]
    o_ptrs = [C.c_void_p(outs[i].data_ptr()) for i in range(layers)]
    arena_refs = [C.byref(a) for a in arenas]

    def step():
        # lengths are identical across layers in a step: plan once, reuse (DecodeMetadataCache)
        N.check(lib.pp_b200_plan_ragged(arena_refs[0], C.byref(params), lens_p, 0, ws_p, ws.numel(), sp))
        for i in range(layers):
            N.check(lib.pp_b200_decode_attention(arena_refs[i], C.byref(params_prefetch if i else params_ready),
                                                 q_ptrs[i], None, None, lens_p, o_ptrs[i], ws_p, ws.numel(), st_p, sp))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise SystemExit(f"device status after warm-up: {N.status_message(int(status.item()))}")

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    # ---- timed region: K steps, device time (CUDA events), max over ranks
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_total = ms_local = start.elapsed_time(end)
    ranks = per_rank(pg, dev, ms_local, args.steps, clocks)
    t = torch.tensor([ms_total], dtype=torch.float64)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps

    # ---- roofline of the attention call: its average duration over the timed region (events on the
    # launching stream bracket all K steps; a step is one plan + `layers` attention calls, so this
    # charges the plan and the combine kernels to the attention call).  This rank's own time.
    call_ms = ms_local / (args.steps * layers)

    per_call = bytes_per_call(dict(w, branches=B))
    peak, peak_kind = load_peaks()
    achieved = per_call / (call_ms * 1e-3) / 1e9
    value = world * layers * per_call / (ms_step * 1e-3) / 1e9
    tokens_per_s = total_branches / (ms_step * 1e-3)

    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                # the captured figure is for the workload's own head size
                traffic = None if args.head_dim else json.load(f).get(args.workload)
        except Exception:
            traffic = None

    # ---- end to end through the public API: host queries in, host outputs back
    e2e = None
    if not args.no_e2e:
        q_host = qs.cpu().pin_memory()
        o_host = torch.empty(outs.shape, dtype=outs.dtype).pin_memory()
        q_dev = torch.empty_like(qs)
        wsp = ws

        def e2e_step():
            q_dev.copy_(q_host, non_blocking=True)
            k0, v0, ks0, vs0 = caches[0]
            ops.plan_ragged(k0, v0, ks0, vs0, lengths, H, wsp, split_tokens=args.split, max_ctas=args.max_ctas)
            for i, (k, v, ks, vs) in enumerate(caches):
                ops.decode_attention(q_dev[i], k, v, ks, vs, lengths, H, out_dtype=torch.bfloat16,
                                     split_tokens=args.split, workspace=wsp, plan_ready=True, out=outs[i],
                                     prefetch_history=i > 0 and not args.no_prefetch, max_ctas=args.max_ctas)
            o_host.copy_(outs, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        e_steps = max(1, min(args.steps, 50))
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        def ranks_max(x: float) -> float:
            te = torch.tensor([x], dtype=torch.float64)
            if pg is not None:
                pg.all_reduce(te, op=pg.ReduceOp.MAX)
            return float(te.item())

        serial_ms = ranks_max(s0.elapsed_time(s1) / e_steps)

        # the same steps with the host copies overlapped on copy streams (two slots)
        q2, o2 = [torch.empty_like(qs) for _ in range(2)], [torch.empty_like(outs) for _ in range(2)]

        def up(s, j):
            q2[j].copy_(q_host, non_blocking=True)

        def run(s, j):
            k0, v0, ks0, vs0 = caches[0]
            ops.plan_ragged(k0, v0, ks0, vs0, lengths, H, wsp, split_tokens=args.split, max_ctas=args.max_ctas)
            for i, (k, v, ks, vs) in enumerate(caches):
                ops.decode_attention(q2[j][i], k, v, ks, vs, lengths, H, out_dtype=torch.bfloat16,
                                     split_tokens=args.split, workspace=wsp, plan_ready=True, out=o2[j][i],
                                     prefetch_history=i > 0 and not args.no_prefetch, max_ctas=args.max_ctas)

        def down(s, j):
            o_host.copy_(o2[j], non_blocking=True)

        pipelined_e2e_ms(max(1, args.warmup), up, run, down, stream, dev)
        barrier()
        e_ms = ranks_max(pipelined_e2e_ms(e_steps, up, run, down, stream, dev) / e_steps)
        barrier()
        e2e = {"value": world * layers * per_call / (e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": q_host.numel() * q_host.element_size(),
               "d2h_bytes_per_step": o_host.numel() * o_host.element_size(), "ms_per_step": e_ms,
               "tokens_per_s": total_branches / (e_ms * 1e-3), "copies": "overlapped on two copy streams",
               "serial_value": world * layers * per_call / (serial_ms * 1e-3) / 1e9, "serial_ms_per_step": serial_ms}

    # ---- final gather of this step's outputs to rank 0 (NCCL, outside the timed region)
    if pg is not None:
        # [layers, rows, D] -> per branch [B, layers, H, D], gathered in global branch order on rank 0
        per_branch = outs.view(layers, B, H, D).transpose(0, 1).contiguous()
        shards.gather(pg, per_branch, group=data_group(pg))

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(w, steps=3, warmup=1, sample_branches=1, threads=os.cpu_count() or 1, budget_s=20.0)

    if rank == 0:
        line = {
            "metric": "decode-attn HBM GB/s (% of peak) & branch tokens/s at 1/2/4/8 B200",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 KV (bf16-rounded dequant), bf16 q/out, f32 accumulate", "data": "synthetic (seeded)",
            "config": attention_config(args, w, world),
            "tokens_per_s": tokens_per_s,
            "percent_of_peak": 100.0 * value / (world * peak),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "per_launch_bytes": per_call, "per_launch_ms": call_ms,
                         "timed": "timed region / attention calls (CUDA events on the launching stream): "
                                  "attn_kernel, with the plan amortised over the step"},
            "clocks": clocks.summary(), "ranks": ranks, "nccl_ranks": world if _DATA_GROUP is not None else 0, "timing_group": "gloo" if pg is not None else None,
            "e2e": e2e,
            # per step: one plan, then per layer the attention kernel (+ the combine kernel with fixed splits)
            "gpu_launches": args.steps * (1 + (2 if args.split else 1) * layers),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
