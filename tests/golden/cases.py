"""Deterministic input cases shared by the golden-vector generator
(make_golden.py, run on a B200 against the reference's own kernels) and the
tests that check the oracle and the CUDA path against those vectors.

The closed-form fixtures restate the reference's own test/self-check inputs:
  prep1      app/src/model/int8_kv_ops.rs:59-73   (sin(i*0.17)*2, past [2,1], split 32)
  prep2      app/src/model/int8_kv_ops.rs:75-101  (rows 4, capacity 67, heads 2, view offset 1,
                                                   past [0,66], splits {32,128})
  cache_*    app/src/model/int8_cache.rs:19-23    (sin(i*0.173)*2 + bias)
  hip_bf16   app/native/aten_hip/cpp/kv_int8.cpp:168-176 (bf16 K/V, B=2, H=2, C=257)
Random cases use numpy PCG64 streams from fixed seeds.
"""
from __future__ import annotations

import hashlib

import numpy as np


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def prep1() -> dict:
    i = np.arange(384, dtype=np.float32)
    x = (np.sin(i * np.float32(0.17)) * np.float32(2.0)).astype(np.float32).reshape(2, 3, 64)
    j = np.arange(128, dtype=np.float32)
    q = np.cos(j * np.float32(0.07)).astype(np.float32).reshape(2, 64)
    sk = np.sin(j * np.float32(0.09)).astype(np.float32).reshape(2, 64)
    return dict(x=x, q=q, sk=sk, past=np.array([2, 1], dtype=np.uint32), heads=1, split=32)


def prep2() -> dict:
    rows, cap, heads = 4, 67, 2
    n = (rows + 1) * cap * 64
    i = np.arange(n, dtype=np.float32)
    hist = (np.sin(i * np.float32(0.013)) * np.float32(1.7)).astype(np.float32).reshape(rows + 1, cap, 64)
    vals = (np.cos(i * np.float32(0.019)) * np.float32(0.8)).astype(np.float32).reshape(rows + 1, cap, 64)

    def vec(factor, phase):
        j = np.arange((rows + 1) * 64, dtype=np.float32)
        return np.sin(j * np.float32(factor) + np.float32(phase)).astype(np.float32).reshape(rows + 1, 64)

    return dict(hist=hist, vals=vals, q=vec(0.027, 0.4), sk=vec(0.031, 1.1), sv=vec(0.047, -0.8),
                past_all=np.array([999, 0, 66], dtype=np.uint32), rows=rows, cap=cap, heads=heads)


def cache_data(heads: int, count: int, bias: float) -> np.ndarray:
    i = np.arange(heads * count * 64, dtype=np.float32)
    return (np.sin(i * np.float32(0.173)) * np.float32(2.0) + np.float32(bias)).astype(np.float32).reshape(
        heads, count, 64)


CACHE_CASES = [(2, 3, 0.0), (2, 3, 1.0), (2, 1, -5.0), (2, 63, 0.0), (2, 2, 4.0), (2, 2, 7.0), (2, 1, -99.0)] + [
    (2, 1, field * 5.0) for field in range(9)]


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def hip_bf16() -> dict:
    B, H, Cn = 2, 2, 257
    i = np.arange(B * H * Cn * 64, dtype=np.float32)
    k = to_bf16_bits(np.sin(i * np.float32(0.013))).reshape(B, H, Cn, 64)
    v = to_bf16_bits(np.cos(i * np.float32(0.019))).reshape(B, H, Cn, 64)
    return dict(k_bits=k, v_bits=v)


def edge_rows() -> np.ndarray:
    """Rows exercising the scale floor, exact ties, clamping and extremes."""
    rows = []
    rows.append(np.zeros(64, np.float32))                          # scale floor 1e-12, all zero codes
    rows.append(np.full(64, 1e-11, np.float32))                    # below the floor: s = 1e-12
    t = np.zeros(64, np.float32)
    t[0] = 127.0                                                   # s = 1 exactly
    t[1:9] = [2.5, 3.5, -2.5, -3.5, 0.5, -0.5, 126.5, -126.5]      # exact ties -> half to even
    rows.append(t)
    rows.append(np.linspace(-1e30, 1e30, 64, dtype=np.float32))    # huge magnitudes
    rows.append(np.linspace(-3e-38, 3e-38, 64, dtype=np.float32))  # subnormal/tiny range
    r = np.random.Generator(np.random.PCG64(7)).standard_normal(64, dtype=np.float32)
    r[5] = -np.abs(r).max() * 2                                    # negative extreme -> -127
    rows.append(r)
    rows.append(np.full(64, -4.0, np.float32))                     # constant negative row
    return np.stack(rows).astype(np.float32)


# Random reference-mode cases (head_dim 64, capacity <= 1024: the reference's limits).
RANDOM_CASES = [
    # name, seed, branches, heads, capacity, pasts (per branch), split
    ("rand_small", 11, 3, 2, 40, [0, 17, 40], 32),
    ("rand_ragged", 12, 4, 4, 300, [299, 1, 150, 64], 128),
    ("rand_split1024", 13, 2, 3, 1000, [999, 500], 1024),
    ("rand_invalid", 14, 2, 2, 64, [64, 65], 32),  # past == capacity is valid, > capacity gives NaN
]


def random_case(seed: int, branches: int, heads: int, cap: int) -> dict:
    g = np.random.Generator(np.random.PCG64(seed))
    rows = branches * heads
    k = g.standard_normal((rows, cap, 64), dtype=np.float32)
    v = g.standard_normal((rows, cap, 64), dtype=np.float32)
    q = g.standard_normal((rows, 64), dtype=np.float32)
    sk = g.standard_normal((rows, 64), dtype=np.float32)
    sv = g.standard_normal((rows, 64), dtype=np.float32)
    return dict(k=k, v=v, q=q, sk=sk, sv=sv)


def cfg0_case(seed: int = 0) -> dict:
    """batch 1, 16 heads, head_dim 64, context 1024, fp32
    query per head, K/V from N(0,1) quantized per (token, head)."""
    g = np.random.Generator(np.random.PCG64(seed))
    k = g.standard_normal((16, 1024, 64), dtype=np.float32)
    v = g.standard_normal((16, 1024, 64), dtype=np.float32)
    q = g.standard_normal((16, 64), dtype=np.float32)
    return dict(k=k, v=v, q=q)


# ------------------------------------------------------------- decoder step
# Inputs for the reference's pp_graph_qkv / pp_graph_swiglu (graph_ops.cu) and
# the matching oracle and CUDA functions.  Model-dtype arrays are float32
# values that are exactly representable in bf16 (so the f32 and bf16 runs see
# the same numbers); bf16 runs pass their bits.

def rope_tables(max_context: int, dim: int) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin [max_context, dim/2] in f32 as PrimitiveModel builds them
    (mod.rs:322-330): inv = 1 / 10000^(2p/dim), angle = pos * inv."""
    pair = np.arange(dim // 2, dtype=np.float32)
    inv = (np.float32(1.0) / np.power(np.float32(10000.0), (pair * np.float32(2.0)) / np.float32(dim))).astype(np.float32)
    pos = np.arange(max_context, dtype=np.float32)[:, None]
    ang = (pos * inv[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def bf16_exact(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(to_bf16_bits(np.asarray(x, dtype=np.float32)))


def qkv_case(seed: int, rows: int, heads: int, dim: int, max_context: int) -> dict:
    """QKV projection output [rows, 3*heads*dim], the parameter block
    [q_norm | k_norm | cos | sin] and positions, all bf16-exact."""
    g = np.random.Generator(np.random.PCG64(seed))
    qkv = bf16_exact(g.standard_normal((rows, 3 * heads * dim)).astype(np.float32) * np.float32(2.5))
    qn = bf16_exact(1.0 + 0.2 * g.standard_normal(dim).astype(np.float32))
    kn = bf16_exact(1.0 + 0.2 * g.standard_normal(dim).astype(np.float32))
    cos, sin = rope_tables(max_context, dim)
    params = np.concatenate([qn, kn, bf16_exact(cos).ravel(), bf16_exact(sin).ravel()]).astype(np.float32)
    positions = g.integers(0, max_context, rows).astype(np.uint32)
    positions[0] = 0
    positions[-1] = max_context - 1
    return dict(qkv=qkv, params=params, positions=positions)


def swiglu_case(seed: int, rows: int, hidden: int) -> np.ndarray:
    g = np.random.Generator(np.random.PCG64(seed))
    x = g.standard_normal((rows, 2 * hidden)).astype(np.float32) * np.float32(3.0)
    x[0, :8] = [0.0, -0.0, 88.0, -88.0, 1e-30, -1e-30, 20.0, -20.0]
    return bf16_exact(x)


QKV_CASES = [  # name, seed, rows, heads, dim (the reference kernel supports 64), max_context
    ("qkv_a", 31, 5, 4, 64, 96),
    ("qkv_b", 32, 3, 16, 64, 1024),
]
SWIGLU_CASES = [("swiglu_a", 41, 7, 300), ("swiglu_b", 42, 3, 5632)]


# ---------------------------------------------------------------- sampling
# Inputs for the reference's fused Rényi sampler (renyi_sample.cu): name, seed,
# batch, choices, guidance, alpha, cfg, token offset.  Each case mixes legal
# windows, peaky and flat heads, ties and the invalid rows the kernel falls
# back on (bad uniform, empty or out-of-range window, non-finite logits).
RENYI_CASES = [
    ("renyi_a", 51, 12, 270, 1, 4.0, 1.0, 100),
    ("renyi_b", 52, 9, 2048, 2, 3.5, 2.5, 2048),
    ("renyi_c", 53, 8, 17, 2, 1.5, 0.0, 0),
]


def renyi_case(seed: int, batch: int, choices: int, guidance: int) -> dict:
    g = np.random.Generator(np.random.PCG64(seed))
    raw = (g.standard_normal((batch * guidance, choices)) * 2.0).astype(np.float32)
    uniforms = g.uniform(0.0, 1.0, batch).astype(np.float32)
    starts = g.integers(0, choices // 2, batch).astype(np.uint32)
    counts = np.maximum(1, g.integers(1, choices - starts + 1)).astype(np.uint32)
    bounds = np.stack([starts, counts], 1).astype(np.uint32)
    rg = lambda r: slice(r * guidance, (r + 1) * guidance)  # noqa: E731
    raw[rg(0)] *= 8.0                      # peaky head: support 1
    raw[rg(1)] *= 0.0                      # flat head: support = count, ties broken by column
    uniforms[1] = np.float32(0.999)
    uniforms[2] = np.float32(0.0)          # rank 0: the arg-max path
    bounds[3] = (0, choices)               # the whole head
    uniforms[4] = np.float32(1.0)          # invalid uniform
    bounds[5] = (choices, 1)               # window outside the head
    if batch > 6:
        raw[rg(6)][0, choices // 3] = np.float32(np.nan)  # non-finite logit: fallback
    if batch > 7:
        bounds[7] = (1, 0)                 # empty window
    return dict(raw=raw, uniforms=uniforms, bounds=bounds)


# ------------------------------------------------------- float-KV attention
# Inputs for the reference's float-KV fused decode attention
# (decode_attention.cu, fused_attention.rs): name, seed, KV dtype, batch,
# heads, size (the key length), row capacity (row stride in tokens, >= size),
# lengths ("none" or "ragged"), split_tokens, q row stride (elements).
# Every token at or past its row's length holds NaN: the kernel must never
# let it reach the output.  Ragged lengths include 0 and size + 1 (NaN rows),
# 1 and size.
FLOAT_CASES = [
    ("fa_prep", 0, "f32", 1, 1, 257, 257, "none", 128, 64),
    ("fa_f32_dense", 71, "f32", 3, 2, 300, 300, "none", 0, 64),
    ("fa_bf16_ragged", 72, "bf16", 4, 3, 1024, 1100, "ragged", 0, 64),
    ("fa_bf16_split", 73, "bf16", 2, 4, 700, 700, "ragged", 128, 128),
    ("fa_f32_clamp", 74, "f32", 5, 2, 100, 128, "ragged", 1, 64),
    ("fa_f32_peaky", 75, "f32", 2, 2, 513, 520, "none", 0, 80),
    ("fa_bf16_wide", 76, "bf16", 2, 2, 1024, 1024, "none", 5000, 64),
]


def float_case(seed: int, dtype: str, batch: int, heads: int, size: int, cap: int, lengths: str,
               q_stride: int, d: int = 64) -> dict:
    """q f32 [rows, q_stride] (first d used); k, v [rows, cap, d] as f32 or
    bf16 bits (uint16); lengths u32 [batch] or None."""
    rows = batch * heads
    if seed == 0:  # the reference's prepare_optional_kernels fixture (mod.rs:447-452): zeros
        q = np.zeros((rows, q_stride), np.float32)
        k = np.zeros((rows, cap, d), np.float32)
        v = np.zeros((rows, cap, d), np.float32)
        lens = None
    else:
        g = np.random.Generator(np.random.PCG64(seed))
        q = g.standard_normal((rows, q_stride)).astype(np.float32)
        k = g.standard_normal((rows, cap, d)).astype(np.float32)
        v = g.standard_normal((rows, cap, d)).astype(np.float32)
        if seed == 75:  # peaky softmax: large scores, ties of the maximum across splits
            k *= np.float32(6.0)
            k[0, 10] = k[0, 400]
        lens = None
        if lengths == "ragged":
            lens = g.integers(1, size + 1, batch).astype(np.uint32)
            edge = [size, 1, 0, size + 1]
            lens[:min(batch, 4)] = edge[:min(batch, 4)]
        for r in range(rows):
            n = size if lens is None else int(lens[r // heads])
            k[r, min(n, cap):] = np.nan
            v[r, min(n, cap):] = np.nan
    if dtype == "bf16":
        k, v = to_bf16_bits(k), to_bf16_bits(v)
    return dict(q=q, k=k, v=v, lengths=lens)
