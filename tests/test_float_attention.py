"""Float-KV fused decode attention (fused_attention.rs + decode_attention.cu).

CPU: the oracle restatement against the reference kernels' own outputs
(tests/golden/ref_float_attn.npz, made on a B200 by make_float_golden.py),
and the host-side checks of the C ABI and of the Python mirror.
GPU: pp_b200_decode_attention_float against the same outputs and, at larger
and head_dim-128 shapes the reference kernel does not cover, against the
oracle: 2e-3 relative / 1e-3 absolute (the path's tolerance) and, tighter,
1e-5 / 2e-5 for f32 outputs; bf16 outputs within one bf16 unit."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

import cases as K

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_float_attn.npz")
TIGHT = dict(rtol=1e-5, atol=2e-5)
PATH_TOL = dict(rtol=2e-3, atol=1e-3)


@pytest.fixture(scope="module")
def float_golden():
    return np.load(GOLDEN)


def _case(name):
    for c in K.FLOAT_CASES:
        if c[0] == name:
            return c
    raise KeyError(name)


def assert_same_nan_rows(got, want):
    np.testing.assert_array_equal(np.isnan(got).all(1), np.isnan(want).all(1))
    assert not np.isnan(got[~np.isnan(want).all(1)]).any()


@pytest.mark.parametrize("case", K.FLOAT_CASES, ids=[c[0] for c in K.FLOAT_CASES])
def test_oracle_matches_reference_kernels(oracle, float_golden, case):
    name, seed, dtype, batch, heads, size, cap, lengths, split, qs = case
    c = K.float_case(seed, dtype, batch, heads, size, cap, lengths, qs)
    lens = c["lengths"]
    assert K.sha(c["q"], c["k"], c["v"], *([] if lens is None else [lens])) == str(float_golden[f"{name}_input_sha"])
    got = oracle.float_attention(c["q"], c["k"], c["v"], lens, heads, size=size, split_tokens=split, threads=4)
    want = float_golden[name]
    assert_same_nan_rows(got, want)
    ok = ~np.isnan(want)
    # same summation orders; only exp differs (C library vs CUDA's expf)
    np.testing.assert_allclose(got[ok], want[ok], rtol=2e-6, atol=1e-6)


def _kv(pp, rows=4, heads=2, d=64, tokens=100, dtype=None, ks=None, vs=None, k=0x1000, v=0x2000):
    N = pp._native
    g = N.PpFloatKv()
    g.struct_size = C.sizeof(N.PpFloatKv)
    g.rows, g.heads, g.head_dim, g.tokens = rows, heads, d, tokens
    g.dtype = N.DTYPE_BF16 if dtype is None else dtype
    g.k_row_stride = tokens * d if ks is None else ks
    g.v_row_stride = tokens * d if vs is None else vs
    g.k, g.v = k, v
    return g


def test_abi_rejects_what_the_reference_rejects(pp):
    """fused_attention.rs:12-25 geometry, plus the 16-byte rule of the tensor
    copies; every check runs before any device work."""
    N = pp._native
    ws = C.c_void_p(0x10000)
    q = C.c_void_p(0x20000)

    def call(g, q_stride=64, qp=q):
        return N.lib.pp_b200_decode_attention_float(C.byref(g), None, qp, q_stride, None, q, ws, 1 << 20, None, None)

    bad = [
        _kv(pp, rows=5, heads=2),              # rows % heads
        _kv(pp, heads=0),
        _kv(pp, d=96),                         # head width
        _kv(pp, tokens=0),
        _kv(pp, dtype=7),
        _kv(pp, k=0),                          # NULL K
        _kv(pp, k=0x1008),                     # K base not 16-byte aligned
        _kv(pp, ks=100 * 64 + 4),              # bf16 row stride of 8 bytes mod 16
        _kv(pp, vs=100 * 64 - 64),             # rows overlap
    ]
    for g in bad:
        assert call(g) == N.STATUS_PRECONDITION, (g.rows, g.heads, g.head_dim, g.tokens)
    assert "fused" in N.last_error()
    assert N.lib.pp_b200_float_attention_workspace_size(C.byref(_kv(pp, d=96)), None) == 0
    assert N.lib.pp_b200_float_attention_workspace_size(C.byref(_kv(pp)), None) > 0


def test_python_mirror_rejects_cpu_tensors(pp):
    q = torch.zeros(2, 1, 64)
    k = torch.zeros(2, 8, 64)
    with pytest.raises(pp._native.PreconditionError, match="needs CUDA"):
        pp.fused_attention.decode_attention(q, k, k, None, 1)


# ----------------------------------------------------------------------- GPU


def to_dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def kv_dev(a: np.ndarray, dev) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def host(t):
    return t.detach().float().cpu().numpy().reshape(t.shape[0], -1)


def run_case(pp, cuda, c, heads, size, split, **kw):
    q = to_dev(c["q"], cuda)
    d = c["k"].shape[2]
    q3 = q[:, :d].unsqueeze(1)  # [rows, 1, d] with the case's row stride
    k = kv_dev(c["k"], cuda)[:, :size]
    v = kv_dev(c["v"], cuda)[:, :size]
    lens = None if c["lengths"] is None else to_dev(c["lengths"].astype(np.int32), cuda)
    return pp.fused_attention.decode_attention(q3, k, v, lens, heads, split, **kw)


@pytest.mark.gpu
@pytest.mark.parametrize("case", K.FLOAT_CASES, ids=[c[0] for c in K.FLOAT_CASES])
@pytest.mark.parametrize("plan", ["reference_split", "stream_k"])
def test_matches_reference_kernels(pp, cuda, float_golden, case, plan):
    name, seed, dtype, batch, heads, size, cap, lengths, split, qs = case
    c = K.float_case(seed, dtype, batch, heads, size, cap, lengths, qs)
    out = host(run_case(pp, cuda, c, heads, size, split if plan == "reference_split" else 0))
    want = float_golden[name]
    assert_same_nan_rows(out, want)
    ok = ~np.isnan(want)
    np.testing.assert_allclose(out[ok], want[ok], **TIGHT)


def random_rows(seed, batch, heads, d, cap, dtype, ragged=True):
    g = np.random.Generator(np.random.PCG64(seed))
    rows = batch * heads
    q = g.standard_normal((rows, d)).astype(np.float32)
    k = g.standard_normal((rows, cap, d)).astype(np.float32)
    v = g.standard_normal((rows, cap, d)).astype(np.float32)
    lens = g.integers(1, cap + 1, batch).astype(np.uint32) if ragged else None
    if dtype == "bf16":
        k, v = K.to_bf16_bits(k), K.to_bf16_bits(v)
    return q, k, v, lens


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("qdt,odt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16)])
def test_ragged_shapes_vs_oracle(pp, oracle, cuda, d, dtype, qdt, odt):
    batch, heads, cap = 6, 8, 2500
    q, k, v, lens = random_rows(90 + d, batch, heads, d, cap, dtype)
    lens[0], lens[1] = cap, 1
    qd = to_dev(q, cuda).to(qdt)
    out = pp.fused_attention.decode_attention(qd.unsqueeze(1), kv_dev(k, cuda), kv_dev(v, cuda),
                                              to_dev(lens.astype(np.int32), cuda), heads, out_dtype=odt)
    qo = qd.float().cpu().numpy()  # the query the kernel saw
    want = oracle.float_attention(qo, k, v, lens, heads, threads=oracle.max_threads())
    got = host(out)
    if odt == torch.float32:
        np.testing.assert_allclose(got, want, **TIGHT)
    else:
        wb = oracle.bf16_round(want)
        np.testing.assert_allclose(got, wb, rtol=2 ** -7, atol=1e-6)
    np.testing.assert_allclose(got, want, rtol=PATH_TOL["rtol"] if odt == torch.float32 else 2 ** -7,
                               atol=PATH_TOL["atol"])


@pytest.mark.gpu
@pytest.mark.parametrize("split", [32, 1024])
def test_fixed_splits_and_whole_rows_agree(pp, cuda, split):
    q, k, v, lens = random_rows(7, 4, 4, 64, 3000, "bf16")
    args = (to_dev(q, cuda).unsqueeze(1), kv_dev(k, cuda), kv_dev(v, cuda), to_dev(lens.astype(np.int32), cuda), 4)
    a = host(pp.fused_attention.decode_attention(*args, split))
    b = host(pp.fused_attention.decode_attention(*args, 0))
    np.testing.assert_allclose(a, b, **TIGHT)


@pytest.mark.gpu
def test_plan_reuse_prefetch_and_repeat_are_bit_identical(pp, cuda):
    q, k, v, lens = random_rows(8, 8, 16, 64, 4096, "bf16")
    fa = pp.fused_attention
    qd, kd, vd = to_dev(q, cuda).unsqueeze(1), kv_dev(k, cuda), kv_dev(v, cuda)
    ld = to_dev(lens.astype(np.int32), cuda)
    first = fa.decode_attention(qd, kd, vd, ld, 16)
    again = fa.decode_attention(qd, kd, vd, ld, 16)
    kv = fa.kv_struct(kd, vd, 16)
    ws = torch.empty(fa.workspace_bytes(kv, pp.int8_kv_ops.attn_params()), dtype=torch.uint8, device=cuda)
    fa.plan_ragged(kd, vd, ld, 16, ws)
    planned = fa.decode_attention(qd, kd, vd, ld, 16, workspace=ws, plan_ready=True)
    prefetched = fa.decode_attention(qd, kd, vd, ld, 16, workspace=ws, plan_ready=True, prefetch_history=True)
    for o in (again, planned, prefetched):
        assert torch.equal(o, first)


@pytest.mark.gpu
def test_view_of_larger_cache_and_no_lengths(pp, oracle, cuda):
    """K/V as the first `size` tokens of a larger cache (row stride = capacity
    * d), strided q rows, lengths None: every row attends to all `size`."""
    q, k, v, _ = random_rows(9, 3, 4, 64, 1200, "f32", ragged=False)
    size = 777
    k[:, size:] = np.nan
    v[:, size:] = np.nan
    qw = np.zeros((q.shape[0], 96), np.float32)
    qw[:, :64] = q
    qd = to_dev(qw, cuda)[:, :64].unsqueeze(1)
    out = pp.fused_attention.decode_attention(qd, kv_dev(k, cuda)[:, :size], kv_dev(v, cuda)[:, :size], None, 4)
    want = oracle.float_attention(qw, k, v, None, 4, size=size, threads=4)
    np.testing.assert_allclose(host(out), want, **TIGHT)


@pytest.mark.gpu
def test_full_size_properties(pp, oracle, cuda):
    """32 branches x 16 heads x 4096 tokens of bf16 (the bench workload):
    a constant V row comes back exactly as that constant (the weights sum to
    one), and a sample of rows matches the oracle."""
    batch, heads, cap, d = 32, 16, 4096, 64
    g = torch.Generator(device=cuda).manual_seed(5)
    rows = batch * heads
    q = torch.randn(rows, 1, d, device=cuda, generator=g)
    k = torch.randn(rows, cap, d, device=cuda, generator=g).to(torch.bfloat16)
    c = torch.randn(rows, 1, d, device=cuda, generator=g).to(torch.bfloat16)
    v = c.expand(rows, cap, d).contiguous()
    out = pp.fused_attention.decode_attention(q, k, v, None, heads)
    np.testing.assert_allclose(host(out), host(c.float()), **TIGHT)
    v = torch.randn(rows, cap, d, device=cuda, generator=g).to(torch.bfloat16)
    out = host(pp.fused_attention.decode_attention(q, k, v, None, heads))
    sample = np.arange(0, rows, 37)
    kb = k[sample].view(torch.int16).cpu().numpy().view(np.uint16)
    vb = v[sample].view(torch.int16).cpu().numpy().view(np.uint16)
    want = oracle.float_attention(q[sample, 0].cpu().numpy(), kb, vb, None, 1, threads=oracle.max_threads())
    np.testing.assert_allclose(out[sample], want, **TIGHT)


def test_prepare_optional_rejects_unsupported_widths(pp):
    """mod.rs:444-446: the fused path needs a supported head width."""
    N = pp._native
    assert N.lib.pp_b200_prepare_optional(0, 0, 0, N.DTYPE_BF16, 96, 0) == N.STATUS_OK  # nothing requested
    assert N.lib.pp_b200_prepare_optional(0, 0, 1, N.DTYPE_BF16, 96, 0) == N.STATUS_PRECONDITION
    assert N.last_error() == "当前模型后端不支持此融合解码路径"
    assert N.lib.pp_b200_prepare_optional(0, 1, 0, N.DTYPE_BF16, 64, 0) == N.STATUS_PRECONDITION


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("fusion,split_k", [(True, True), (False, True), (True, False)])
def test_prepare_optional_kernels_pass(pp, cuda, dtype, fusion, split_k):
    pp.fused_attention.prepare_optional_kernels(cuda, fusion, split_k, dtype=dtype, head_width=64, ffn_hidden=5632)
    pp.fused_attention.prepare_optional_kernels(cuda, fusion, split_k, dtype=dtype, head_width=128, ffn_hidden=300)
