"""Decoder-step operations on the CPU: the oracle restatement of the
reference's pp_graph_qkv / pp_graph_swiglu (graph_ops.cu) against the outputs
of the reference kernels themselves (tests/golden/ref_graph.npz, made on a B200
by tests/golden/make_graph_golden.py), the RoPE table builder, and the host-side
geometry checks of the C ABI entry points."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

import cases as K

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_graph.npz")


@pytest.fixture(scope="module")
def graph_golden():
    return np.load(GOLDEN)


def as_f32(bits: np.ndarray, bf: bool) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32) if bf else bits.view(np.float32)


def assert_within_one_bf16_ulp(got: np.ndarray, want: np.ndarray) -> None:
    """The oracle's reciprocal square root and exp are the C library's, the
    device's are the hardware's: a rounded bf16 result may land one unit away."""
    g, w = got.astype(np.int32), want.astype(np.int32)
    assert np.abs(g - w).max() <= 1, f"max bf16 unit difference {np.abs(g - w).max()}"
    assert (g != w).mean() < 0.01


@pytest.mark.parametrize("case", K.QKV_CASES, ids=[c[0] for c in K.QKV_CASES])
def test_oracle_qkv_rope_matches_reference_kernel(oracle, graph_golden, case):
    name, seed, rows, heads, dim, mc = case
    c = K.qkv_case(seed, rows, heads, dim, mc)
    assert K.sha(c["qkv"], c["params"], c["positions"]) == str(graph_golden[f"{name}_input_sha"])
    got = oracle.qkv_rope(c["qkv"], c["params"], c["positions"], rows, heads, dim, mc, bf=False)
    # f32: the one-ulp difference of the reciprocal square root can be magnified
    # where RoPE subtracts two nearly equal products, hence the absolute term
    np.testing.assert_allclose(got, as_f32(graph_golden[f"{name}_f32"], False).reshape(got.shape), rtol=2e-6,
                               atol=1e-6)
    gb = oracle.qkv_rope(K.to_bf16_bits(c["qkv"]), K.to_bf16_bits(c["params"]), c["positions"], rows, heads, dim, mc,
                         bf=True)
    assert_within_one_bf16_ulp(gb.ravel(), graph_golden[f"{name}_bf16"].ravel())


@pytest.mark.parametrize("case", K.SWIGLU_CASES, ids=[c[0] for c in K.SWIGLU_CASES])
def test_oracle_swiglu_matches_reference_kernel(oracle, graph_golden, case):
    name, seed, rows, hidden = case
    x = K.swiglu_case(seed, rows, hidden)
    assert K.sha(x) == str(graph_golden[f"{name}_input_sha"])
    got = oracle.swiglu(x, rows, hidden, bf=False)
    np.testing.assert_allclose(got, as_f32(graph_golden[f"{name}_f32"], False).reshape(got.shape), rtol=1e-6,
                               atol=1e-30)
    gb = oracle.swiglu(K.to_bf16_bits(x), rows, hidden, bf=True)
    assert_within_one_bf16_ulp(gb.ravel(), graph_golden[f"{name}_bf16"].ravel())


def test_oracle_rmsnorm_residual(oracle):
    g = np.random.Generator(np.random.PCG64(5))
    x = K.bf16_exact(g.standard_normal((3, 96)).astype(np.float32))
    r = K.bf16_exact(g.standard_normal((3, 96)).astype(np.float32))
    w = K.bf16_exact(1 + 0.1 * g.standard_normal(96).astype(np.float32))
    out, xs = oracle.rmsnorm(x, w, 3, 96, 1e-6, bf=False, residual=r)
    s = x + r
    want = s / np.sqrt((s.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(xs, s, rtol=0, atol=0)
    np.testing.assert_allclose(out, want, rtol=1e-5)


def test_rope_parameters_match_the_model_tables(pp):
    d, mc = 128, 50
    qn = torch.linspace(0.5, 1.5, d)
    kn = torch.linspace(1.5, 0.5, d)
    p = pp.decoder.rope_parameters(qn, kn, mc).numpy()
    cos, sin = K.rope_tables(mc, d)
    np.testing.assert_array_equal(p[:d], qn.numpy())
    np.testing.assert_array_equal(p[d:2 * d], kn.numpy())
    np.testing.assert_array_equal(p[2 * d:2 * d + mc * d // 2], cos.ravel())
    np.testing.assert_array_equal(p[2 * d + mc * d // 2:], sin.ravel())


def test_abi_rejects_bad_decoder_geometry_before_any_launch(pp):
    N = pp._native
    g = N.PpQkvRope()
    g.struct_size = C.sizeof(N.PpQkvRope)
    g.rows, g.heads, g.head_dim, g.max_context, g.dtype = 2, 4, 96, 16, N.DTYPE_BF16
    dummy = C.c_void_p(16)
    assert N.lib.pp_b200_qkv_rope(C.byref(g), dummy, dummy, dummy, dummy, None, None) == N.STATUS_PRECONDITION
    assert "geometry" in N.last_error()
    g.head_dim, g.dtype = 64, 7
    assert N.lib.pp_b200_qkv_rope(C.byref(g), dummy, dummy, dummy, dummy, None, None) == N.STATUS_PRECONDITION
    g.dtype = N.DTYPE_BF16
    assert N.lib.pp_b200_qkv_rope_append(C.byref(g), dummy, dummy, dummy, None, dummy, 1, dummy, dummy, dummy, None,
                                         None) == N.STATUS_PRECONDITION
    assert N.lib.pp_b200_swiglu(dummy, dummy, 0, 8, N.DTYPE_BF16, None) == N.STATUS_PRECONDITION
    assert N.lib.pp_b200_rmsnorm(dummy, None, None, dummy, dummy, 2, 8, float("nan"), N.DTYPE_BF16,
                                 None) == N.STATUS_PRECONDITION
    assert N.lib.pp_b200_rmsnorm(dummy, None, None, dummy, dummy, 0, 8, 1e-6, N.DTYPE_BF16,
                                 None) == N.STATUS_PRECONDITION
