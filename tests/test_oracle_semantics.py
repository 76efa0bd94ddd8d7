"""The oracle against the reference's own semantics, on the CPU.

Independent restatements used here:
  * the reference's torch quantizer of its HIP provider
    (app/native/aten_hip/cpp/kv_int8.cpp:162-166: x / (max|x|/127 clamped at
    1e-12), round half to even, clamp +-127) - written here with torch ops;
  * torch's own f32 -> bf16 conversion (round to nearest even);
  * the reference's self-check tolerances (int8_kv_ops.rs:62,73,101).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as K


def torch_quantize(x: np.ndarray):
    """Reference formula of kv_int8.cpp:162-166, evaluated by torch (f32)."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    scale = (t.abs().amax(-1) / 127.0).clamp_min(1e-12)
    codes = torch.round(t / scale.unsqueeze(-1)).clamp(-127, 127).to(torch.int8)
    return codes.view(torch.uint8).numpy(), scale.numpy()


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("d", [64, 128])
def test_quantize_matches_reference_torch_formula(oracle, seed, d):
    g = np.random.Generator(np.random.PCG64(seed))
    x = (g.standard_normal((257, d), dtype=np.float32) * g.uniform(0.01, 50, (257, 1))).astype(np.float32)
    codes, scales = oracle.quantize(x)
    tc, ts = torch_quantize(x)
    assert np.array_equal(codes, tc)
    assert np.array_equal(scales.view(np.uint32), ts.view(np.uint32))


def test_quantize_edge_rows(oracle):
    x = K.edge_rows()
    codes, scales = oracle.quantize(x)
    tc, ts = torch_quantize(x)
    assert np.array_equal(codes, tc) and np.array_equal(scales, ts)
    assert scales[0] == np.float32(1e-12) and not codes[0].any()
    assert scales[2] == np.float32(1.0)
    # ties to even: 2.5->2, 3.5->4, -2.5->-2, -3.5->-4, 0.5->0, -0.5->0, 126.5->126, -126.5->-126
    assert codes[2, 1:9].view(np.int8).tolist() == [2, 4, -2, -4, 0, 0, 126, -126]
    assert codes[5].view(np.int8).min() == -127


def test_quantize_rejects_non_finite(oracle):
    x = np.zeros((2, 64), np.float32)
    x[1, 3] = np.inf
    with pytest.raises(oracle.NonFiniteInput):
        oracle.quantize(x)
    x[1, 3] = np.nan
    with pytest.raises(oracle.NonFiniteInput):
        oracle.quantize(x)


def test_quantize_bf16_input_is_widened_exactly(oracle):
    c = K.hip_bf16()
    bits = c["k_bits"].reshape(-1, 64)[:300]
    a = oracle.quantize(bits, 64)
    b = oracle.quantize(K.bf16_to_f32(bits))
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_bf16_round_matches_torch(oracle):
    g = np.random.Generator(np.random.PCG64(3))
    x = np.concatenate([g.standard_normal(100000, dtype=np.float32) * 1e3,
                        np.float32([0.0, -0.0, 1.0, 3.3895314e38, -3.3895314e38, 1e-40])])
    ours = np.array([oracle.lib().oracle_bf16_round(float(v)) for v in x[:2000]], np.float32)
    theirs = torch.from_numpy(x[:2000]).to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32))
    assert np.array_equal(oracle.bf16_round(x).view(np.uint32), torch.from_numpy(x).to(torch.bfloat16).float().numpy().view(np.uint32))


def test_prepare_round_trip_tolerance(oracle):
    """int8_kv_ops.rs:59-62: dequantize(quantize(x)) within 0.009 of x."""
    c = K.prep1()
    codes, scales = oracle.quantize(c["x"])
    back = oracle.dequantize(codes, scales, round_bf16=False)
    assert np.all(np.isfinite(back)) and np.max(np.abs(back - c["x"])) < 0.009


def test_accounting_136_bytes_per_token_head():
    """int8_cache.rs:47-50: 64 int8 K + 64 int8 V + two f32 scales = 136 B,
    53.1% of bf16 K+V; at head_dim 128 it is 264 B."""
    assert 64 * 2 + 4 * 2 == 136 and 136 * 1000 // 256 == 531
    assert 128 * 2 + 4 * 2 == 264


def _softmax_attention_f64(q, k, v, scale):
    s = (k.astype(np.float64) @ q.astype(np.float64)) * scale
    p = np.exp(s - s.max())
    return (p[:, None] * v.astype(np.float64)).sum(0) / p.sum()


def test_attention_matches_float64_on_rounded_values(oracle):
    """The oracle's f32 loops agree with an f64 evaluation of the same formula
    on the bf16-rounded dequantized history to f32 accuracy."""
    c = K.random_case(5, 2, 2, 50)
    k, ks = oracle.quantize(c["k"])
    v, vs = oracle.quantize(c["v"])
    past = np.array([50, 23], np.uint32)
    out = oracle.attention(c["q"], k, v, ks, vs, past, 2, sk=c["sk"], sv=c["sv"])
    kd = oracle.dequantize(k, ks, True)
    vd = oracle.dequantize(v, vs, True)
    for r in range(4):
        n = past[r // 2]
        kk = np.concatenate([kd[r, :n], c["sk"][r][None]])
        vv = np.concatenate([vd[r, :n], c["sv"][r][None]])
        ref = _softmax_attention_f64(c["q"][r], kk, vv, 0.125)
        np.testing.assert_allclose(out[r], ref, rtol=2e-5, atol=2e-6)


def test_attention_history_mode_equals_scratch_of_last_token(oracle):
    """All-int8 attention over L tokens equals reference mode over L-1 tokens
    with the bf16-dequantized token L-1 as the f32 scratch."""
    c = K.random_case(6, 1, 3, 33)
    k, ks = oracle.quantize(c["k"])
    v, vs = oracle.quantize(c["v"])
    hist = oracle.attention(c["q"], k, v, ks, vs, np.array([33], np.uint32), 3)
    kd = oracle.dequantize(k, ks, True)
    vd = oracle.dequantize(v, vs, True)
    ref = oracle.attention(c["q"], k, v, ks, vs, np.array([32], np.uint32), 3, sk=kd[:, 32], sv=vd[:, 32])
    assert np.array_equal(hist, ref)


def test_attention_invalid_lengths_give_nan(oracle):
    c = K.random_case(8, 2, 1, 8)
    k, ks = oracle.quantize(c["k"])
    v, vs = oracle.quantize(c["v"])
    out = oracle.attention(c["q"], k, v, ks, vs, np.array([9, 8], np.uint32), 1, sk=c["sk"], sv=c["sv"])
    assert np.isnan(out[0]).all() and np.isfinite(out[1]).all()
    out = oracle.attention(c["q"], k, v, ks, vs, np.array([0, 8], np.uint32), 1)
    assert np.isnan(out[0]).all() and np.isfinite(out[1]).all()
    out = oracle.attention(c["q"], k, v, ks, vs, np.array([0, 3], np.uint32), 1, sk=c["sk"], sv=c["sv"])
    np.testing.assert_array_equal(out[0], c["sv"][0])  # empty history: only the scratch token


def test_quant_append_commit_and_partial(oracle):
    rows, heads, cap, d = 6, 3, 10, 64
    g = np.random.Generator(np.random.PCG64(9))
    xk = g.standard_normal((rows, d), dtype=np.float32)
    xv = g.standard_normal((rows, d), dtype=np.float32)
    K_ = np.zeros((rows, cap, d), np.uint8)
    V_ = np.zeros_like(K_)
    KS = np.zeros((rows, cap), np.float32)
    VS = np.zeros_like(KS)
    oracle.quant_append(xk, xv, heads, np.array([4, 9], np.uint32), True, K_, V_, KS, VS)
    ck, sk = oracle.quantize(xk)
    assert np.array_equal(K_[0, 4], ck[0]) and np.array_equal(K_[5, 9], ck[5]) and KS[4, 9] == sk[4]
    oracle.quant_append(xk, xv, heads, np.array([5, 0], np.uint32), False, K_, V_, KS, VS)
    assert not K_[0, 5].any() and KS[0, 5] == 1.0 and VS[3, 0] == 1.0
    with pytest.raises(ValueError):
        oracle.quant_append(xk, xv, heads, np.array([10, 0], np.uint32), True, K_, V_, KS, VS)
