"""Pins the oracle (oracle/int8kv_oracle.c) to the reference's own CUDA
kernels: tests/golden/ref_int8kv.npz holds outputs of pp_i8_scale/pack/
unpack/attention/merge (app/src/model/int8_kv.cu, compiled from the
reference sources, run on a B200 by tests/golden/make_golden.py).

Codes and scales must match bit-exactly; attention within the reference's
own self-check tolerance of 2e-5 (int8_kv_ops.rs:73,101)."""
from __future__ import annotations

import numpy as np
import pytest

import cases as K

TOL = 2e-5


def u32(x):
    return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)


def test_prep1(oracle, golden):
    c = K.prep1()
    codes, scales = oracle.quantize(c["x"])
    assert np.array_equal(codes, golden["prep1_codes"])
    assert np.array_equal(u32(scales), u32(golden["prep1_scales"]))
    assert np.array_equal(u32(oracle.dequantize(codes, scales, False)), u32(golden["prep1_unpack"]))
    out = oracle.attention(c["q"], codes, codes, scales, scales, c["past"], c["heads"], sk=c["sk"], sv=c["sk"])
    np.testing.assert_allclose(out, golden["prep1_out"].reshape(2, 64), rtol=0, atol=TOL)


def test_prep2(oracle, golden):
    c = K.prep2()
    rows, heads = c["rows"], c["heads"]
    k, ks = oracle.quantize(c["hist"][1:])
    v, vs = oracle.quantize(c["vals"][1:])
    assert np.array_equal(k, golden["prep2_k_codes"]) and np.array_equal(v, golden["prep2_v_codes"])
    assert np.array_equal(u32(ks), u32(golden["prep2_k_scales"])) and np.array_equal(u32(vs), u32(golden["prep2_v_scales"]))
    out = oracle.attention(c["q"][1:], k, v, ks, vs, c["past_all"][1:], heads, sk=c["sk"][1:], sv=c["sv"][1:])
    for split in (32, 128):
        np.testing.assert_allclose(out, golden[f"prep2_out_s{split}"].reshape(rows, 64), rtol=0, atol=TOL)


def test_cache_generator_codes(oracle, golden):
    for idx, (h, n, bias) in enumerate(K.CACHE_CASES):
        codes, scales = oracle.quantize(K.cache_data(h, n, bias))
        assert np.array_equal(codes, golden[f"cache{idx}_codes"]), idx
        assert np.array_equal(u32(scales), u32(golden[f"cache{idx}_scales"])), idx


def test_bf16_inputs(oracle, golden):
    c = K.hip_bf16()
    for name in ("k", "v"):
        codes, scales = oracle.quantize(c[f"{name}_bits"], 64)
        assert K.sha(codes) == str(golden[f"hip_{name}_codes_sha"])
        assert np.array_equal(u32(scales), u32(golden[f"hip_{name}_scales"]))


def test_edge_rows(oracle, golden):
    codes, scales = oracle.quantize(K.edge_rows())
    assert np.array_equal(codes, golden["edge_codes"])
    assert np.array_equal(u32(scales), u32(golden["edge_scales"]))


@pytest.mark.parametrize("case", K.RANDOM_CASES, ids=[c[0] for c in K.RANDOM_CASES])
def test_random_reference_mode(oracle, golden, case):
    name, seed, b, h, cap, pasts, split = case
    c = K.random_case(seed, b, h, cap)
    assert K.sha(c["k"], c["v"], c["q"], c["sk"], c["sv"]) == str(golden[f"{name}_input_sha"])
    k, ks = oracle.quantize(c["k"])
    v, vs = oracle.quantize(c["v"])
    assert K.sha(k, ks, v, vs) == str(golden[f"{name}_codes_sha"])
    out = oracle.attention(c["q"], k, v, ks, vs, np.array(pasts, np.uint32), h, sk=c["sk"], sv=c["sv"])
    ref = golden[f"{name}_out"].reshape(out.shape)
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    np.testing.assert_allclose(out[~np.isnan(ref)], ref[~np.isnan(ref)], rtol=0, atol=TOL)


def test_cfg0_history_mode(oracle, golden):
    c = K.cfg0_case(0)
    assert K.sha(c["k"], c["v"], c["q"]) == str(golden["cfg0_input_sha"])
    k, ks = oracle.quantize(c["k"])
    v, vs = oracle.quantize(c["v"])
    assert K.sha(k, ks, v, vs) == str(golden["cfg0_codes_sha"])
    out = oracle.attention(c["q"], k, v, ks, vs, np.array([1024], np.uint32), 16, threads=4)
    np.testing.assert_allclose(out, golden["cfg0_out"].reshape(16, 64), rtol=0, atol=TOL)
