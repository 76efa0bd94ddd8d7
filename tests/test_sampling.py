"""Fused Rényi sampling (fused_sampling.rs / renyi_sample.cu).

CPU: the oracle restatement against the reference kernel's own outputs
(tests/golden/ref_renyi.npz, made on a B200 by make_renyi_golden.py) and the
host-side checks of the entry point.  GPU: the CUDA kernel against the same
outputs, bit for bit (tokens, fallback flags and supports are integers)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

import cases as K

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_renyi.npz")


@pytest.fixture(scope="module")
def renyi_golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("case", K.RENYI_CASES, ids=[c[0] for c in K.RENYI_CASES])
def test_oracle_matches_reference_sampler(oracle, renyi_golden, case):
    name, seed, batch, choices, guidance, alpha, cfg, offset = case
    c = K.renyi_case(seed, batch, choices, guidance)
    assert K.sha(c["raw"], c["uniforms"], c["bounds"]) == str(renyi_golden[f"{name}_input_sha"])
    got = oracle.renyi_sample(c["raw"], c["uniforms"], c["bounds"], guidance, alpha, cfg, offset)
    np.testing.assert_array_equal(got, renyi_golden[name])


def test_sampler_rejects_what_the_reference_rejects(pp):
    """fused_sampling.rs:17-67: guidance 1/2, 1..2048 choices, alpha > 1,
    cfg >= 0 (== 1 without guidance), no token-range overflow."""
    N = pp._native
    d = C.c_void_p(16)
    call = lambda batch, choices, guidance, alpha, cfg, offset: N.lib.pp_b200_renyi_sample(  # noqa: E731
        d, d, d, d, batch, choices, guidance, alpha, cfg, offset, None)
    assert call(2, 2049, 1, 4.0, 1.0, 0) == N.STATUS_PRECONDITION
    assert call(2, 128, 3, 4.0, 1.0, 0) == N.STATUS_PRECONDITION
    assert call(2, 128, 1, 1.0, 1.0, 0) == N.STATUS_PRECONDITION
    assert call(2, 128, 1, float("nan"), 1.0, 0) == N.STATUS_PRECONDITION
    assert call(2, 128, 1, 4.0, 2.0, 0) == N.STATUS_PRECONDITION
    assert call(2, 128, 2, 4.0, float("inf"), 0) == N.STATUS_PRECONDITION
    assert call(2, 128, 1, 4.0, 1.0, 0xFFFFFFFF) == N.STATUS_PRECONDITION
    assert "guidance" in N.last_error() or "overflow" in N.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("case", K.RENYI_CASES, ids=[c[0] for c in K.RENYI_CASES])
def test_sampler_bit_exact_with_reference_kernel(pp, cuda, renyi_golden, case):
    name, seed, batch, choices, guidance, alpha, cfg, offset = case
    c = K.renyi_case(seed, batch, choices, guidance)
    tok, ok, sup = pp.sampling.renyi_sample(torch.from_numpy(c["raw"]).to(cuda),
                                            torch.from_numpy(c["uniforms"]).to(cuda).reshape(-1, 1),
                                            torch.from_numpy(c["bounds"].astype(np.int32)).to(cuda),
                                            alpha, cfg, guidance, offset)
    got = torch.stack([tok.view(-1), ok.view(-1), sup.view(-1)]).cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(got, renyi_golden[name])


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                                    "oracle", "_ref", "renyi_ref.cubin")),
                    reason="the reference sampler was not built (no reference tree when this checkout was built)")
@pytest.mark.parametrize("ties", [False, True])
def test_sampler_random_heads_live_against_reference_kernel(pp, cuda, ties):
    """Random heads through the reference's own kernel and ours in one process,
    bit for bit on every row (both use the same fast exp/log).  With `ties`
    the logits sit on a coarse grid with +0 and -0 among them, so the rank-th
    token is often one of many equal values and the column order decides."""
    from ref_runner import RefRenyiKernel

    ref = RefRenyiKernel()
    g = np.random.Generator(np.random.PCG64(71 + ties))
    for batch, choices, guidance, alpha, cfg in ((64, 2048, 2, 4.0, 1.5), (96, 1000, 1, 2.0, 1.0),
                                                 (40, 257, 2, 8.0, 3.0), (33, 2048, 1, 1.5, 1.0)):
        raw = (g.standard_normal((batch * guidance, choices)) * g.uniform(0.1, 6.0)).astype(np.float32)
        if ties:
            raw = np.round(raw * 2.0) / 2.0
            raw[np.abs(raw) == 0] = np.where(g.uniform(size=(raw == 0).sum()) < 0.5, -0.0, 0.0)
            raw = raw.astype(np.float32)
        u = g.uniform(0, 1, batch).astype(np.float32)
        u[:3] = np.array([0.0, np.nextafter(np.float32(1), np.float32(0)), 0.5], np.float32)
        starts = g.integers(0, choices // 2, batch)
        bounds = np.stack([starts, g.integers(1, choices - starts + 1)], 1).astype(np.uint32)
        raw_d, u_d = torch.from_numpy(raw).to(cuda), torch.from_numpy(u).to(cuda)
        b_d = torch.from_numpy(bounds.astype(np.int32)).to(cuda)
        tok, ok, sup = pp.sampling.renyi_sample(raw_d, u_d, b_d, alpha, cfg, guidance, 11)
        got = torch.stack([tok.view(-1), ok.view(-1), sup.view(-1)]).cpu().numpy().view(np.uint32)
        want = ref.sample(raw_d, u_d, b_d, guidance, alpha, cfg, 11).cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(got, want, err_msg=f"{batch}x{choices} guidance {guidance}")


@pytest.mark.gpu
def test_sampler_random_heads_vs_oracle(pp, oracle, cuda):
    """Larger random batches: every row's (token, flag, support) as the oracle's."""
    g = np.random.Generator(np.random.PCG64(61))
    for batch, choices, guidance, alpha, cfg in ((128, 1000, 2, 4.0, 1.5), (64, 2048, 1, 2.0, 1.0)):
        raw = (g.standard_normal((batch * guidance, choices)) * g.uniform(0.1, 6.0)).astype(np.float32)
        u = g.uniform(0, 1, batch).astype(np.float32)
        starts = g.integers(0, choices // 2, batch)
        bounds = np.stack([starts, g.integers(1, choices - starts + 1)], 1).astype(np.uint32)
        tok, ok, sup = pp.sampling.renyi_sample(torch.from_numpy(raw).to(cuda), torch.from_numpy(u).to(cuda),
                                                torch.from_numpy(bounds.astype(np.int32)).to(cuda),
                                                alpha, cfg, guidance, 7)
        got = torch.stack([tok.view(-1), ok.view(-1), sup.view(-1)]).cpu().numpy().view(np.uint32)
        want = oracle.renyi_sample(raw, u, bounds, guidance, alpha, cfg, 7)
        # the oracle's exp/log are the C library's: a support within a rounding step may move by one
        same = (got == want).all(0)
        assert same.mean() > 0.97, np.nonzero(~same)
        assert (np.abs(got[2].astype(np.int64) - want[2]) <= 1).all()
