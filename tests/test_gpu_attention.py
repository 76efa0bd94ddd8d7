"""Int8 decode attention on the B200 through the C ABI.

Reference mode (f32 scratch token, head_dim 64) against the outputs of the
reference's own CUDA kernels (tests/golden/ref_int8kv.npz) within the
reference's self-check tolerance 2e-5 (int8_kv_ops.rs:73,101); history mode
at the BASELINE shapes against the oracle within 2e-3 relative / 1e-3
absolute, plus size-independent properties at full size."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

import cases as K

pytestmark = pytest.mark.gpu

REF_TOL = 2e-5


def to_dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("split", [32, 128, 0])
def test_prep1_matches_reference_kernels(pp, cuda, golden, split):
    ops = pp.int8_kv_ops
    c = K.prep1()
    codes, scales = ops.quantize(to_dev(c["x"], cuda))
    q = to_dev(c["q"], cuda).reshape(2, 1, 64)
    sk = to_dev(c["sk"], cuda).reshape(2, 1, 64)
    past = torch.tensor([2, 1], dtype=torch.int32, device=cuda)
    out = ops.attention(q, codes, codes, scales, scales, sk, sk, past, 1, split)
    np.testing.assert_allclose(host(out), golden["prep1_out"], rtol=0, atol=REF_TOL)


@pytest.mark.parametrize("split", [32, 128, 0])
def test_prep2_offsets_heads_splits_match_reference(pp, cuda, golden, split):
    """Non-zero view offsets (scale arrays only 4-byte aligned), two heads per
    sequence, an empty history and unequal lengths (int8_kv_ops.rs:75-101)."""
    ops = pp.int8_kv_ops
    c = K.prep2()
    rows, heads = c["rows"], c["heads"]
    k, ks = ops.quantize(to_dev(c["hist"], cuda)[1:].contiguous())
    v, vs = ops.quantize(to_dev(c["vals"], cuda)[1:].contiguous())
    kb, vb = torch.cat([k[0:1], k])[1:], torch.cat([v[0:1], v])[1:]
    ksb, vsb = torch.cat([ks[0:1], ks])[1:], torch.cat([vs[0:1], vs])[1:]
    assert ksb.data_ptr() % 16 != 0  # exercises the misaligned scale path
    q = to_dev(c["q"], cuda)[1:].reshape(rows, 1, 64)
    sk = to_dev(c["sk"], cuda)[1:].reshape(rows, 1, 64)
    sv = to_dev(c["sv"], cuda)[1:].reshape(rows, 1, 64)
    past = to_dev(c["past_all"].astype(np.int32), cuda)[1:]
    out = host(ops.attention(q, kb, vb, ksb, vsb, sk, sv, past, heads, split))
    for s in (32, 128):
        np.testing.assert_allclose(out, golden[f"prep2_out_s{s}"], rtol=0, atol=REF_TOL)


@pytest.mark.parametrize("case", K.RANDOM_CASES, ids=[c[0] for c in K.RANDOM_CASES])
@pytest.mark.parametrize("split_override", [None, 0])
def test_random_reference_mode_matches_reference_kernels(pp, cuda, golden, case, split_override):
    name, seed, b, h, cap, pasts, split = case
    ops = pp.int8_kv_ops
    c = K.random_case(seed, b, h, cap)
    assert K.sha(c["k"], c["v"], c["q"], c["sk"], c["sv"]) == str(golden[f"{name}_input_sha"])
    rows = b * h
    k, ks = ops.quantize(to_dev(c["k"], cuda))
    v, vs = ops.quantize(to_dev(c["v"], cuda))
    assert K.sha(k.cpu().numpy(), ks.cpu().numpy(), v.cpu().numpy(), vs.cpu().numpy()) == str(
        golden[f"{name}_codes_sha"])
    past = torch.tensor(pasts, dtype=torch.int32, device=cuda)
    sp = split if split_override is None else split_override
    out = host(ops.attention(to_dev(c["q"], cuda).reshape(rows, 1, 64), k, v, ks, vs,
                             to_dev(c["sk"], cuda).reshape(rows, 1, 64), to_dev(c["sv"], cuda).reshape(rows, 1, 64),
                             past, h, sp))
    ref = golden[f"{name}_out"]
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    np.testing.assert_allclose(out[~np.isnan(ref)], ref[~np.isnan(ref)], rtol=0, atol=REF_TOL)


def test_cfg0_history_mode_matches_reference_kernels(pp, cuda, golden):
    """BASELINE config 0 (1 branch, 16 heads, d 64, context 1024, f32 q/out)."""
    ops = pp.int8_kv_ops
    c = K.cfg0_case(0)
    assert K.sha(c["k"], c["v"], c["q"]) == str(golden["cfg0_input_sha"])
    k, ks = ops.quantize(to_dev(c["k"], cuda))
    v, vs = ops.quantize(to_dev(c["v"], cuda))
    assert K.sha(k.cpu().numpy(), ks.cpu().numpy(), v.cpu().numpy(), vs.cpu().numpy()) == str(golden["cfg0_codes_sha"])
    out = ops.decode_attention(to_dev(c["q"], cuda), k, v, ks, vs, torch.tensor([1024], dtype=torch.int32, device=cuda), 16)
    np.testing.assert_allclose(host(out), golden["cfg0_out"].reshape(16, 64), rtol=0, atol=REF_TOL)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                                    "oracle", "_ref", "int8_kv_ref.cubin")),
                    reason="reference kernels were not built (no reference tree when this checkout was built)")
@pytest.mark.parametrize("seed", [31, 32])
def test_live_against_reference_kernels(pp, cuda, seed):
    """Same inputs through the reference's kernels and ours, in one process."""
    from ref_runner import RefInt8Kernels

    ref = RefInt8Kernels()
    g = np.random.Generator(np.random.PCG64(seed))
    b, h, cap = 5, 3, int(g.integers(100, 1025))
    rows = b * h
    kx = to_dev(g.standard_normal((rows, cap, 64), dtype=np.float32) * 2, cuda)
    vx = to_dev(g.standard_normal((rows, cap, 64), dtype=np.float32), cuda)
    k, ks = ref.quantize(kx)
    v, vs = ref.quantize(vx)
    k2, ks2 = pp.int8_kv_ops.quantize(kx)
    assert torch.equal(k, k2) and torch.equal(ks, ks2)
    q = to_dev(g.standard_normal((rows, 1, 64), dtype=np.float32), cuda)
    sk = to_dev(g.standard_normal((rows, 1, 64), dtype=np.float32), cuda)
    sv = to_dev(g.standard_normal((rows, 1, 64), dtype=np.float32), cuda)
    pasts = torch.tensor(g.integers(0, cap + 1, b), dtype=torch.int32, device=cuda)
    for split in (32, 128, 512):
        want = ref.attention(q, k, v, ks, vs, sk, sv, pasts, h, split)
        got = pp.int8_kv_ops.attention(q, k, v, ks, vs, sk, sv, pasts, h, split)
        np.testing.assert_allclose(host(got), host(want), rtol=0, atol=REF_TOL)


REF_CUBIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                         "int8_kv_ref.cubin")


@pytest.mark.parametrize("lengths", ["uniform", "ragged"])
def test_deployed_shape_every_row(pp, oracle, cuda, lengths):
    """The reference model's own step shape: 8 branches x 24 heads, d 64,
    capacity 1024, reference mode.  With every branch at 1023 history tokens
    the plan gives each CTA whole rows; with ragged histories it cuts rows
    across CTAs.  Every row of three layer calls on one plan (the later two
    streaming history before the previous call ends) is checked against the
    oracle and, where the reference's kernels were built, against them."""
    ops = pp.int8_kv_ops
    g = np.random.Generator(np.random.PCG64(64 + (lengths == "ragged")))
    branches, heads, cap, d = 8, 24, 1024, 64
    rows = branches * heads
    if lengths == "uniform":
        past_h = np.full(branches, cap - 1, dtype=np.int32)
    else:
        past_h = g.integers(0, cap, branches).astype(np.int32)
        past_h[0], past_h[1] = 0, cap - 1
    past = torch.tensor(past_h, device=cuda)
    layers = []
    for _ in range(3):
        k, ks = ops.quantize(to_dev(g.standard_normal((rows, cap, d), dtype=np.float32), cuda))
        v, vs = ops.quantize(to_dev(g.standard_normal((rows, cap, d), dtype=np.float32), cuda))
        q, sk, sv = (to_dev(g.standard_normal((rows, d), dtype=np.float32), cuda) for _ in range(3))
        layers.append((q, k, v, ks, vs, sk, sv))
    k0, v0, ks0, vs0 = layers[0][1:5]
    params = ops.attn_params(q_dtype=torch.float32, out_dtype=torch.float32)
    ws = ops.new_workspace(ops.arena_struct(k0, v0, ks0, vs0, heads), params, cuda)
    ops.plan_ragged(k0, v0, ks0, vs0, past, heads, ws, scratch=True)
    outs = [ops.decode_attention(q, k, v, ks, vs, past, heads, scratch_k=sk, scratch_v=sv, out_dtype=torch.float32,
                                 workspace=ws, plan_ready=True, prefetch_history=i > 0)
            for i, (q, k, v, ks, vs, sk, sv) in enumerate(layers)]
    ref = None
    if os.path.exists(REF_CUBIN):
        from ref_runner import RefInt8Kernels

        ref = RefInt8Kernels()
    for (q, k, v, ks, vs, sk, sv), out in zip(layers, outs):
        want = oracle.attention(host(q), k.cpu().numpy(), v.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy(),
                                past_h, heads, sk=host(sk), sv=host(sv), threads=oracle.max_threads())
        np.testing.assert_allclose(host(out), want.reshape(rows, d), rtol=0, atol=REF_TOL)
        if ref is not None:
            r = ref.attention(q.view(rows, 1, d), k, v, ks, vs, sk.view(rows, 1, d), sv.view(rows, 1, d), past, heads,
                              128)
            np.testing.assert_allclose(host(out), host(r).reshape(rows, d), rtol=0, atol=REF_TOL)


def assert_bf16_close(got, ref_f32):
    """bf16 outputs: the f32 result must round to within one bf16 ulp of the
    oracle's f32 result rounded the same way (output rounding is up to 2^-8
    relative, so a plain 2e-3 relative bound cannot hold for bf16 outputs)."""
    import oracle as O

    ref_b = O.bf16_round(np.ascontiguousarray(ref_f32, dtype=np.float32))
    mag = np.maximum(np.abs(ref_b), np.float32(2.0**-126))
    ulp = np.exp2(np.floor(np.log2(mag)) - 7).astype(np.float32)
    diff = np.abs(np.asarray(got, np.float32) - ref_b)
    bad = diff > np.maximum(ulp, 1e-3)
    assert not bad.any(), f"{bad.sum()} bf16 outputs beyond one ulp, max diff {diff.max()}"


def _random_arena(pp, branches, heads, d, cap, dev, seed, dist="normal"):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rows = branches * heads
    if dist == "student_t":
        # Student-t(3) * 0.7 with 1% of channels scaled by 8
        def draw():
            z = torch.randn(rows, cap, d, device=dev, generator=g)
            chi = torch.randn(rows, cap, d, 3, device=dev, generator=g).pow(2).sum(-1)
            t = z / torch.sqrt(chi / 3) * 0.7
            mask = torch.rand(d, device=dev, generator=g) < 0.01
            mask[int(torch.randint(0, d, (1,), device=dev, generator=g))] = True
            return torch.where(mask, t * 8, t)
    else:
        def draw():
            return torch.randn(rows, cap, d, device=dev, generator=g)
    ops = pp.int8_kv_ops
    k, ks = ops.quantize(draw())
    v, vs = ops.quantize(draw())
    return k, v, ks, vs, g


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("scratch", [False, True])
def test_batched_branches_match_single_branch_calls(pp, cuda, d, scratch):
    """The reference checks its batched forward against one sequence at a time
    (app/src/model/batch.rs:389-475).  Here: one call over a ragged batch of
    branches against one call per branch on that branch's rows of the same
    arena.  With fixed splits every row is computed and merged alone, so the
    two agree bit for bit; the automatic plan cuts rows differently in the
    two cases, so they agree to f32 rounding."""
    ops = pp.int8_kv_ops
    branches, heads, cap = 6, 4, 900
    k, v, ks, vs, g = _random_arena(pp, branches, heads, d, cap, cuda, 4000 + d + scratch)
    rows = branches * heads
    lens_h = [899, 1, 513, 0 if scratch else 7, 256, 640]
    lens = torch.tensor(lens_h, dtype=torch.int32, device=cuda)
    q = torch.randn(rows, d, device=cuda, generator=g)
    sk = torch.randn(rows, d, device=cuda, generator=g) if scratch else None
    sv = torch.randn(rows, d, device=cuda, generator=g) if scratch else None
    for split in (128, 0):
        batched = ops.decode_attention(q, k, v, ks, vs, lens, heads, scratch_k=sk, scratch_v=sv,
                                       out_dtype=torch.float32, split_tokens=split)
        for b in range(branches):
            rs = slice(b * heads, (b + 1) * heads)
            one = ops.decode_attention(q[rs], k[rs], v[rs], ks[rs], vs[rs], lens[b:b + 1], heads,
                                       scratch_k=None if sk is None else sk[rs], scratch_v=None if sv is None else sv[rs],
                                       out_dtype=torch.float32, split_tokens=split)
            if split:
                assert torch.equal(one, batched[rs]), f"branch {b}"
            else:
                np.testing.assert_allclose(host(one), host(batched[rs]), rtol=1e-5, atol=2e-6, err_msg=f"branch {b}")


@pytest.mark.parametrize("max_ctas", [0, 8])
@pytest.mark.parametrize("scratch", [False, True])
def test_head_dim_64_both_stage_configs(pp, oracle, cuda, max_ctas, scratch):
    """int8 head_dim 64 runs the 12-warp, 384-token-stage kernel when the
    arena holds at most 6144 tokens per CTA and the 15-warp, 480-token one
    above that: 64 rows x 2048 tokens on all SMs takes the first, on 8 CTAs
    the second.  Every row against the oracle, history and reference mode."""
    ops = pp.int8_kv_ops
    branches, heads, cap, d = 16, 4, 2048, 64
    k, v, ks, vs, g = _random_arena(pp, branches, heads, d, cap, cuda, 640 + max_ctas + scratch)
    rows = branches * heads
    lens_h = [cap, 1, 2047, 1023, 480, 481, 17, 0 if scratch else 5, 1500, 961, 384, 385, 2000, 33, 767, 1152]
    lens = torch.tensor(lens_h, dtype=torch.int32, device=cuda)
    q = torch.randn(rows, d, device=cuda, generator=g)
    sk = torch.randn(rows, d, device=cuda, generator=g) if scratch else None
    sv = torch.randn(rows, d, device=cuda, generator=g) if scratch else None
    if scratch:
        lens = torch.clamp(lens, max=cap - 1)  # reference mode: history plus the scratch token
    out = ops.decode_attention(q, k, v, ks, vs, lens, heads, scratch_k=sk, scratch_v=sv, out_dtype=torch.float32,
                               max_ctas=max_ctas)
    ref = _oracle_all(oracle, q, k, v, ks, vs, lens.cpu().numpy(), heads, sk=sk, sv=sv)
    np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=2e-5)


def _oracle_rows(oracle, q, k, v, ks, vs, lens, heads, pick, sk=None, sv=None):
    idx = torch.as_tensor(pick, device=k.device)
    sub = lambda t: t[idx].cpu().numpy()  # noqa: E731
    lk = np.asarray(lens)[np.asarray(pick) // heads]
    return oracle.attention(host(q[idx]), sub(k), sub(v), sub(ks), sub(vs), lk, 1,
                            sk=None if sk is None else host(sk[idx]), sv=None if sv is None else host(sv[idx]),
                            threads=oracle.max_threads())


def _oracle_all(oracle, q, k, v, ks, vs, lens, heads, sk=None, sv=None):
    """The oracle on every row of the arena, on all host threads."""
    return oracle.attention(host(q), k.cpu().numpy(), v.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy(),
                            np.asarray(lens), heads, sk=None if sk is None else host(sk),
                            sv=None if sv is None else host(sv), threads=oracle.max_threads())


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("qdt,odt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                     (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("split", [0, 48, 1000])
def test_history_mode_ragged_vs_oracle(pp, oracle, cuda, d, qdt, odt, split):
    branches, heads, cap = 6, 4, 700
    k, v, ks, vs, g = _random_arena(pp, branches, heads, d, cap, cuda, 7 + d)
    lens = [1, 700, 333, 16, 17, 650]
    q = torch.randn(branches * heads, d, device=cuda, generator=g).to(qdt)
    out = pp.int8_kv_ops.decode_attention(q, k, v, ks, vs, torch.tensor(lens, dtype=torch.int32, device=cuda), heads,
                                          out_dtype=odt, split_tokens=split)
    assert out.dtype == odt
    ref = _oracle_rows(oracle, q, k, v, ks, vs, lens, heads, list(range(branches * heads)))
    if odt == torch.float32:  # f32 output: BASELINE tolerance, and in fact far inside it
        np.testing.assert_allclose(host(out), ref, rtol=2e-3, atol=1e-3)
        np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=2e-5)
    else:
        assert_bf16_close(host(out), ref)


def test_invalid_lengths_give_nan_rows_and_status(pp, cuda):
    k, v, ks, vs, g = _random_arena(pp, 3, 2, 128, 64, cuda, 3)
    q = torch.randn(6, 128, device=cuda, generator=g)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = pp.int8_kv_ops.decode_attention(q, k, v, ks, vs, torch.tensor([0, 65, 64], dtype=torch.int32, device=cuda),
                                          2, status=status)
    o = host(out)
    assert np.isnan(o[:4]).all() and np.isfinite(o[4:]).all()
    assert int(status.item()) & pp._native.DEV_LENGTH_RANGE


def test_plan_reuse_across_layers(pp, oracle, cuda):
    """One ragged plan serves all layers of a step (DecodeMetadataCache reuse)."""
    ops = pp.int8_kv_ops
    branches, heads, d, cap, layers = 4, 4, 128, 300, 3
    lens = torch.tensor([300, 1, 77, 150], dtype=torch.int32, device=cuda)
    arenas = [_random_arena(pp, branches, heads, d, cap, cuda, 40 + i) for i in range(layers)]
    k0, v0, ks0, vs0, _ = arenas[0]
    arena = ops.arena_struct(k0, v0, ks0, vs0, heads)
    params = ops.attn_params(q_dtype=torch.bfloat16, out_dtype=torch.float32)
    ws = ops.new_workspace(arena, params, cuda)
    import ctypes as C
    pp._native.check(pp._native.lib.pp_b200_plan_ragged(C.byref(arena), C.byref(params), ops._ptr(lens), 0,
                                                         ops._ptr(ws), ws.numel(), ops._stream(lens)))
    for i, (k, v, ks, vs, g) in enumerate(arenas):
        q = torch.randn(branches * heads, d, device=cuda, generator=g).to(torch.bfloat16)
        out = ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32, workspace=ws,
                                   plan_ready=True)
        ref = _oracle_rows(oracle, q, k, v, ks, vs, lens.cpu().numpy(), heads, list(range(branches * heads)))
        np.testing.assert_allclose(host(out), ref, rtol=0, atol=2e-5)


def test_repeated_calls_on_one_plan_are_bit_identical(pp, oracle, cuda):
    """Rows split over several CTAs are merged by the CTA that finishes them
    last, counted in the workspace; the count must be back at zero after every
    call, so the same call repeated on one plan gives the same bits."""
    ops = pp.int8_kv_ops
    branches, heads, d, cap = 24, 16, 128, 2000
    lens = torch.tensor([2000, 1, 1999, 640, 17, 1500] * 4, dtype=torch.int32, device=cuda)
    k, v, ks, vs, g = _random_arena(pp, branches, heads, d, cap, cuda, 77)
    q = torch.randn(branches * heads, d, device=cuda, generator=g).to(torch.bfloat16)
    first = ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32)
    arena = ops.arena_struct(k, v, ks, vs, heads)
    params = ops.attn_params(q_dtype=torch.bfloat16, out_dtype=torch.float32)
    ws = ops.new_workspace(arena, params, cuda)
    import ctypes as C
    pp._native.check(pp._native.lib.pp_b200_plan_ragged(C.byref(arena), C.byref(params), ops._ptr(lens), 0,
                                                         ops._ptr(ws), ws.numel(), ops._stream(lens)))
    for _ in range(5):
        again = ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32, workspace=ws,
                                     plan_ready=True)
        assert torch.equal(again, first)
    rows = list(range(0, branches * heads, 7))
    ref = _oracle_rows(oracle, q, k, v, ks, vs, lens.cpu().numpy(), heads, rows)
    np.testing.assert_allclose(host(first)[rows], ref, rtol=0, atol=2e-5)


def test_prefetch_history_gives_the_same_bits(pp, cuda):
    """Layers that follow another layer's attention may stream their history
    before it completes; the outputs must not change."""
    ops = pp.int8_kv_ops
    branches, heads, d, cap, layers = 8, 16, 128, 3000, 4
    lens = torch.tensor([3000, 5, 2999, 1200, 17, 640, 3000, 1], dtype=torch.int32, device=cuda)
    arenas = [_random_arena(pp, branches, heads, d, cap, cuda, 60 + i) for i in range(layers)]
    qs = [torch.randn(branches * heads, d, device=cuda, generator=g).to(torch.bfloat16) for (_, _, _, _, g) in arenas]
    k0, v0, ks0, vs0, _ = arenas[0]
    ws = ops.new_workspace(ops.arena_struct(k0, v0, ks0, vs0, heads), ops.attn_params(), cuda)
    ops.plan_ragged(k0, v0, ks0, vs0, lens, heads, ws)
    runs = []
    for prefetch in (False, True):
        outs = []
        for i, (k, v, ks, vs, _) in enumerate(arenas):
            outs.append(ops.decode_attention(qs[i], k, v, ks, vs, lens, heads, out_dtype=torch.float32, workspace=ws,
                                             plan_ready=True, prefetch_history=prefetch and i > 0))
        torch.cuda.synchronize()
        runs.append(outs)
    for a, b in zip(*runs):
        assert torch.equal(a, b)
    with pytest.raises(pp.PreconditionError):
        ops.decode_attention(qs[0], k0, v0, ks0, vs0, lens, heads, workspace=ws, prefetch_history=True)


def test_prepare_self_check_passes(pp, cuda):
    pp.int8_kv_ops.prepare(cuda)


def test_cfg1_full_size(pp, oracle, cuda):
    """BASELINE config 1 at full size: 32 branches x 16 heads, d 128, context
    4096, bf16 q.  Every one of the 512 output rows against the oracle: bf16
    out (one bf16 ulp), f32 out with the stream-K plan and with the
    reference's fixed 128-token splits (2e-3 / 1e-3, and 1e-5 / 2e-5)."""
    branches, heads, d, L = 32, 16, 128, 4096
    k, v, ks, vs, g = _random_arena(pp, branches, heads, d, L, cuda, 1)
    q = torch.randn(branches * heads, d, device=cuda, generator=g).to(torch.bfloat16)
    lens = torch.full((branches,), L, dtype=torch.int32, device=cuda)
    ref = _oracle_all(oracle, q, k, v, ks, vs, lens.cpu().numpy(), heads)
    out = pp.int8_kv_ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.bfloat16)
    assert torch.isfinite(out.float()).all()
    assert_bf16_close(host(out), ref)
    for split in (0, 128):
        out32 = host(pp.int8_kv_ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32,
                                                     split_tokens=split))
        np.testing.assert_allclose(out32, ref, rtol=2e-3, atol=1e-3)
        np.testing.assert_allclose(out32, ref, rtol=1e-5, atol=2e-5)


def test_cfg4_long_context_split_sweep(pp, oracle, cuda):
    """8 branches x 16 heads, d 128, context 16384,
    heavy-tailed K/V with outlier channels.  Split factors 4, 8, 16, 32 and
    the stream-K plan, each checked on all 128 rows against the oracle."""
    branches, heads, d, L = 8, 16, 128, 16384
    k, v, ks, vs, g = _random_arena(pp, branches, heads, d, L, cuda, 4, dist="student_t")
    q = torch.randn(branches * heads, d, device=cuda, generator=g).to(torch.bfloat16)
    lens = torch.full((branches,), L, dtype=torch.int32, device=cuda)
    ref = _oracle_all(oracle, q, k, v, ks, vs, lens.cpu().numpy(), heads)
    for splits in (4, 8, 16, 32, 0):
        o = host(pp.int8_kv_ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32,
                                                 split_tokens=L // splits if splits else 0))
        assert np.isfinite(o).all()
        np.testing.assert_allclose(o, ref, rtol=2e-3, atol=1e-3, err_msg=f"splits {splits}")
        # tighter, for f32 reassociation over 16384 heavy-tailed terms whose signed sums cancel: measured
        # up to 1.4e-4 relative on a few outputs near 12
        np.testing.assert_allclose(o, ref, rtol=5e-4, atol=5e-5, err_msg=f"splits {splits}")
    ob = host(pp.int8_kv_ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.bfloat16))
    assert_bf16_close(ob, ref)


def test_a_stalled_wait_ends_with_a_status_not_a_hang(pp, oracle, cuda):
    """Failure detection without a fault: a bounded wait on a barrier that
    nothing completes gives up after its limit (2 ms here), the status word
    reports PP_DEV_WAIT_TIMEOUT, and the context keeps working."""
    N = pp._native
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    N.check(N.lib.pp_b200_diag_bounded_wait(C.c_void_p(status.data_ptr()), 2000,
                                            C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert int(status.item()) & N.DEV_WAIT_TIMEOUT
    assert "timed out" in N.status_message(int(status.item()))
    c = K.prep1()
    codes, scales = pp.int8_kv_ops.quantize(to_dev(c["x"], cuda))
    assert torch.isfinite(codes.float()).all()
