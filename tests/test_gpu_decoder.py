"""Decoder-step kernels on the B200 through the C ABI.

QKV RoPE and SwiGLU are compared bit for bit with the reference's own
pp_graph_qkv / pp_graph_swiglu outputs (tests/golden/ref_graph.npz); the
head_dim-128 generalisation and RMSNorm against the oracle within one bf16
unit (the oracle's reciprocal square root is the C library's); the fused
append against the unfused kernel and the oracle quantizer bit for bit; the
whole synthetic decoder step against a plain PyTorch f32 restatement."""
from __future__ import annotations

import math
import os

import numpy as np
import pytest
import torch

import cases as K

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_graph.npz")


@pytest.fixture(scope="module")
def graph_golden():
    return np.load(GOLDEN)


def dev(x: np.ndarray, dt: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda().to(dt)


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("bf", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", K.QKV_CASES, ids=[c[0] for c in K.QKV_CASES])
def test_qkv_rope_bit_exact_with_reference_kernel(pp, cuda, graph_golden, case, bf):
    name, seed, rows, heads, dim, mc = case
    c = K.qkv_case(seed, rows, heads, dim, mc)
    dt = torch.bfloat16 if bf else torch.float32
    out = pp.decoder.qkv_rope(dev(c["qkv"], dt), dev(c["params"], dt),
                              torch.from_numpy(c["positions"].astype(np.int32)).cuda(), heads, dim, mc)
    np.testing.assert_array_equal(bits(out).ravel(), graph_golden[f"{name}_{'bf16' if bf else 'f32'}"].ravel())


@pytest.mark.parametrize("bf", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", K.SWIGLU_CASES, ids=[c[0] for c in K.SWIGLU_CASES])
def test_swiglu_bit_exact_with_reference_kernel(pp, cuda, graph_golden, case, bf):
    name, seed, rows, hidden = case
    dt = torch.bfloat16 if bf else torch.float32
    out = pp.decoder.swiglu(dev(K.swiglu_case(seed, rows, hidden), dt))
    np.testing.assert_array_equal(bits(out).ravel(), graph_golden[f"{name}_{'bf16' if bf else 'f32'}"].ravel())


def _ulps(a: np.ndarray, b: np.ndarray) -> int:
    return int(np.abs(a.astype(np.int32) - b.astype(np.int32)).max())


def test_qkv_rope_head_dim_128_vs_oracle(pp, oracle, cuda):
    rows, heads, dim, mc = 9, 16, 128, 2048
    c = K.qkv_case(77, rows, heads, dim, mc)
    out = pp.decoder.qkv_rope(dev(c["qkv"], torch.bfloat16), dev(c["params"], torch.bfloat16),
                              torch.from_numpy(c["positions"].astype(np.int32)).cuda(), heads, dim, mc)
    want = oracle.qkv_rope(K.to_bf16_bits(c["qkv"]), K.to_bf16_bits(c["params"]), c["positions"], rows, heads, dim,
                           mc, bf=True)
    got = bits(out).reshape(want.shape)
    assert _ulps(got, want) <= 1 and (got != want).mean() < 0.01
    np.testing.assert_array_equal(got[2], want[2])  # v passes through untouched


def test_qkv_rope_append_matches_unfused_and_quantizer(pp, oracle, cuda):
    D = pp.decoder
    rows, heads, dim, mc, cap = 6, 16, 128, 512, 40
    c = K.qkv_case(78, rows, heads, dim, mc)
    qkv, params = dev(c["qkv"], torch.bfloat16), dev(c["params"], torch.bfloat16)
    pos = torch.from_numpy(c["positions"].astype(np.int32)).cuda()
    planes = D.qkv_rope(qkv, params, pos, heads, dim, mc)
    arena = pp.kv_cache.Int8KvArena.zeros(rows, heads, dim, cap, cuda)
    arena.k.fill_(7)
    arena.k_scale.fill_(3.0)
    offs = torch.tensor([0, 39, 5, 17, 1, 38], dtype=torch.int32, device=cuda)
    q, sk, sv = D.qkv_rope_append(qkv, params, pos, arena, offs, mc)
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.int16), planes[0].view(torch.int16))
    assert torch.equal(sk, planes[1].float()) and torch.equal(sv, planes[2].float())
    slot = offs.repeat_interleave(heads).long()
    r = torch.arange(rows * heads, device=cuda)
    for codes, scales, plane in ((arena.k, arena.k_scale, planes[1]), (arena.v, arena.v_scale, planes[2])):
        want_codes, want_scales = oracle.quantize(bits(plane), dim)
        np.testing.assert_array_equal(codes[r, slot].cpu().numpy(), want_codes)
        np.testing.assert_array_equal(scales[r, slot].cpu().numpy().view(np.uint32), want_scales.view(np.uint32))
    untouched = torch.ones(rows * heads, cap, dtype=torch.bool, device=cuda)
    untouched[r, slot] = False
    assert (arena.k[untouched] == 7).all() and (arena.k_scale[untouched] == 3.0).all()
    # partial query: placeholder codes and unit scale
    D.qkv_rope_append(qkv, params, pos, arena, offs, mc, commit=False)
    torch.cuda.synchronize()
    assert (arena.k[r, slot] == 0).all() and (arena.v_scale[r, slot] == 1.0).all()


def test_qkv_rope_append_reports_out_of_range_slots(pp, cuda):
    D, N = pp.decoder, pp._native
    rows, heads, dim, mc, cap = 2, 2, 64, 16, 8
    c = K.qkv_case(79, rows, heads, dim, mc)
    qkv, params = dev(c["qkv"], torch.bfloat16), dev(c["params"], torch.bfloat16)
    arena = pp.kv_cache.Int8KvArena.zeros(rows, heads, dim, cap, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    D.qkv_rope_append(qkv, params, torch.tensor([0, 3], dtype=torch.int32, device=cuda), arena,
                      torch.tensor([2, 8], dtype=torch.int32, device=cuda), mc, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & N.DEV_OFFSET_RANGE
    assert (arena.k_scale[2:] == 0).all() and (arena.k_scale[:2, 2] > 0).all()
    status.zero_()
    D.qkv_rope(qkv, params, torch.tensor([0, 16], dtype=torch.int32, device=cuda), heads, dim, mc, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & N.DEV_POSITION_RANGE


@pytest.mark.parametrize("width", [2048, 200])  # 16-byte vector path and the strided path
def test_rmsnorm_vs_oracle_and_in_place_residual(pp, oracle, cuda, width):
    D = pp.decoder
    g = np.random.Generator(np.random.PCG64(81))
    rows = 5
    x = K.bf16_exact(g.standard_normal((rows, width)).astype(np.float32) * 2)
    r = K.bf16_exact(g.standard_normal((rows, width)).astype(np.float32))
    w = K.bf16_exact(1 + 0.1 * g.standard_normal(width).astype(np.float32))
    xt, rt, wt = dev(x, torch.bfloat16), dev(r, torch.bfloat16), dev(w, torch.bfloat16)
    out = D.rmsnorm(xt, wt)
    want, _ = oracle.rmsnorm(K.to_bf16_bits(x), K.to_bf16_bits(w), rows, width, 1e-6, bf=True)
    assert _ulps(bits(out), want) <= 1
    out2 = D.rmsnorm(xt, wt, residual=rt, x_sum=xt)  # x <- x + r in place
    want2, xs = oracle.rmsnorm(K.to_bf16_bits(x), K.to_bf16_bits(w), rows, width, 1e-6, bf=True,
                               residual=K.to_bf16_bits(r))
    np.testing.assert_array_equal(bits(xt), xs)
    assert _ulps(bits(out2), want2) <= 1


def _torch_step(m, x: torch.Tensor, past: torch.Tensor, k_hist, v_hist, ks_hist, vs_hist) -> torch.Tensor:
    """The decode step in plain PyTorch f32 (history dequantized as the
    reference does, bf16(i8 * s)); the model's bf16 rounding is not repeated,
    so this is a loose check of the wiring, not of the rounding."""
    cfg = m.cfg
    H, d, W = cfg.heads, cfg.head_dim, cfg.width
    B = x.shape[0]

    def rms(v, w):
        return v * torch.rsqrt((v * v).mean(-1, keepdim=True) + 1e-6) * w.float()

    h = x.float()
    for li, L in enumerate(m.layers):
        qkv = rms(h, L["norm1"]) @ L["qkv"].float().t()
        q, k, v = qkv[:, :W].reshape(B, H, d), qkv[:, W:2 * W].reshape(B, H, d), qkv[:, 2 * W:].reshape(B, H, d)
        p = L["rope"].float()
        q, k = rms(q, p[:d]), rms(k, p[d:2 * d])
        cos = p[2 * d:2 * d + cfg.max_context * d // 2].reshape(cfg.max_context, d // 2)
        sin = p[2 * d + cfg.max_context * d // 2:].reshape(cfg.max_context, d // 2)
        c, s = cos[past.long()][:, None, :], sin[past.long()][:, None, :]

        def rope(t):
            e, o = t[..., 0::2], t[..., 1::2]
            return torch.stack([e * c - o * s, e * s + o * c], -1).reshape(t.shape)

        q, k = rope(q), rope(k)
        att = torch.empty(B, H, d, device=x.device)
        for b in range(B):
            n = int(past[b])
            for hh in range(H):
                row = b * H + hh
                kh = (k_hist[li][row, :n].to(torch.int8).float() * ks_hist[li][row, :n, None]).to(torch.bfloat16).float()
                vh = (v_hist[li][row, :n].to(torch.int8).float() * vs_hist[li][row, :n, None]).to(torch.bfloat16).float()
                keys = torch.cat([kh, k[b, hh][None]])
                vals = torch.cat([vh, v[b, hh][None]])
                w = torch.softmax(keys @ q[b, hh] / math.sqrt(d), 0)
                att[b, hh] = w @ vals
        h = h + att.reshape(B, W) @ L["proj"].float().t()
        gu = rms(h, L["norm2"]) @ L["gate_up"].float().t()
        gate, up = gu[:, :cfg.ffn_hidden], gu[:, cfg.ffn_hidden:]
        h = h + (torch.nn.functional.silu(gate) * up) @ L["down"].float().t()
    return rms(h, m.final_norm)


def test_synthetic_decoder_step_matches_torch_restatement(pp, cuda):
    D = pp.decoder
    cfg = D.DecoderConfig(layers=3, width=512, heads=4, head_dim=128, ffn_hidden=1024, max_context=128)
    m = D.SyntheticDecoder(cfg, branches=3, capacity=100, device=cuda, seed=5)
    m.fill_history(None, seed=6)
    past = torch.tensor([17, 0, 99], dtype=torch.int32, device=cuda)
    hist = [(a.k.clone(), a.v.clone(), a.k_scale.clone(), a.v_scale.clone()) for a in m.arenas]
    x = torch.randn(3, cfg.width, device=cuda, generator=torch.Generator(device=cuda).manual_seed(7)).to(torch.bfloat16)
    want = _torch_step(m, x, past, *zip(*hist))
    got = m.step(x.clone(), past).float()
    torch.cuda.synchronize()
    assert int(m.status.item()) == 0
    cos = torch.nn.functional.cosine_similarity(got, want, dim=-1)
    assert (cos > 0.995).all(), cos
    # the step appended each branch's new token at slot past[b] of every layer
    rows = torch.arange(3 * cfg.heads, device=cuda)
    slot = past.repeat_interleave(cfg.heads).long()
    assert all((a.k_scale[rows, slot] != hk[2][rows, slot]).all() for a, hk in zip(m.arenas, hist))


def test_captured_step_replays_the_eager_step(pp, cuda):
    """The step recorded as a CUDA graph gives the eager step's bits, and its
    history length advances by one per replay."""
    D = pp.decoder
    cfg = D.DecoderConfig(layers=2, width=256, heads=2, head_dim=128, ffn_hidden=512, max_context=64)
    m = D.SyntheticDecoder(cfg, branches=3, capacity=64, device=cuda, seed=8)
    m.fill_history(None, seed=9)
    gen = torch.Generator(device=cuda).manual_seed(10)
    xs = [torch.randn(3, cfg.width, device=cuda, generator=gen).to(torch.bfloat16) for _ in range(3)]
    start = torch.tensor([5, 0, 30], dtype=torch.int32, device=cuda)
    snap = [(a.k.clone(), a.v.clone(), a.k_scale.clone(), a.v_scale.clone()) for a in m.arenas]
    eager = []
    for i, x in enumerate(xs):
        eager.append(m.step(x.clone(), start + i).clone())
    for a, (k, v, ks, vs) in zip(m.arenas, snap):  # back to the history before the eager steps
        a.k.copy_(k), a.v.copy_(v), a.k_scale.copy_(ks), a.v_scale.copy_(vs)
    past = start.clone()
    cap = m.capture(past)
    past.copy_(start)
    for a, (k, v, ks, vs) in zip(m.arenas, snap):
        a.k.copy_(k), a.v.copy_(v), a.k_scale.copy_(ks), a.v_scale.copy_(vs)
    for i, x in enumerate(xs):
        got = cap.replay(x)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), eager[i].view(torch.int16)), f"step {i}"
    assert torch.equal(past, start + 3)


def test_decoder_step_without_history_prefetch_gives_the_same_bits(pp, cuda):
    D = pp.decoder
    cfg = D.DecoderConfig(layers=2, width=256, heads=2, head_dim=128, ffn_hidden=512, max_context=64)
    m = D.SyntheticDecoder(cfg, branches=3, capacity=64, device=cuda, seed=11)
    m.fill_history(None, seed=12)
    past = torch.tensor([40, 7, 0], dtype=torch.int32, device=cuda)
    x = torch.randn(3, cfg.width, device=cuda, generator=torch.Generator(device=cuda).manual_seed(13)).to(torch.bfloat16)
    with_prefetch = m.step(x.clone(), past).clone()
    m.prefetch = False
    without = m.step(x.clone(), past).clone()
    torch.cuda.synchronize()
    assert torch.equal(with_prefetch.view(torch.int16), without.view(torch.int16))


def test_cfg3_every_layer_attention_vs_oracle(pp, oracle, cuda):
    """BASELINE config 3 at full size (24 layers, width 2048, 16 x 128 heads,
    SwiGLU 5632, 16 branches at context 2048): one decode step, and after
    each layer's attention the output of all 256 rows is checked against the
    oracle on the same arena, query and f32 scratch token (reference mode:
    the history of `past` int8 tokens plus the current token in f32)."""
    import oracle as O

    D = pp.decoder
    cfg = D.DecoderConfig()  # 24 x 2048, 16 x 128, 5632
    B, L0 = 16, 2048
    m = D.SyntheticDecoder(cfg, branches=B, capacity=L0 + 8, device=cuda, seed=31)
    m.fill_history(None, seed=32)
    past = torch.full((B,), L0, dtype=torch.int32, device=cuda)
    x = (torch.randn(B, cfg.width, device=cuda, generator=torch.Generator(device=cuda).manual_seed(33)) * 0.5)
    seen = []

    def probe(li, q, sk, sv, arena, att):
        torch.cuda.synchronize()
        ref = O.attention(q.float().cpu().numpy(), arena.k.cpu().numpy(), arena.v.cpu().numpy(),
                          arena.k_scale.cpu().numpy(), arena.v_scale.cpu().numpy(), past.cpu().numpy(), cfg.heads,
                          sk=sk.cpu().numpy(), sv=sv.cpu().numpy(), threads=O.max_threads())
        got = att.float().cpu().numpy()
        ref_b = O.bf16_round(ref)
        mag = np.maximum(np.abs(ref_b), np.float32(2.0**-126))
        ulp = np.exp2(np.floor(np.log2(mag)) - 7).astype(np.float32)
        bad = np.abs(got - ref_b) > np.maximum(ulp, 1e-3)
        assert not bad.any(), f"layer {li}: {bad.sum()} of {bad.size} attention outputs beyond one bf16 ulp"
        seen.append(li)

    out = m.step(x.to(torch.bfloat16), past, probe=probe)
    torch.cuda.synchronize()
    assert int(m.status.item()) == 0
    assert seen == list(range(cfg.layers))
    assert torch.isfinite(out.float()).all()
