"""Quantize / dequantize / quantize-and-append on the B200 through the C ABI,
bit-exact against the oracle and against the reference kernels' own codes
(tests/golden/ref_int8kv.npz)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases as K

pytestmark = pytest.mark.gpu


def to_dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def u32(x):
    return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("seed", [0, 1])
def test_quantize_bit_exact_vs_oracle(pp, oracle, cuda, d, dtype, seed):
    g = np.random.Generator(np.random.PCG64(100 + seed))
    rows = 3000
    x = (g.standard_normal((rows, d), dtype=np.float32) * g.uniform(1e-3, 1e3, (rows, 1))).astype(np.float32)
    if dtype == torch.bfloat16:
        bits = K.to_bf16_bits(x)
        xt = to_dev(bits.view(np.int16), cuda).view(torch.bfloat16)
        ref_codes, ref_scales = oracle.quantize(bits, d)
    else:
        xt = to_dev(x, cuda)
        ref_codes, ref_scales = oracle.quantize(x)
    codes, scales = pp.int8_kv_ops.quantize(xt.reshape(1, rows, d))
    assert np.array_equal(codes.cpu().numpy().reshape(rows, d), ref_codes)
    assert np.array_equal(u32(scales.cpu().numpy().reshape(rows)), u32(ref_scales))


def _near_tie_rows(d, bf16, seed, rows=512):
    """Rows whose elements sit on, and a few units in the last place around,
    x / s = k + 0.5 for every code k, where the quotient's rounding decides
    the code.  Element 0 is the row maximum that sets s.  bf16 rows use
    power-of-two scales, so the ties are exact; f32 rows use arbitrary scales."""
    g = np.random.Generator(np.random.PCG64(900 + seed))
    out = np.zeros((rows, d), np.float32)
    for r in range(rows):
        if bf16:
            s = np.float32(2.0 ** int(g.integers(-30, 12)))
            m = np.float32(127) * s
        else:
            m = np.float32(127 * g.uniform(1e-3, 1e2))
            s = np.float32(np.float32(m) / np.float32(127))
        k = g.integers(-127, 127, d - 1)
        x = (k.astype(np.float32) + np.float32(0.5)) * s
        if bf16:
            bits = (x.view(np.uint32) >> 16).astype(np.int64) + g.integers(-1, 2, d - 1)
            x = (bits.astype(np.uint32) << 16).view(np.float32)
        else:
            x = (x.view(np.int32) + g.integers(-3, 4, d - 1).astype(np.int32)).view(np.float32)
        out[r, 0] = m if g.integers(0, 2) else -m
        out[r, 1:] = np.clip(x, -np.abs(m), np.abs(m))
    return out


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantize_near_ties_bit_exact(pp, oracle, cuda, d, dtype):
    """Codes of elements whose quotient x / s falls on or next to a half-integer,
    by the bulk quantizer and by quantize-and-append, equal the oracle's (exact
    f32 division, round half to even)."""
    bf16 = dtype == torch.bfloat16
    x = _near_tie_rows(d, bf16, d + bf16)
    rows = x.shape[0]
    if bf16:
        bits = K.to_bf16_bits(x)
        assert np.array_equal((bits.astype(np.uint32) << 16).view(np.float32), x)  # the rows are bf16 values
        xt = to_dev(bits.view(np.int16), cuda).view(torch.bfloat16)
        ref_codes, ref_scales = oracle.quantize(bits, d)
    else:
        xt = to_dev(x, cuda)
        ref_codes, ref_scales = oracle.quantize(x)
    codes, scales = pp.int8_kv_ops.quantize(xt.reshape(1, rows, d))
    assert np.array_equal(codes.cpu().numpy().reshape(rows, d), ref_codes)
    assert np.array_equal(u32(scales.cpu().numpy().reshape(rows)), u32(ref_scales))
    # the same rows through quantize-and-append (one token per (branch, head) row)
    heads = 16
    arena = pp.kv_cache.Int8KvArena.zeros(rows // heads, heads, d, 4, cuda)
    offs = torch.full((rows // heads,), 2, dtype=torch.int32, device=cuda)
    arena.append(xt, xt, offs)
    torch.cuda.synchronize()
    assert np.array_equal(arena.k[:, 2].cpu().numpy(), ref_codes)
    assert np.array_equal(arena.v[:, 2].cpu().numpy(), ref_codes)
    assert np.array_equal(u32(arena.k_scale[:, 2].cpu().numpy()), u32(ref_scales))


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                                    "oracle", "_ref", "int8_kv_ref.cubin")),
                    reason="reference kernels were not built (no reference tree when this checkout was built)")
def test_quantize_large_arena_live_against_reference_kernels(pp, cuda):
    """A cfg1-sized arena at the reference's head size (512 rows x 4096 tokens
    x 64, heavy-tailed values, every 7th token built on or next to half-integer
    quotients): codes and scales from pp_i8_scale + pp_i8_pack and from this
    library, byte for byte."""
    from ref_runner import RefInt8Kernels

    ref = RefInt8Kernels()
    g = torch.Generator(device=cuda)
    g.manual_seed(97)
    x = torch.randn(512, 4096, 64, device=cuda, generator=g)
    x = x * torch.exp(torch.randn(512, 4096, 1, device=cuda, generator=g))  # per-token magnitude spread
    # every 7th token: half-integer multiples of amax / 127 (quotients x / s on or next to ties)
    amax = x[:, ::7].abs().amax(-1, keepdim=True)
    ties = torch.randint(-254, 255, x[:, ::7].shape, device=cuda, generator=g).float() * 0.5
    ties[..., 0] = 127.0
    x[:, ::7] = ties * (amax / 127.0)
    want_codes, want_scales = ref.quantize(x.contiguous())
    codes, scales = pp.int8_kv_ops.quantize(x.contiguous())
    assert torch.equal(codes, want_codes)
    assert torch.equal(scales.view(torch.int32), want_scales.view(torch.int32))
    del x, ties


def test_quantize_matches_reference_kernel_codes(pp, cuda, golden):
    """Codes and scales equal the reference CUDA kernels' (pp_i8_scale/pack)."""
    ops = pp.int8_kv_ops
    c = K.prep1()
    codes, scales = ops.quantize(to_dev(c["x"], cuda))
    assert np.array_equal(codes.cpu().numpy(), golden["prep1_codes"])
    assert np.array_equal(u32(scales.cpu().numpy()), u32(golden["prep1_scales"]))
    for idx, (h, n, bias) in enumerate(K.CACHE_CASES):
        codes, scales = ops.quantize(to_dev(K.cache_data(h, n, bias), cuda))
        assert np.array_equal(codes.cpu().numpy(), golden[f"cache{idx}_codes"])
        assert np.array_equal(u32(scales.cpu().numpy()), u32(golden[f"cache{idx}_scales"]))
    e = K.edge_rows()
    codes, scales = ops.quantize(to_dev(e, cuda).reshape(1, -1, 64))
    assert np.array_equal(codes.cpu().numpy().reshape(e.shape), golden["edge_codes"])
    assert np.array_equal(u32(scales.cpu().numpy().reshape(-1)), u32(golden["edge_scales"]))


def test_quantize_bf16_input_matches_reference_on_widened_values(pp, cuda, golden):
    """bf16 K/V are widened exactly (int8_kv_ops.rs:12): feeding bf16 directly
    gives the reference kernels' codes for the widened f32 values."""
    c = K.hip_bf16()
    for name in ("k", "v"):
        bits = c[f"{name}_bits"].reshape(-1, 257, 64)
        t = to_dev(bits.view(np.int16), cuda).view(torch.bfloat16)
        codes, scales = pp.int8_kv_ops.quantize(t)
        assert K.sha(codes.cpu().numpy()) == str(golden[f"hip_{name}_codes_sha"])
        assert np.array_equal(u32(scales.cpu().numpy().reshape(-1)), u32(golden[f"hip_{name}_scales"].reshape(-1)))


def test_quantize_non_finite_is_reported(pp, cuda):
    x = torch.zeros(2, 4, 128, device=cuda)
    x[1, 2, 5] = float("nan")
    with pytest.raises(ValueError, match="non-finite INT8 KV input"):
        pp.int8_kv_ops.quantize(x)
    x[1, 2, 5] = float("inf")
    with pytest.raises(ValueError, match="non-finite"):
        pp.int8_kv_ops.quantize(x)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 128])
def test_dequantize_vs_oracle(pp, oracle, cuda, out_dtype, d):
    g = np.random.Generator(np.random.PCG64(5))
    x = g.standard_normal((7, 33, d), dtype=np.float32) * 3
    codes, scales = oracle.quantize(x)
    dc, ds = to_dev(codes, cuda), to_dev(scales, cuda)
    exact = pp.int8_kv_ops.dequantize(dc, ds, torch.float32, round_bf16=False).cpu().numpy()
    assert np.array_equal(u32(exact), u32(oracle.dequantize(codes, scales, False)))
    got = pp.int8_kv_ops.dequantize(dc, ds, out_dtype).float().cpu().numpy()
    want = oracle.dequantize(codes, scales, out_dtype == torch.bfloat16)
    assert np.array_equal(u32(got), u32(want))


def test_dequantize_unaligned_view_and_prefill_shape(pp, oracle, cuda):
    """The prefill path (int8_cache.rs:363-371 `prefill_prefix`: the whole int8
    history back to bf16) at a prefill-sized [16, 1024, 64], and the same codes
    through a 4-byte-offset view, which takes the element-wise kernel."""
    g = np.random.Generator(np.random.PCG64(6))
    x = g.standard_normal((16, 1024, 64), dtype=np.float32) * 2
    codes, scales = oracle.quantize(x)
    want = oracle.dequantize(codes, scales, True)
    dc, ds = to_dev(codes, cuda), to_dev(scales, cuda)
    got = pp.int8_kv_ops.dequantize(dc, ds, torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(u32(got), u32(want))
    buf = torch.empty(codes.size + 16, dtype=torch.uint8, device=cuda)
    view = buf[4:4 + codes.size].view(codes.shape)
    view.copy_(dc)
    assert view.data_ptr() % 16 == 4
    got2 = pp.int8_kv_ops.dequantize(view, ds, torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(u32(got2), u32(want))


def _arena_np(a):
    return (a.k.cpu().numpy(), a.v.cpu().numpy(), a.k_scale.cpu().numpy(), a.v_scale.cpu().numpy())


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quant_append_commit_ragged_bit_exact(pp, oracle, cuda, d, dtype):
    branches, heads, cap = 5, 3, 40
    g = np.random.Generator(np.random.PCG64(21))
    arena = pp.kv_cache.Int8KvArena.zeros(branches, heads, d, cap, cuda)
    ref = [x.copy() for x in _arena_np(arena)]
    rows = branches * heads
    for step, offs in enumerate(([0, 5, 39, 17, 1], [1, 6, 0, 18, 2], [2, 2, 2, 2, 2])):
        xk = g.standard_normal((rows, d), dtype=np.float32) * (step + 1)
        xv = g.standard_normal((rows, d), dtype=np.float32)
        if dtype == torch.bfloat16:
            xk, xv = K.bf16_to_f32(K.to_bf16_bits(xk)), K.bf16_to_f32(K.to_bf16_bits(xv))
        offsets = torch.tensor(offs, dtype=torch.int32, device=cuda)
        arena.append(to_dev(xk, cuda).to(dtype), to_dev(xv, cuda).to(dtype), offsets, commit=True)
        oracle.quant_append(xk, xv, heads, np.array(offs, np.uint32), True, *ref)
        got = _arena_np(arena)
        for a, b in zip(got, ref):
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_quant_append_partial_writes_placeholder(pp, oracle, cuda):
    branches, heads, d, cap = 2, 2, 128, 8
    arena = pp.kv_cache.Int8KvArena.zeros(branches, heads, d, cap, cuda)
    x = torch.randn(branches * heads, d, device=cuda)
    arena.append(x, x, torch.tensor([3, 3], dtype=torch.int32, device=cuda), commit=True)
    before = [t.clone() for t in (arena.k, arena.k_scale)]
    arena.append(x * 2, x * 2, torch.tensor([3, 4], dtype=torch.int32, device=cuda), commit=False)
    k = arena.k.cpu()
    assert not k[:2, 3].any() and (arena.k_scale[:2, 3] == 1).all()  # branch 0 slot 3 overwritten
    assert torch.equal(k[2:, 3], before[0][2:, 3].cpu())              # branch 1 slot 3 untouched
    assert not k[2:, 4].any() and (arena.v_scale[2:, 4] == 1).all()


def test_quant_append_offset_out_of_range_is_flagged_not_written(pp, cuda):
    arena = pp.kv_cache.Int8KvArena.zeros(2, 2, 64, 4, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    x = torch.randn(4, 64, device=cuda)
    arena.append(x, x, torch.tensor([4, 1], dtype=torch.int32, device=cuda), status=status)
    assert int(status.item()) & pp._native.DEV_OFFSET_RANGE
    assert not arena.k[:2].any() and arena.k[2:, 1].any()


def test_growth_copies_codes_and_scales_without_requantizing(pp, cuda):
    """int8_cache.rs:110-124: growth copies the committed prefix unchanged."""
    arena = pp.kv_cache.Int8KvArena.zeros(3, 2, 128, 64, cuda)
    lens = torch.tensor([63, 10, 0], dtype=torch.int32, device=cuda)
    arena.k.random_(0, 256)
    arena.v.random_(0, 256)
    arena.k_scale.uniform_(0.1, 1)
    arena.v_scale.uniform_(0.1, 1)
    big = arena.grown(128, lens)
    assert big.capacity == 128
    for r, n in enumerate([63, 63, 10, 10, 0, 0]):
        assert torch.equal(big.k[r, :n], arena.k[r, :n]) and torch.equal(big.v[r, :n], arena.v[r, :n])
        assert torch.equal(big.k_scale[r, :n], arena.k_scale[r, :n])
        assert not big.k[r, n:].any() and not big.k_scale[r, n:].any()


def test_cfg2_ragged_append_256_steps_codes_bit_exact(pp, oracle, cuda):
    """64 branches, 16 heads, d 128, initial lengths
    U[256, 8192], one bf16 N(0, 0.5^2) K/V token appended per branch per step
    for 256 steps.  After every step the int8 codes and scales of every
    appended token are checked bit-exactly against the oracle; at the first
    and last step and every 16th step the decode attention of all 1024 rows
    is checked against the oracle over a host copy of the arena that the
    checked appends keep up to date."""
    branches, heads, d = 64, 16, 128
    g = np.random.Generator(np.random.PCG64(2))
    lengths = g.integers(256, 8193, branches).astype(np.int64)
    cap = int(lengths.max()) + 256
    rows = branches * heads
    arena = pp.kv_cache.Int8KvArena.zeros(branches, heads, d, cap, cuda)
    tg = torch.Generator(device=cuda)
    tg.manual_seed(2)
    arena.k.random_(0, 256, generator=tg)
    arena.v.random_(0, 256, generator=tg)
    arena.k_scale.uniform_(0.005, 0.05, generator=tg)
    arena.v_scale.uniform_(0.005, 0.05, generator=tg)
    mirror = [t.cpu().numpy() for t in (arena.k, arena.v, arena.k_scale, arena.v_scale)]
    lens_dev = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    row_idx = torch.arange(rows, device=cuda)
    checked = 0
    for step in range(256):
        xk = (torch.randn(rows, d, device=cuda, generator=tg) * 0.5).to(torch.bfloat16)
        xv = (torch.randn(rows, d, device=cuda, generator=tg) * 0.5).to(torch.bfloat16)
        arena.append(xk, xv, lens_dev)
        slot_np = lens_dev.repeat_interleave(heads).cpu().numpy()
        slot = torch.from_numpy(slot_np).to(cuda).long()
        got_k = arena.k[row_idx, slot].cpu().numpy()
        got_ks = arena.k_scale[row_idx, slot].cpu().numpy()
        got_v = arena.v[row_idx, slot].cpu().numpy()
        got_vs = arena.v_scale[row_idx, slot].cpu().numpy()
        bk = xk.view(torch.int16).cpu().numpy().view(np.uint16)
        bv = xv.view(torch.int16).cpu().numpy().view(np.uint16)
        ck, sk = oracle.quantize(bk, d)
        cv, sv = oracle.quantize(bv, d)
        assert np.array_equal(got_k, ck) and np.array_equal(got_v, cv), f"codes differ at step {step}"
        assert np.array_equal(u32(got_ks), u32(sk)) and np.array_equal(u32(got_vs), u32(sv))
        r = np.arange(rows)
        mirror[0][r, slot_np], mirror[1][r, slot_np] = ck, cv
        mirror[2][r, slot_np], mirror[3][r, slot_np] = sk, sv
        lens_dev += 1
        if step == 0 or step % 16 == 15:
            q = torch.randn(rows, d, device=cuda, generator=tg).to(torch.bfloat16)
            out = arena.attention(q, lens_dev, out_dtype=torch.float32)
            ref = oracle.attention(q.float().cpu().numpy(), *mirror, lens_dev.cpu().numpy(), heads,
                                   threads=oracle.max_threads())
            got = out.cpu().numpy()
            np.testing.assert_allclose(got, ref, rtol=2e-3, atol=1e-3, err_msg=f"step {step}")
            checked += 1
    assert checked == 17
