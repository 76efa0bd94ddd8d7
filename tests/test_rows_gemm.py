"""Decode-row GEMM (pp_b200_rows_gemm over weights packed by
pp_b200_rows_gemm_pack): out = x @ w.T for <= 16 rows, bf16 in and out with
f32 accumulation, replacing the reference's matmul on the decode rows
(batch.rs:134,155-170).  Checked against PyTorch in f32: the kernel's
output is the f32 sum rounded once to bf16, so it may differ from the
rounded f32 reference by one bf16 unit where the two sums straddle a
rounding boundary."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch


def test_rows_gemm_rejects_bad_geometry(pp):
    N = pp._native
    p = C.c_void_p(0x10000)

    def call(m, n, k, ldx=None, ldo=None, x=p, w=p, out=p):
        return N.lib.pp_b200_rows_gemm(x, ldx or k, w, out, ldo or n, m, n, k, None, None)

    assert call(0, 64, 64) == N.STATUS_PRECONDITION
    assert call(17, 64, 64) == N.STATUS_PRECONDITION
    assert call(4, 60, 64) == N.STATUS_PRECONDITION
    assert call(4, 64, 96) == N.STATUS_PRECONDITION
    assert call(4, 64, 64, ldx=68) == N.STATUS_PRECONDITION  # 136-byte x rows
    assert call(4, 64, 64, w=C.c_void_p(0x10008)) == N.STATUS_PRECONDITION  # packed w misaligned
    assert call(4, 64, 64, x=None) == N.STATUS_PRECONDITION
    assert "rows_gemm" in N.last_error()
    assert N.lib.pp_b200_rows_gemm_pack(p, 64, 60, 64, p, None) == N.STATUS_PRECONDITION
    assert N.lib.pp_b200_rows_gemm_pack(p, 60, 64, 64, p, None) == N.STATUS_PRECONDITION


def _check(got: torch.Tensor, x: torch.Tensor, w: torch.Tensor):
    want = (x.float() @ w.float().t())
    g, r = got.float().cpu().numpy(), want.cpu().numpy()
    ulp = np.abs(want.to(torch.bfloat16).float().cpu().numpy()) * 2.0 ** -7
    np.testing.assert_array_less(np.abs(g - r), ulp + 1e-6 * np.abs(r).max() + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("m", [1, 5, 16])
@pytest.mark.parametrize("n,k", [(6144, 2048), (2048, 2048), (11264, 2048), (2048, 5632), (8, 64), (200, 192),
                                 (1536, 512), (512, 1024), (64, 6144), (16, 4160), (256, 9216), (72, 3136)])
def test_rows_gemm_matches_f32(pp, cuda, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).to(torch.bfloat16)
    out = pp.decoder.rows_gemm(x, pp.decoder.rows_gemm_pack(w), n)
    _check(out, x, w)


@pytest.mark.gpu
def test_rows_gemm_strided_and_deterministic(pp, cuda):
    """Row strides wider than k (views) and repeated calls: bit-identical
    results, nothing written past n."""
    g = torch.Generator(device=cuda).manual_seed(3)
    xb = torch.randn(16, 2048 + 64, device=cuda, generator=g).to(torch.bfloat16)
    wb = (torch.randn(2048, 2048 + 128, device=cuda, generator=g) / 45).to(torch.bfloat16)
    x, w = xb[:, :2048], wb[:, :2048]
    ob = torch.zeros(16, 2048 + 8, dtype=torch.bfloat16, device=cuda)
    out = ob[:, :2048]
    packed = pp.decoder.rows_gemm_pack(w)  # from a strided view of a wider matrix
    pp.decoder.rows_gemm(x, packed, 2048, out=out)
    first = out.clone()
    for _ in range(3):
        pp.decoder.rows_gemm(x, packed, 2048, out=out)
        assert torch.equal(out.view(torch.int16), first.view(torch.int16))
    _check(out, x, w)
    assert torch.count_nonzero(ob[:, 2048:]) == 0


@pytest.mark.gpu
def test_rows_gemm_back_to_back_shapes(pp, cuda):
    """The four projection shapes of a decoder layer launched back to back
    (each streams its weights while the previous one finishes), 3 rows."""
    g = torch.Generator(device=cuda).manual_seed(4)
    shapes = [(1536, 512), (512, 512), (2048, 512), (512, 1024), (6144, 2048), (2048, 5632)]
    xs = [torch.randn(3, k, device=cuda, generator=g).to(torch.bfloat16) for n, k in shapes]
    ws = [(torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).to(torch.bfloat16) for n, k in shapes]
    packed = [pp.decoder.rows_gemm_pack(w) for w in ws]
    outs = [pp.decoder.rows_gemm(x, p, w.shape[0]) for x, w, p in zip(xs, ws, packed)]
    for o, x, w in zip(outs, xs, ws):
        _check(o, x, w)


@pytest.mark.gpu
def test_rows_gemm_pack_layout(pp, cuda):
    """Block b of 8 rows at b * k * 16 bytes as [k / 64][row][64], 16-byte chunk
    c of row r at position c ^ r."""
    n, k = 16, 128
    w = torch.arange(n * k, device=cuda, dtype=torch.float32).to(torch.bfloat16).view(n, k)
    packed = pp.decoder.rows_gemm_pack(w).view(torch.bfloat16).view(n // 8, k // 64, 8, 8, 8).cpu()
    ref = w.cpu().view(n // 8, 8, k // 64, 8, 8).permute(0, 2, 1, 3, 4)  # [blk][chunk64][row][c][8]
    for r in range(8):
        for c in range(8):
            assert torch.equal(packed[:, :, r, c ^ r], ref[:, :, r, c])
