"""The no-allocation attention entry point (pp_b200_decode_attention_static).

It exists for callers that cannot allocate device memory when they call
attention, e.g. a host that gives a plugin only its input and output buffers
or a serving loop that forbids cudaMalloc after start-up.  It must produce the
same results as pp_b200_decode_attention, which takes a caller workspace.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.  It also passes on its own in
a fresh process (the first call on the device does the one-time set-up)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _static_call(pp, q, k, v, ks, vs, lens, heads, out, *, sk=None, sv=None, split=0):
    ops, N = pp.int8_kv_ops, pp._native
    arena = ops.arena_struct(k, v, ks, vs, heads)
    params = ops.attn_params(split_tokens=split, q_dtype=q.dtype, out_dtype=out.dtype)
    return N.lib.pp_b200_decode_attention_static(C.byref(arena), C.byref(params), ops._ptr(q), ops._ptr(sk),
                                                 ops._ptr(sv), ops._ptr(lens), ops._ptr(out), None, ops._stream(q))


def test_static_scratch_matches_workspace_entry_point_on_consecutive_calls(pp, cuda):
    ops, N = pp.int8_kv_ops, pp._native
    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    branches, heads, d, cap = 6, 16, 128, 1500
    rows = branches * heads
    k, ks = ops.quantize(torch.randn(rows, cap, d, device=cuda, generator=g))
    v, vs = ops.quantize(torch.randn(rows, cap, d, device=cuda, generator=g))
    # two calls in a row with different queries and ragged lengths
    for call, lens_list in enumerate(([1500, 1, 700, 333, 64, 1499], [17, 1500, 1500, 2, 900, 1024])):
        lens = torch.tensor(lens_list, dtype=torch.int32, device=cuda)
        q = torch.randn(rows, d, device=cuda, generator=g).to(torch.bfloat16)
        out = torch.empty(rows, d, dtype=torch.float32, device=cuda)
        N.check(_static_call(pp, q, k, v, ks, vs, lens, heads, out))
        want = ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=2e-5,
                                   err_msg=f"call {call}")


def test_static_scratch_reference_mode_matches(pp, cuda):
    """Reference mode (f32 scratch token, head_dim 64), two calls in a row."""
    ops, N = pp.int8_kv_ops, pp._native
    g = torch.Generator(device=cuda)
    g.manual_seed(12)
    branches, heads, d, cap = 3, 4, 64, 300
    rows = branches * heads
    k, ks = ops.quantize(torch.randn(rows, cap, d, device=cuda, generator=g))
    v, vs = ops.quantize(torch.randn(rows, cap, d, device=cuda, generator=g))
    for pasts in ([0, 300, 150], [299, 7, 64]):
        past = torch.tensor(pasts, dtype=torch.int32, device=cuda)
        q = torch.randn(rows, d, device=cuda, generator=g)
        sk = torch.randn(rows, d, device=cuda, generator=g)
        sv = torch.randn(rows, d, device=cuda, generator=g)
        out = torch.empty(rows, d, dtype=torch.float32, device=cuda)
        N.check(_static_call(pp, q, k, v, ks, vs, past, heads, out, sk=sk, sv=sv, split=128))
        want = ops.attention(q.reshape(rows, 1, d), k, v, ks, vs, sk.reshape(rows, 1, d), sv.reshape(rows, 1, d), past,
                             heads, 128)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), want.reshape(rows, d).cpu().numpy(), rtol=0, atol=2e-5)


def test_static_scratch_rejects_geometry_beyond_its_size(pp, cuda):
    """A workspace larger than the 4 MiB scratch is refused before any launch."""
    ops, N = pp.int8_kv_ops, pp._native
    branches, heads, d, cap = 64, 16, 128, 8192
    rows = branches * heads
    k = torch.zeros(rows, cap, d, dtype=torch.uint8, device=cuda)
    ks = torch.zeros(rows, cap, dtype=torch.float32, device=cuda)
    q = torch.zeros(rows, d, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(rows, d, dtype=torch.bfloat16, device=cuda)
    lens = torch.full((branches,), cap, dtype=torch.int32, device=cuda)
    status = _static_call(pp, q, k, k, ks, ks, lens, heads, out, split=64)
    assert status == N.STATUS_PRECONDITION
    assert "static" in N.last_error() and "workspace" in N.last_error()


def test_static_scratch_refuses_plan_reuse(pp, cuda):
    """PP_ATTN_PLAN_READY would reuse a plan that another call may have
    overwritten in the shared scratch: refused before any launch."""
    ops, N = pp.int8_kv_ops, pp._native
    k = torch.zeros(4, 64, 128, dtype=torch.uint8, device=cuda)
    ks = torch.ones(4, 64, dtype=torch.float32, device=cuda)
    q = torch.zeros(4, 128, dtype=torch.float32, device=cuda)
    out = torch.zeros(4, 128, dtype=torch.float32, device=cuda)
    lens = torch.full((1,), 64, dtype=torch.int32, device=cuda)
    arena = ops.arena_struct(k, k, ks, ks, 4)
    params = ops.attn_params(plan_ready=True)
    st = N.lib.pp_b200_decode_attention_static(C.byref(arena), C.byref(params), ops._ptr(q), None, None,
                                               ops._ptr(lens), ops._ptr(out), None, ops._stream(q))
    assert st == N.STATUS_PRECONDITION
    assert "caller-owned workspace" in N.last_error()


def test_static_scratch_default_params_and_no_device_allocation(pp, cuda):
    """params = NULL takes the defaults (f32 q and out, stream-K plan) and
    matches the workspace entry point; a run of calls after the first leaves
    the device's free memory unchanged (nothing is allocated)."""
    ops, N = pp.int8_kv_ops, pp._native
    g = torch.Generator(device=cuda)
    g.manual_seed(13)
    branches, heads, d, cap = 4, 8, 128, 900
    rows = branches * heads
    k, ks = ops.quantize(torch.randn(rows, cap, d, device=cuda, generator=g))
    v, vs = ops.quantize(torch.randn(rows, cap, d, device=cuda, generator=g))
    lens = torch.tensor([900, 3, 512, 77], dtype=torch.int32, device=cuda)
    q = torch.randn(rows, d, device=cuda, generator=g)
    out = torch.empty(rows, d, dtype=torch.float32, device=cuda)
    arena = ops.arena_struct(k, v, ks, vs, heads)

    def call():
        N.check(N.lib.pp_b200_decode_attention_static(C.byref(arena), None, ops._ptr(q), None, None, ops._ptr(lens),
                                                      ops._ptr(out), None, ops._stream(q)))

    call()
    want = ops.decode_attention(q, k, v, ks, vs, lens, heads, out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=2e-5)
    free_before, _ = torch.cuda.mem_get_info(cuda)
    for _ in range(8):
        call()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(cuda)
    assert free_after == free_before
    np.testing.assert_allclose(out.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=2e-5)
