"""The C ABI library on the CPU: it loads, exports exactly what
include/pp_b200.h declares, and its host-side logic (geometry checks, batch
rows, write offsets, branch partition) behaves like the reference's.
No test here launches a kernel."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pp_b200.h")


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"\b(pp_b200_\w+)\s*\(", text))


def test_header_and_binding_agree(pp):
    assert declared_symbols() == set(pp._native.EXPORTED)


def test_library_exports_every_declared_symbol(pp):
    lib = C.CDLL(pp._native.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", pp._native.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (pp_b200_\w+)", out))
    assert exported == declared_symbols()


def test_abi_version(pp):
    assert pp.abi_version() == 1


@pytest.mark.parametrize("logical", [1, 16, 17, 32, 64, 96, 1000])
def test_batch_rows_preserve_requested_counts(pp, logical):
    """batch_geometry.rs:23-28."""
    kv = pp.kv_cache
    assert kv.checked_batch_rows(logical, 1) == logical
    assert kv.checked_batch_rows(logical, 2) == logical * 2


def test_batch_rows_reject_invalid_geometry(pp):
    """batch_geometry.rs:31-38."""
    kv = pp.kv_cache
    with pytest.raises(pp.PreconditionError):
        kv.checked_batch_rows(0, 1)
    with pytest.raises(pp.PreconditionError):
        kv.checked_batch_rows(1, 3)
    with pytest.raises(pp.PreconditionError):
        kv.checked_batch_rows(2**64 - 1, 2)
    last = (2**32 - 1) // 9
    assert kv.checked_batch_rows(last, 2) == last * 2
    with pytest.raises(pp.PreconditionError):
        kv.checked_batch_rows(last + 1, 1)


def test_write_offsets_validation(pp):
    """write_plan.rs:126-139 with capacity 1024 (the reference's MAX_CONTEXT)."""
    N = pp._native

    def check(lens, heads, width, cap=1024):
        arr = (C.c_uint64 * max(1, len(lens)))(*lens)
        return N.lib.pp_b200_check_write_offsets(arr, len(lens), heads, width, cap)

    assert check([1, 7, 1023], 2, 3) == 0
    assert check([], 1, 1) == 1
    assert check([0], 0, 1) == 1
    assert check([0], 1, 0) == 1
    assert check([1024], 1, 1) == 1
    assert check([0, 1], 2**32 - 1, 2) == 0  # representable in 64-bit, unlike usize::MAX in the reference
    assert "maximum context" in (check([5000], 1, 64), N.last_error())[1]


def test_write_plan_key_mismatch_rejected(pp):
    """write_plan.rs:133-138: a plan is reusable only for the same offsets/shape."""
    import torch

    plan = pp.kv_cache.BatchWritePlan([1, 3], 2, 3, 1024, torch.device("cpu"))
    plan.validate([1, 3], 2, 3, torch.device("cpu"))
    for offs in ([3, 1], [1, 4], [1]):
        with pytest.raises(pp.PreconditionError):
            plan.validate(offs, 2, 3, torch.device("cpu"))
    with pytest.raises(pp.PreconditionError):
        plan.validate([1, 3], 1, 3, torch.device("cpu"))
    with pytest.raises(pp.PreconditionError):
        plan.validate([1, 3], 2, 4, torch.device("cpu"))
    with pytest.raises(pp.PreconditionError):
        pp.kv_cache.BatchWritePlan([1024], 1, 1, 1024, torch.device("cpu"))


def test_partition_is_deterministic_and_balanced(pp):
    import numpy as np

    g = np.random.Generator(np.random.PCG64(1))
    costs = [int(x) for x in g.integers(256, 8193, 64)]
    for shards in (1, 2, 4, 8):
        a, load = pp.kv_cache.partition_branches(costs, shards)
        b, _ = pp.kv_cache.partition_branches(costs, shards)
        assert a == b and sorted(set(a)) == list(range(shards))
        assert sum(load) == sum(costs)
        for s in range(shards):
            assert load[s] == sum(c for c, sh in zip(costs, a) if sh == s)
        # LPT bound: max load <= mean + max single cost
        assert max(load) <= sum(costs) / shards + max(costs)


def test_partition_equal_branches_split_evenly(pp):
    a, load = pp.kv_cache.partition_branches([2048] * 128, 8)
    assert load == [16 * 2048] * 8 and all(a.count(s) == 16 for s in range(8))


def test_partition_rejects_empty(pp):
    with pytest.raises(pp.PreconditionError):
        pp.kv_cache.partition_branches([], 2)
    with pytest.raises(pp.PreconditionError):
        pp.kv_cache.partition_branches([1], 0)


def test_attention_geometry_rejected_before_any_device_work(pp):
    """Invalid geometry returns PRECONDITION without touching a device (the
    container has none), as the reference validates before launching."""
    N = pp._native
    a = N.PpKvArena()
    a.struct_size = C.sizeof(N.PpKvArena)
    a.rows, a.heads, a.head_dim, a.capacity = 4, 3, 64, 16  # rows % heads != 0
    a.k = a.v = a.k_scale = a.v_scale = 256
    p = N.PpAttnParams()
    p.struct_size = C.sizeof(N.PpAttnParams)
    ws = C.c_void_p(4096)
    st = N.lib.pp_b200_decode_attention(C.byref(a), C.byref(p), C.c_void_p(256), None, None, C.c_void_p(256),
                                        C.c_void_p(256), ws, 1 << 20, None, None)
    assert st == N.STATUS_PRECONDITION and "geometry" in N.last_error()
    a.heads, a.head_dim = 2, 96
    st = N.lib.pp_b200_decode_attention(C.byref(a), C.byref(p), C.c_void_p(256), None, None, C.c_void_p(256),
                                        C.c_void_p(256), ws, 1 << 20, None, None)
    assert st == N.STATUS_PRECONDITION and "64|128" in N.last_error()
    a.head_dim = 64
    a.k = 8  # misaligned codes
    st = N.lib.pp_b200_decode_attention(C.byref(a), C.byref(p), C.c_void_p(256), None, None, C.c_void_p(256),
                                        C.c_void_p(256), ws, 1 << 20, None, None)
    assert st == N.STATUS_PRECONDITION and "16-byte" in N.last_error()
    a.k = 256
    st = N.lib.pp_b200_decode_attention(C.byref(a), C.byref(p), C.c_void_p(256), C.c_void_p(256), None,
                                        C.c_void_p(256), C.c_void_p(256), ws, 1 << 20, None, None)
    assert st == N.STATUS_PRECONDITION and "scratch" in N.last_error()
    a.rows, a.capacity = 1 << 20, 1 << 12  # rows*capacity beyond TMA coordinates
    st = N.lib.pp_b200_decode_attention(C.byref(a), C.byref(p), C.c_void_p(256), None, None, C.c_void_p(256),
                                        C.c_void_p(256), ws, 1 << 20, None, None)
    assert st == N.STATUS_PRECONDITION and "overflow" in N.last_error()


def test_quantize_geometry_rejected(pp):
    N = pp._native
    assert N.lib.pp_b200_quantize(C.c_void_p(256), 0, 0, 64, C.c_void_p(256), C.c_void_p(256), None, None) == 1
    assert N.lib.pp_b200_quantize(C.c_void_p(256), 0, 4, 32, C.c_void_p(256), C.c_void_p(256), None, None) == 1
    assert N.lib.pp_b200_quantize(C.c_void_p(256), 7, 4, 64, C.c_void_p(256), C.c_void_p(256), None, None) == 1


def test_workspace_size_is_an_upper_bound(pp):
    N = pp._native
    a = N.PpKvArena()
    a.struct_size = C.sizeof(N.PpKvArena)
    a.rows, a.heads, a.head_dim, a.capacity = 512, 16, 128, 4096
    p = N.PpAttnParams()
    p.struct_size = C.sizeof(N.PpAttnParams)
    p.max_ctas = 148
    auto = N.lib.pp_b200_attention_workspace_size(C.byref(a), C.byref(p))
    # stream-K: rows + ctas partials of (d + 4) floats, plus tables
    assert auto >= (512 + 148) * (128 + 4) * 4
    p.split_tokens = 128
    fixed = N.lib.pp_b200_attention_workspace_size(C.byref(a), C.byref(p))
    assert fixed >= 512 * 32 * (128 + 4) * 4


def test_status_messages_are_classifiable(pp):
    N = pp._native
    assert "EXECUTION_UNCERTAIN" in N.status_message(N.DEV_WAIT_TIMEOUT)
    assert N.status_message(N.DEV_NONFINITE_INPUT) == "non-finite INT8 KV input"
    assert N.status_message(0) == "ok"
