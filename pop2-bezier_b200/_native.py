"""ctypes binding of libpp_b200.so (the C ABI declared in include/pp_b200.h).

The library is loaded from this package directory.  There is no fallback:
if the library is missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpp_b200.so")

STATUS_OK = 0
STATUS_PRECONDITION = 1
STATUS_INVALID_OUTPUT = 2
STATUS_UNCERTAIN = 3

DTYPE_F32 = 0
DTYPE_BF16 = 1

DEV_NONFINITE_INPUT = 0x1
DEV_OFFSET_RANGE = 0x2
DEV_LENGTH_RANGE = 0x4
DEV_WAIT_TIMEOUT = 0x8
DEV_POSITION_RANGE = 0x10

ATTN_PLAN_READY = 0x1
ATTN_PREFETCH_HISTORY = 0x2

# Every symbol include/pp_b200.h declares; the CPU test suite checks the
# library exports exactly these.
EXPORTED = (
    "pp_b200_abi_version",
    "pp_b200_last_error",
    "pp_b200_quantize",
    "pp_b200_dequantize",
    "pp_b200_quant_append",
    "pp_b200_copy_prefix",
    "pp_b200_attention_workspace_size",
    "pp_b200_plan_ragged",
    "pp_b200_decode_attention",
    "pp_b200_decode_attention_static",
    "pp_b200_status_message",
    "pp_b200_diag_bounded_wait",
    "pp_b200_checked_batch_rows",
    "pp_b200_check_write_offsets",
    "pp_b200_sched_partition",
    "pp_b200_sched_lane_seed",
    "pp_b200_sched_uniform",
    "pp_b200_sched_uniforms",
    "pp_b200_qkv_rope",
    "pp_b200_qkv_rope_append",
    "pp_b200_swiglu",
    "pp_b200_rmsnorm",
    "pp_b200_renyi_sample",
    "pp_b200_float_attention_workspace_size",
    "pp_b200_plan_ragged_float",
    "pp_b200_decode_attention_float",
    "pp_b200_prepare",
    "pp_b200_prepare_optional",
)


class PpKvArena(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("rows", C.c_uint32),
        ("heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("capacity", C.c_uint32),
        ("reserved", C.c_uint32),
        ("k", C.c_void_p),
        ("v", C.c_void_p),
        ("k_scale", C.c_void_p),
        ("v_scale", C.c_void_p),
    ]


class PpAttnParams(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("split_tokens", C.c_uint32),
        ("q_dtype", C.c_int32),
        ("out_dtype", C.c_int32),
        ("softmax_scale", C.c_float),
        ("flags", C.c_uint32),
        ("max_ctas", C.c_uint32),
        ("reserved", C.c_uint32),
    ]


class PpFloatKv(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("rows", C.c_uint32),
        ("heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("tokens", C.c_uint32),
        ("dtype", C.c_int32),
        ("k_row_stride", C.c_uint64),
        ("v_row_stride", C.c_uint64),
        ("k", C.c_void_p),
        ("v", C.c_void_p),
    ]


class PpQkvRope(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("rows", C.c_uint32),
        ("heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("max_context", C.c_uint32),
        ("dtype", C.c_int32),
        ("reserved", C.c_uint32 * 2),
    ]


class PreconditionError(ValueError):
    """Status 1: invalid geometry or argument; nothing was launched."""


class InvalidOutputError(RuntimeError):
    """Status 2: a device check found invalid data."""


class ExecutionUncertainError(RuntimeError):
    """Status 3: CUDA failure; device state is uncertain, discard the KV state."""


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python pop2-bezier_b200/build_native.py` "
            "(there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    vp, u32, i32, u64, sz = C.c_void_p, C.c_uint32, C.c_int32, C.c_uint64, C.c_size_t
    P = C.POINTER
    sig = {
        "pp_b200_abi_version": (u32, []),
        "pp_b200_last_error": (C.c_char_p, []),
        "pp_b200_quantize": (i32, [vp, i32, u64, u32, vp, vp, vp, vp]),
        "pp_b200_dequantize": (i32, [vp, vp, u64, u32, i32, i32, vp, vp]),
        "pp_b200_quant_append": (i32, [P(PpKvArena), vp, vp, i32, vp, u32, vp, vp]),
        "pp_b200_copy_prefix": (i32, [P(PpKvArena), P(PpKvArena), vp, vp]),
        "pp_b200_attention_workspace_size": (sz, [P(PpKvArena), P(PpAttnParams)]),
        "pp_b200_plan_ragged": (i32, [P(PpKvArena), P(PpAttnParams), vp, u32, vp, sz, vp]),
        "pp_b200_decode_attention": (i32, [P(PpKvArena), P(PpAttnParams), vp, vp, vp, vp, vp, vp, sz, vp, vp]),
        "pp_b200_decode_attention_static": (i32, [P(PpKvArena), P(PpAttnParams), vp, vp, vp, vp, vp, vp, vp]),
        "pp_b200_status_message": (C.c_char_p, [u32]),
        "pp_b200_diag_bounded_wait": (i32, [vp, u32, vp]),
        "pp_b200_checked_batch_rows": (i32, [u64, u32, P(u64)]),
        "pp_b200_check_write_offsets": (i32, [P(u64), u64, u32, u32, u32]),
        "pp_b200_sched_partition": (i32, [P(u64), u32, u32, P(u32), P(u64)]),
        "pp_b200_sched_lane_seed": (u64, [u64, u64]),
        "pp_b200_sched_uniform": (C.c_float, [u64, u64]),
        "pp_b200_sched_uniforms": (i32, [vp, vp, vp, u32, vp, vp]),
        "pp_b200_qkv_rope": (i32, [P(PpQkvRope), vp, vp, vp, vp, vp, vp]),
        "pp_b200_qkv_rope_append": (i32, [P(PpQkvRope), vp, vp, vp, P(PpKvArena), vp, u32, vp, vp, vp, vp, vp]),
        "pp_b200_swiglu": (i32, [vp, vp, u64, u32, i32, vp]),
        "pp_b200_rmsnorm": (i32, [vp, vp, vp, vp, vp, u64, u32, C.c_float, i32, vp]),
        "pp_b200_renyi_sample": (i32, [vp, vp, vp, vp, u32, u32, u32, C.c_float, C.c_float, u32, vp]),
        "pp_b200_float_attention_workspace_size": (sz, [P(PpFloatKv), P(PpAttnParams)]),
        "pp_b200_plan_ragged_float": (i32, [P(PpFloatKv), P(PpAttnParams), vp, vp, sz, vp]),
        "pp_b200_decode_attention_float": (i32, [P(PpFloatKv), P(PpAttnParams), vp, u64, vp, vp, vp, sz, vp, vp]),
        "pp_b200_prepare": (i32, [i32]),
        "pp_b200_prepare_optional": (i32, [i32, u32, u32, i32, u32, u32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    msg = lib.pp_b200_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(status: int) -> None:
    """Raises the exception class matching a non-OK status."""
    if status == STATUS_OK:
        return
    msg = last_error()
    if status == STATUS_PRECONDITION:
        raise PreconditionError(msg)
    if status == STATUS_INVALID_OUTPUT:
        raise InvalidOutputError(msg)
    raise ExecutionUncertainError(msg or f"status {status}")


def status_message(bits: int) -> str:
    return lib.pp_b200_status_message(bits).decode()


def abi_version() -> int:
    return int(lib.pp_b200_abi_version())
