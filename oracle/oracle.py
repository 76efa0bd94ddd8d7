"""ctypes binding of the CPU oracle (oracle/int8kv_oracle.c, graph_oracle.c, sample_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arm of bench.py.  The product never imports this.
Build the shared library with `make -C oracle`.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_int8kv.so")

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: run `make -C oracle`")
        L = C.CDLL(LIB_PATH)
        vp, u32, u64, i32, f32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float
        L.oracle_bf16_round.restype = f32
        L.oracle_bf16_round.argtypes = [f32]
        L.oracle_quantize_f32.restype = i32
        L.oracle_quantize_f32.argtypes = [vp, u64, u32, vp, vp]
        L.oracle_quantize_bf16.restype = i32
        L.oracle_quantize_bf16.argtypes = [vp, u64, u32, vp, vp]
        L.oracle_dequantize.restype = None
        L.oracle_dequantize.argtypes = [vp, vp, u64, u32, vp, i32]
        L.oracle_attention.restype = i32
        L.oracle_attention.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, f32, vp, i32]
        L.oracle_quant_append.restype = i32
        L.oracle_quant_append.argtypes = [vp, vp, u32, u32, u32, u32, vp, i32, vp, vp, vp, vp]
        L.oracle_max_threads.restype = i32
        L.oracle_max_threads.argtypes = []
        L.oracle_qkv_rope.restype = i32
        L.oracle_qkv_rope.argtypes = [vp, vp, vp, vp, u32, u32, u32, u32, i32]
        L.oracle_swiglu.restype = i32
        L.oracle_swiglu.argtypes = [vp, vp, u64, u32, i32]
        L.oracle_renyi_sample.restype = i32
        L.oracle_renyi_sample.argtypes = [vp, vp, vp, vp, u32, u32, u32, f32, f32, u32]
        L.oracle_float_attention.restype = i32
        L.oracle_float_attention.argtypes = [vp, u64, vp, u64, vp, u64, i32, vp, u32, u32, u32, u32, u32, f32, vp, i32]
        L.oracle_rmsnorm.restype = i32
        L.oracle_rmsnorm.argtypes = [vp, vp, vp, vp, vp, u64, u32, f32, i32]
        _lib = L
    return _lib


def _p(a: np.ndarray | None) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data if a is not None else 0)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """RNE f32 -> bf16 bits (half::bf16::from_f32 semantics for finite values)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


class NonFiniteInput(ValueError):
    pass


def quantize(x: np.ndarray, head_dim: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """int8_kv_ops.rs:13-21 on rows of head_dim.  x: f32, or uint16 bf16 bits."""
    d = head_dim or x.shape[-1]
    rows = x.size // d
    packed = np.empty(rows * d, dtype=np.uint8)
    scales = np.empty(rows, dtype=np.float32)
    if x.dtype == np.uint16:
        xs = np.ascontiguousarray(x)
        rc = lib().oracle_quantize_bf16(_p(xs), rows, d, _p(packed), _p(scales))
    else:
        xs = np.ascontiguousarray(x, dtype=np.float32)
        rc = lib().oracle_quantize_f32(_p(xs), rows, d, _p(packed), _p(scales))
    if rc == 1:
        raise NonFiniteInput("non-finite INT8 KV input")
    if rc:
        raise ValueError(f"oracle quantize failed ({rc})")
    return packed.reshape(x.shape[:-1] + (d,)), scales.reshape(x.shape[:-1])


def dequantize(packed: np.ndarray, scales: np.ndarray, round_bf16: bool) -> np.ndarray:
    d = packed.shape[-1]
    rows = packed.size // d
    out = np.empty(packed.size, dtype=np.float32)
    pk = np.ascontiguousarray(packed, dtype=np.uint8)
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    lib().oracle_dequantize(_p(pk), _p(sc), rows, d, _p(out), int(round_bf16))
    return out.reshape(packed.shape)


def attention(q, k, v, ks, vs, lengths, heads: int, *, sk=None, sv=None, scale: float | None = None,
              threads: int = 1) -> np.ndarray:
    """Batched int8 decode attention (reference arithmetic; see the C file).

    q f32 [rows, d]; k, v u8 [rows, cap, d]; ks, vs f32 [rows, cap];
    lengths u32 [rows/heads]; sk, sv f32 [rows, d] or None.  Returns f32 [rows, d].
    """
    rows, cap, d = k.shape
    if scale is None:
        scale = 0.125 if d == 64 else float(np.float32(1.0 / np.sqrt(d)))
    args = [np.ascontiguousarray(q, dtype=np.float32).reshape(rows, d),
            np.ascontiguousarray(k, dtype=np.uint8), np.ascontiguousarray(v, dtype=np.uint8),
            np.ascontiguousarray(ks, dtype=np.float32), np.ascontiguousarray(vs, dtype=np.float32)]
    skc = None if sk is None else np.ascontiguousarray(sk, dtype=np.float32).reshape(rows, d)
    svc = None if sv is None else np.ascontiguousarray(sv, dtype=np.float32).reshape(rows, d)
    lens = np.ascontiguousarray(lengths, dtype=np.uint32)
    out = np.empty((rows, d), dtype=np.float32)
    rc = lib().oracle_attention(_p(args[0]), _p(args[1]), _p(args[2]), _p(args[3]), _p(args[4]), _p(skc), _p(svc),
                                _p(lens), rows, heads, d, cap, scale, _p(out), threads)
    if rc:
        raise ValueError(f"oracle attention failed ({rc})")
    return out


def quant_append(xk, xv, heads: int, offsets, commit: bool, k_arena, v_arena, ks_arena, vs_arena) -> None:
    """In-place oracle append into numpy arenas [rows, cap, d] / [rows, cap]."""
    rows, cap, d = k_arena.shape
    xk = np.ascontiguousarray(xk, dtype=np.float32)
    xv = np.ascontiguousarray(xv, dtype=np.float32)
    offs = np.ascontiguousarray(offsets, dtype=np.uint32)
    rc = lib().oracle_quant_append(_p(xk), _p(xv), rows, heads, d, cap, _p(offs), int(commit), _p(k_arena),
                                   _p(v_arena), _p(ks_arena), _p(vs_arena))
    if rc == 1:
        raise NonFiniteInput("non-finite INT8 KV input")
    if rc:
        raise ValueError(f"oracle append failed ({rc})")


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# ---------------------------------------------------------------- decoder step
# Model-dtype arrays are passed as uint16 bf16 bits (bf=True) or float32.

def _model(a, bf: bool) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16 if bf else np.float32)


def qkv_rope(qkv, params, positions, rows: int, heads: int, dim: int, max_context: int, bf: bool) -> np.ndarray:
    """graph_ops.cu pp_graph_qkv restated: returns planes [3, rows*heads, dim]
    (rows whose position is outside the table stay zero)."""
    qkv, params = _model(qkv, bf), _model(params, bf)
    pos = np.ascontiguousarray(positions, dtype=np.uint32)
    out = np.zeros((3, rows * heads, dim), dtype=np.uint16 if bf else np.float32)
    if lib().oracle_qkv_rope(_p(qkv), _p(params), _p(pos), _p(out), rows, heads, dim, max_context, int(bf)):
        raise ValueError("oracle qkv_rope: unsupported head dim")
    return out


def swiglu(x, rows: int, hidden: int, bf: bool) -> np.ndarray:
    x = _model(x, bf)
    out = np.empty((rows, hidden), dtype=np.uint16 if bf else np.float32)
    lib().oracle_swiglu(_p(x), _p(out), rows, hidden, int(bf))
    return out


def rmsnorm(x, weight, rows: int, width: int, eps: float, bf: bool, residual=None):
    """Returns (out, x_sum); x_sum is None without a residual."""
    x, w = _model(x, bf), _model(weight, bf)
    r = None if residual is None else _model(residual, bf)
    dt = np.uint16 if bf else np.float32
    out = np.empty((rows, width), dtype=dt)
    xs = None if r is None else np.empty((rows, width), dtype=dt)
    lib().oracle_rmsnorm(_p(x), _p(r), _p(xs), _p(w), _p(out), rows, width, eps, int(bf))
    return out, xs


def renyi_sample(raw, uniforms, bounds, guidance: int, alpha: float, cfg: float, offset: int) -> np.ndarray:
    """The reference's fused Rényi sampler restated: raw f32 [batch*guidance,
    choices], uniforms f32 [batch], bounds u32 [batch, 2] -> u32 [3, batch]."""
    raw = np.ascontiguousarray(raw, dtype=np.float32)
    u = np.ascontiguousarray(uniforms, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(bounds, dtype=np.uint32).reshape(-1, 2)
    batch, choices = b.shape[0], raw.shape[1]
    out = np.zeros((3, batch), dtype=np.uint32)
    if lib().oracle_renyi_sample(_p(raw), _p(u), _p(b), _p(out), batch, choices, guidance, alpha, cfg, offset):
        raise ValueError("oracle renyi_sample: unsupported geometry")
    return out


def float_attention(q, k, v, lengths, heads: int, *, size: int | None = None, split_tokens: int = 0,
                    scale: float | None = None, threads: int = 1) -> np.ndarray:
    """Float-KV fused decode attention (float_attn_oracle.c).

    q f32 [rows, q_stride] (first d channels used); k, v [rows, cap, d] f32, or
    uint16 bf16 bits; only the first `size` tokens of a row exist (default
    cap); lengths u32 [rows/heads] or None.  Returns f32 [rows, d]."""
    rows, cap, d = k.shape
    size = cap if size is None else size
    if scale is None:
        scale = 0.125 if d == 64 else float(np.float32(1.0 / np.sqrt(d)))
    bf = k.dtype == np.uint16
    if (v.dtype == np.uint16) != bf:
        raise ValueError("K and V dtypes differ")
    qc = np.ascontiguousarray(q, dtype=np.float32)
    kc, vc = np.ascontiguousarray(k), np.ascontiguousarray(v)
    lens = None if lengths is None else np.ascontiguousarray(lengths, dtype=np.uint32)
    out = np.empty((rows, d), dtype=np.float32)
    rc = lib().oracle_float_attention(_p(qc), qc.shape[1], _p(kc), cap * d, _p(vc), cap * d, int(bf), _p(lens),
                                      rows, heads, d, size, split_tokens, scale, _p(out), threads)
    if rc:
        raise ValueError(f"oracle float attention failed ({rc})")
    return out
