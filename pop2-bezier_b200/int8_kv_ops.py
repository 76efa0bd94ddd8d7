"""Int8 historical-KV operations over the C ABI (device tensors only).

Mirrors the reference module app/src/model/int8_kv_ops.rs: the same function
names, argument meaning and error behaviour, with the CUDA branches served by
libpp_b200.so.  There is no CPU branch: a CPU tensor is rejected, as the
reference's `attention` rejects non-CUDA devices (int8_kv_ops.rs:54).

Differences, all documented at the call:
  * head_dim 128 is accepted besides 64 (the reference hard-codes 64);
  * capacity is not capped at 1024 (MAX_CONTEXT, app/src/model/mod.rs:55);
  * split_tokens == 0 selects the automatic balanced (stream-K) split
    instead of the fixed 128 the reference picks; results agree within f32
    reassociation for any split.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native as N

_F32, _BF16 = N.DTYPE_F32, N.DTYPE_BF16


def _dtype_code(t: torch.Tensor, what: str) -> int:
    if t.dtype == torch.float32:
        return _F32
    if t.dtype == torch.bfloat16:
        return _BF16
    raise N.PreconditionError(f"{what} must be F32 or BF16, got {t.dtype}")


def _stream(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _require_cuda(*ts: torch.Tensor) -> None:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise N.PreconditionError("KV INT8 fused attention is only supported by the CUDA native provider")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise N.PreconditionError("INT8 attention device mismatch")


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def geometry(t: torch.Tensor) -> tuple[int, int]:
    """[heads, tokens, head_dim] dense geometry check (int8_kv_ops.rs:5-10)."""
    if t.dim() != 3:
        raise N.PreconditionError("INT8 KV requires dense [heads,tokens,64|128]")
    h, n, d = t.shape
    if h == 0 or n == 0 or d not in (64, 128) or not t.is_contiguous():
        raise N.PreconditionError("INT8 KV requires dense [heads,tokens,64|128]")
    return h, n


def _new_status(device: torch.device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def read_status(status: torch.Tensor) -> int:
    """Reads a device status word (synchronises with its stream)."""
    return int(status.item()) & 0xFFFFFFFF


def quantize(input: torch.Tensor, *, check_finite: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """(packed u8 [h,n,d], scales f32 [h,n]) of an F32/BF16 [h,n,d] tensor.

    int8_kv_ops.rs:11-29.  With check_finite (the default) a non-finite input
    raises ValueError("non-finite INT8 KV input") like the reference's CPU
    branch; that check reads one device word back.
    """
    h, n = geometry(input)
    _require_cuda(input)
    d = input.shape[2]
    code = _dtype_code(input, "INT8 KV input")
    packed = torch.empty((h, n, d), dtype=torch.uint8, device=input.device)
    scales = torch.empty((h, n), dtype=torch.float32, device=input.device)
    status = _new_status(input.device)
    N.check(N.lib.pp_b200_quantize(_ptr(input), code, h * n, d, _ptr(packed), _ptr(scales), _ptr(status),
                                   _stream(input)))
    if check_finite and read_status(status) & N.DEV_NONFINITE_INPUT:
        raise ValueError("non-finite INT8 KV input")
    return packed, scales


def dequantize(packed: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype, *, round_bf16: bool | None = None
               ) -> torch.Tensor:
    """(i8) packed * scale as `dtype` (int8_kv_ops.rs:30-40).

    round_bf16 defaults to dtype == bfloat16, i.e. the reference's
    `.to_dtype(BF16)`; pass True with float32 to get bf16-rounded values in f32.
    """
    h, n = geometry(packed)
    if packed.dtype != torch.uint8 or scale.dtype != torch.float32 or tuple(scale.shape) != (h, n) \
            or not scale.is_contiguous():
        raise N.PreconditionError("INT8 KV scales differ")
    _require_cuda(packed, scale)
    if dtype not in (torch.float32, torch.bfloat16):
        raise N.PreconditionError(f"unsupported dequantize dtype {dtype}")
    d = packed.shape[2]
    rb = (dtype == torch.bfloat16) if round_bf16 is None else round_bf16
    out = torch.empty((h, n, d), dtype=dtype, device=packed.device)
    N.check(N.lib.pp_b200_dequantize(_ptr(packed), _ptr(scale), h * n, d, int(rb),
                                     _F32 if dtype == torch.float32 else _BF16, _ptr(out), _stream(packed)))
    return out


def arena_struct(k: torch.Tensor, v: torch.Tensor, ks: torch.Tensor, vs: torch.Tensor, heads: int) -> N.PpKvArena:
    rows, cap, d = k.shape
    a = N.PpKvArena()
    a.struct_size = C.sizeof(N.PpKvArena)
    a.rows, a.heads, a.head_dim, a.capacity = rows, heads, d, cap
    a.k, a.v, a.k_scale, a.v_scale = k.data_ptr(), v.data_ptr(), ks.data_ptr(), vs.data_ptr()
    return a


def attn_params(*, split_tokens: int = 0, q_dtype: torch.dtype = torch.float32,
                out_dtype: torch.dtype = torch.float32, softmax_scale: float = 0.0, plan_ready: bool = False,
                max_ctas: int = 0, prefetch_history: bool = False) -> N.PpAttnParams:
    p = N.PpAttnParams()
    p.struct_size = C.sizeof(N.PpAttnParams)
    p.split_tokens = split_tokens
    p.q_dtype = _F32 if q_dtype == torch.float32 else _BF16
    p.out_dtype = _F32 if out_dtype == torch.float32 else _BF16
    p.softmax_scale = softmax_scale
    p.flags = (N.ATTN_PLAN_READY if plan_ready else 0) | (N.ATTN_PREFETCH_HISTORY if prefetch_history else 0)
    p.max_ctas = max_ctas
    return p


def workspace_bytes(arena: N.PpKvArena, params: N.PpAttnParams) -> int:
    return int(N.lib.pp_b200_attention_workspace_size(C.byref(arena), C.byref(params)))


def new_workspace(arena: N.PpKvArena, params: N.PpAttnParams, device: torch.device) -> torch.Tensor:
    return torch.empty(workspace_bytes(arena, params), dtype=torch.uint8, device=device)


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ks: torch.Tensor, vs: torch.Tensor,
                     lengths: torch.Tensor, heads: int, *, scratch_k: torch.Tensor | None = None,
                     scratch_v: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                     split_tokens: int = 0, softmax_scale: float = 0.0, workspace: torch.Tensor | None = None,
                     plan_ready: bool = False, status: torch.Tensor | None = None,
                     out: torch.Tensor | None = None, prefetch_history: bool = False,
                     max_ctas: int = 0) -> torch.Tensor:
    """General entry: int8 decode attention over a [rows, capacity, d] arena.

    q [rows, d] (or [rows, 1, d]) F32/BF16; lengths int32/uint32 [rows/heads].
    With scratch_k/scratch_v (f32 [rows, d]) the reference mode applies: a row
    attends to lengths[b] history tokens plus the scratch token.  Without them
    a row attends to lengths[b] int8 tokens.  Returns [rows, d].
    """
    _require_cuda(q, k, v, ks, vs, lengths, scratch_k, scratch_v)
    rows, cap, d = k.shape
    if k.dtype != torch.uint8 or v.dtype != torch.uint8 or v.shape != k.shape:
        raise N.PreconditionError("INT8 attention geometry differs")
    if ks.dtype != torch.float32 or vs.dtype != torch.float32 or tuple(ks.shape) != (rows, cap) \
            or tuple(vs.shape) != (rows, cap):
        raise N.PreconditionError(f"INT8 scales must be F32[head_rows,capacity]")
    for t in (k, v, ks, vs, q, lengths):
        if not t.is_contiguous():
            raise N.PreconditionError("INT8 attention operands must be contiguous")
    if q.numel() != rows * d:
        raise N.PreconditionError(f"INT8 scratch must be F32[head_rows,1,{d}]")
    if heads <= 0 or rows % heads != 0 or lengths.numel() != rows // heads \
            or lengths.dtype not in (torch.int32, torch.uint32):
        raise N.PreconditionError("INT8 attention lengths differ")
    for t in (scratch_k, scratch_v):
        if t is not None and (t.dtype != torch.float32 or t.numel() != rows * d or not t.is_contiguous()):
            raise N.PreconditionError(f"INT8 scratch must be F32[head_rows,1,{d}]")
    odt = out_dtype or q.dtype
    arena = arena_struct(k, v, ks, vs, heads)
    params = attn_params(split_tokens=split_tokens, q_dtype=q.dtype, out_dtype=odt, softmax_scale=softmax_scale,
                         plan_ready=plan_ready, prefetch_history=prefetch_history, max_ctas=max_ctas)
    if workspace is None:
        workspace = new_workspace(arena, params, q.device)
    if out is None:
        out = torch.empty((rows, d), dtype=odt, device=q.device)
    N.check(N.lib.pp_b200_decode_attention(C.byref(arena), C.byref(params), _ptr(q), _ptr(scratch_k),
                                           _ptr(scratch_v), _ptr(lengths), _ptr(out), _ptr(workspace),
                                           workspace.numel(), _ptr(status), _stream(q)))
    return out


def plan_ragged(k: torch.Tensor, v: torch.Tensor, ks: torch.Tensor, vs: torch.Tensor, lengths: torch.Tensor,
                heads: int, workspace: torch.Tensor, *, split_tokens: int = 0, scratch: bool = False,
                max_ctas: int = 0) -> None:
    """Writes the attention plan for `lengths` into `workspace`, so that the
    decode_attention calls of a step that share these lengths (one per layer)
    can pass plan_ready=True with the same workspace and skip re-planning
    (the reuse DecodeMetadataCache does, decode_metadata.rs:39-142).
    `scratch` marks reference-mode calls (a scratch token after the history);
    split_tokens and max_ctas must be those of the calls that reuse the plan."""
    _require_cuda(k, lengths, workspace)
    arena = arena_struct(k, v, ks, vs, heads)
    params = attn_params(split_tokens=split_tokens, max_ctas=max_ctas)
    N.check(N.lib.pp_b200_plan_ragged(C.byref(arena), C.byref(params), _ptr(lengths), 1 if scratch else 0,
                                      _ptr(workspace), workspace.numel(), _stream(lengths)))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ks: torch.Tensor, vs: torch.Tensor,
              sk: torch.Tensor, sv: torch.Tensor, past: torch.Tensor, heads: int, split_tokens: int) -> torch.Tensor:
    """int8_kv_ops::attention (int8_kv_ops.rs:42-55): reference-mode fused attention.

    q, sk, sv f32 [rows,1,d]; k, v u8 [rows,capacity,d]; ks, vs f32
    [rows,capacity]; past u32/i32 [rows/heads].  Returns f32 [rows,1,d].
    A non-zero split_tokens is clamped to [32, 1024] as the reference does.
    """
    rows, cap, d = geometry(k) + (k.shape[2],)
    if heads <= 0 or rows % heads != 0 or v.shape != k.shape or k.dtype != torch.uint8 or v.dtype != torch.uint8:
        raise N.PreconditionError("INT8 attention geometry differs")
    for t in (q, sk, sv):
        if tuple(t.shape) != (rows, 1, d) or t.dtype != torch.float32 or not t.is_contiguous():
            raise N.PreconditionError(f"INT8 scratch must be F32[head_rows,1,{d}]")
    for t in (ks, vs):
        if tuple(t.shape) != (rows, cap) or t.dtype != torch.float32 or not t.is_contiguous():
            raise N.PreconditionError(f"INT8 scales must be F32[head_rows,capacity]")
    if tuple(past.shape) != (rows // heads,) or past.dtype not in (torch.int32, torch.uint32) \
            or not past.is_contiguous():
        raise N.PreconditionError("INT8 attention lengths differ")
    split = 0 if split_tokens == 0 else max(32, min(1024, split_tokens))
    out = decode_attention(q.reshape(rows, d), k, v, ks, vs, past, heads, scratch_k=sk.reshape(rows, d),
                           scratch_v=sv.reshape(rows, d), out_dtype=torch.float32, split_tokens=split)
    return out.reshape(rows, 1, d)


def prepare(device: torch.device | int) -> None:
    """On-device self-check (int8_kv_ops.rs:57-103); raises on failure."""
    idx = device if isinstance(device, int) else (device.index if device.index is not None else 0)
    if isinstance(device, torch.device) and device.type != "cuda":
        raise N.PreconditionError("KV INT8 needs CUDA in the native provider")
    N.check(N.lib.pp_b200_prepare(idx))
