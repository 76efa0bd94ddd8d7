"""Float-KV fused decode attention over the C ABI (device tensors only).

Mirrors fused_attention::decode_attention (app/src/model/fused_attention.rs:
8-33): q [rows, 1, d] (or [rows, d]), K/V [rows, length, d] in bf16 or f32
with dense channel and token strides (any row stride), optional per-branch
lengths, `heads` heads per branch and the reference's split_tokens.  Returns
f32 [rows, 1, d] like the reference.  The reference's errors are raised as
PreconditionError with its messages; there is no CPU branch (the reference
bails with "select ordinary attention for CPU").

Differences, all documented at the call:
  * head_dim 128 is accepted besides 64, and bf16 q besides f32;
  * the key length is not capped at 1024;
  * split_tokens == 0 selects the balanced stream-K plan instead of one CTA
    per row; a non-zero split_tokens is clamped to [32, 1024] as the
    reference does.  Results agree within f32 reassociation for any split.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native as N
from . import int8_kv_ops as ops

_MSG_SHAPE = "fused decode attention requires F32[batch*heads,1,64] and same-device BF16/F32 K/V"
_MSG_STRIDE = "fused attention requires dense width and token strides"
_MSG_LENGTHS = "fused attention row lengths require same-device U32[batch]"


def kv_struct(k: torch.Tensor, v: torch.Tensor, heads: int) -> N.PpFloatKv:
    rows, n, d = k.shape
    g = N.PpFloatKv()
    g.struct_size = C.sizeof(N.PpFloatKv)
    g.rows, g.heads, g.head_dim, g.tokens = rows, heads, d, n
    g.dtype = N.DTYPE_F32 if k.dtype == torch.float32 else N.DTYPE_BF16
    g.k_row_stride, g.v_row_stride = k.stride(0), v.stride(0)
    g.k, g.v = k.data_ptr(), v.data_ptr()
    return g


def _check(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lengths: torch.Tensor | None, heads: int) -> None:
    """The checks of fused_attention.rs:10-25 (head_dim 64 or 128)."""
    for t in (q, k, v, lengths):
        if t is not None and not t.is_cuda:
            raise N.PreconditionError("NVIDIA fused attention needs CUDA; use ordinary attention on this backend")
    if q.dim() == 2:
        q = q.unsqueeze(1)
    if q.dim() != 3 or k.dim() != 3:
        raise N.PreconditionError(_MSG_SHAPE)
    rows, query, width = q.shape
    key_rows, length, key_width = k.shape
    if heads <= 0 or rows == 0 or rows % heads != 0 or query != 1 or width not in (64, 128) or key_rows != rows \
            or key_width != width or length == 0 or tuple(v.shape) != tuple(k.shape) \
            or q.dtype not in (torch.float32, torch.bfloat16) or k.dtype not in (torch.float32, torch.bfloat16) \
            or k.dtype != v.dtype or q.device != k.device or q.device != v.device:
        raise N.PreconditionError(_MSG_SHAPE)
    for t in (k, v):
        if t.stride(2) != 1 or t.stride(1) != width:
            raise N.PreconditionError(_MSG_STRIDE)
    if q.stride(2) != 1:
        raise N.PreconditionError(_MSG_STRIDE)
    if lengths is not None:
        if lengths.dim() != 1 or lengths.numel() != rows // heads or lengths.dtype not in (torch.int32, torch.uint32) \
                or not lengths.is_contiguous() or lengths.device != q.device:
            raise N.PreconditionError(_MSG_LENGTHS)


def workspace_bytes(kv: N.PpFloatKv, params: N.PpAttnParams) -> int:
    return int(N.lib.pp_b200_float_attention_workspace_size(C.byref(kv), C.byref(params)))


def plan_ragged(k: torch.Tensor, v: torch.Tensor, lengths: torch.Tensor | None, heads: int, workspace: torch.Tensor,
                *, split_tokens: int = 0, q_dtype: torch.dtype = torch.float32) -> None:
    """Writes the split plan for these lengths into `workspace` (reused by
    calls with plan_ready=True, e.g. by every layer of one decode step)."""
    kv = kv_struct(k, v, heads)
    params = ops.attn_params(split_tokens=split_tokens, q_dtype=q_dtype)
    N.check(N.lib.pp_b200_plan_ragged_float(C.byref(kv), C.byref(params), ops._ptr(lengths), ops._ptr(workspace),
                                            workspace.numel(), ops._stream(k)))


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lengths: torch.Tensor | None, heads: int,
                     split_tokens: int = 0, *, out_dtype: torch.dtype = torch.float32, softmax_scale: float = 0.0,
                     workspace: torch.Tensor | None = None, plan_ready: bool = False,
                     prefetch_history: bool = False, status: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused float-KV decode attention; returns [rows, 1, d] (out_dtype, f32
    by default as the reference)."""
    _check(q, k, v, lengths, heads)
    rows, d = k.shape[0], k.shape[2]
    q_stride = q.stride(0)
    kv = kv_struct(k, v, heads)
    params = ops.attn_params(split_tokens=split_tokens, q_dtype=q.dtype, out_dtype=out_dtype,
                             softmax_scale=softmax_scale, plan_ready=plan_ready, prefetch_history=prefetch_history)
    if workspace is None:
        workspace = torch.empty(workspace_bytes(kv, params), dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty((rows, 1, d), dtype=out_dtype, device=q.device)
    N.check(N.lib.pp_b200_decode_attention_float(C.byref(kv), C.byref(params), ops._ptr(q), q_stride,
                                                 ops._ptr(lengths), ops._ptr(out), ops._ptr(workspace),
                                                 workspace.numel(), ops._ptr(status), ops._stream(q)))
    return out


def prepare_optional_kernels(device: torch.device | int, fusion: bool, split_k: bool, *,
                             dtype: torch.dtype = torch.bfloat16, head_width: int = 64, ffn_hidden: int = 0) -> None:
    """PrimitiveModel::prepare_optional_kernels (mod.rs:440-460): on-device
    zero-input checks of the fused attention (and SwiGLU with `fusion`);
    raises PreconditionError with the reference's messages."""
    idx = device.index if isinstance(device, torch.device) else int(device)
    code = N.DTYPE_F32 if dtype == torch.float32 else N.DTYPE_BF16
    N.check(N.lib.pp_b200_prepare_optional(0 if idx is None else idx, int(fusion), int(split_k), code, head_width,
                                           ffn_hidden))
