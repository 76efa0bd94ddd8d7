"""Device sampling after the output heads, on the C ABI.

renyi_sample mirrors fused_sampling::sample (app/src/inference/
fused_sampling.rs:69-90): Rényi-entropy truncated sampling with classifier-
free guidance, one logical row per block, bit-identical to the reference's
pp_renyi_sample.
"""
from __future__ import annotations

import torch

from . import _native as N
from . import int8_kv_ops as ops


def renyi_sample(raw: torch.Tensor, uniforms: torch.Tensor, bounds: torch.Tensor, alpha: float, cfg: float,
                 guidance: int, offset: int, *, out: torch.Tensor | None = None):
    """raw f32 [batch*guidance, choices]; uniforms f32 [batch, 1]; bounds u32
    (or i32) [batch, 2] = (start, count).  Returns (tokens, ok, support), each
    [batch, 1] u32 views of one [3, batch] buffer, like the reference."""
    ops._require_cuda(raw, uniforms, bounds)
    if raw.dim() != 2 or guidance not in (1, 2) or raw.shape[0] == 0 or raw.shape[0] % guidance \
            or not 1 <= raw.shape[1] <= 2048:
        raise N.PreconditionError(
            "fused sampler needs 1/2 guidance rows and a nonempty head of at most 2048 choices")
    batch = raw.shape[0] // guidance
    if uniforms.numel() != batch or bounds.numel() != 2 * batch:
        raise N.PreconditionError("fused sampler logical row, uniform or bounds shape mismatch")
    if raw.dtype != torch.float32 or uniforms.dtype != torch.float32 or bounds.dtype not in (torch.int32,
                                                                                             torch.uint32):
        raise N.PreconditionError("fused sampler expects FP32 logits/uniforms and U32 bounds")
    for t in (raw, uniforms, bounds):
        if not t.is_contiguous():
            raise N.PreconditionError("fused sampler inputs must be contiguous; nonzero view offsets are supported")
    if out is None:
        out = torch.empty((3, batch), dtype=torch.int32, device=raw.device)
    N.check(N.lib.pp_b200_renyi_sample(ops._ptr(raw), ops._ptr(uniforms), ops._ptr(bounds), ops._ptr(out), batch,
                                       raw.shape[1], guidance, float(alpha), float(cfg), int(offset),
                                       ops._stream(raw)))
    return out[0].view(batch, 1), out[1].view(batch, 1), out[2].view(batch, 1)
