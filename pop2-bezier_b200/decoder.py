"""Decoder step around the int8 KV path, on the C ABI.

Operations (ctypes over libpp_b200.so, torch tensors for memory):
  qkv_rope          graph_ops::qkv (app/src/model/graph_ops.rs:144-174)
  qkv_rope_append   the same fused with the int8 quantize-and-append of K/V
                    and the f32 scratch of reference-mode attention
                    (app/src/model/batch.rs:143-155, int8_cache.rs:326-359)
  swiglu            graph_ops::swiglu (graph_ops.rs:175-193)
  rmsnorm           candle_nn::ops::rms_norm with an optional residual add
  rope_parameters   the [q_norm | k_norm | cos | sin] block of the reference's
                    qk_rope_parameters, with PrimitiveModel's RoPE tables
                    (mod.rs:322-330)

SyntheticDecoder runs the batched decode step of PrimitiveModel
(batch.rs:120-170, mod.rs:669-746) with random weights: per layer RMSNorm ->
QKV projection -> q/k RMSNorm + RoPE + int8 append -> int8 decode attention
(history + the current token as f32 scratch) -> output projection + residual
-> RMSNorm -> gate/up projection -> SwiGLU -> down projection + residual, then
the final RMSNorm.  The projections are cuBLAS GEMMs (torch.matmul), as the
reference's are (`x.matmul(&w.t())`, batch.rs:134,155-170); everything else
is this library's kernels.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from . import int8_kv_ops as ops
from . import kv_cache


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return N.DTYPE_BF16
    if t.dtype == torch.float32:
        return N.DTYPE_F32
    raise N.PreconditionError(f"static graph requires BF16 or F32 model tensors, got {t.dtype}")


def _geometry(qkv: torch.Tensor, heads: int, head_dim: int, max_context: int) -> N.PpQkvRope:
    if qkv.dim() != 2 or qkv.shape[1] != 3 * heads * head_dim or not qkv.is_contiguous():
        raise N.PreconditionError("graph QKV/RoPE geometry differs")
    g = N.PpQkvRope()
    g.struct_size = C.sizeof(N.PpQkvRope)
    g.rows = qkv.shape[0]
    g.heads = heads
    g.head_dim = head_dim
    g.max_context = max_context
    g.dtype = _dtype_code(qkv)
    return g


def _check_params(params: torch.Tensor, qkv: torch.Tensor, head_dim: int, max_context: int) -> None:
    if params.dtype != qkv.dtype or params.numel() != 2 * head_dim + max_context * head_dim \
            or not params.is_contiguous():
        raise N.PreconditionError("graph QKV/RoPE geometry differs: parameter block")


def _positions(p: torch.Tensor, rows: int, what: str) -> None:
    if p.numel() != rows or p.dtype not in (torch.int32, torch.uint32) or not p.is_contiguous():
        raise N.PreconditionError(f"{what} must be contiguous U32 [rows]")


def rope_parameters(q_norm: torch.Tensor, k_norm: torch.Tensor, max_context: int) -> torch.Tensor:
    """[q_norm | k_norm | cos | sin] in the norms' dtype and device; the tables
    are PrimitiveModel's: inv = 1 / 10000^(2p/d), angle = pos * inv in f32."""
    d = q_norm.numel()
    pair = np.arange(d // 2, dtype=np.float32)
    inv = (np.float32(1.0) / np.power(np.float32(10000.0), (pair * np.float32(2.0)) / np.float32(d))).astype(np.float32)
    ang = (np.arange(max_context, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(q_norm.device, q_norm.dtype)
    sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(q_norm.device, q_norm.dtype)
    return torch.cat([q_norm.reshape(-1), k_norm.reshape(-1), cos.reshape(-1), sin.reshape(-1)]).contiguous()


def qkv_rope(qkv: torch.Tensor, params: torch.Tensor, positions: torch.Tensor, heads: int, head_dim: int,
             max_context: int, *, out: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """Planes [3, rows*heads, head_dim] (rotated q, rotated k, v) of a QKV
    projection output [rows, 3*heads*head_dim]."""
    ops._require_cuda(qkv, params, positions)
    g = _geometry(qkv, heads, head_dim, max_context)
    _check_params(params, qkv, head_dim, max_context)
    _positions(positions, g.rows, "graph positions")
    if out is None:
        out = torch.empty((3, g.rows * heads, head_dim), dtype=qkv.dtype, device=qkv.device)
    N.check(N.lib.pp_b200_qkv_rope(C.byref(g), ops._ptr(qkv), ops._ptr(params), ops._ptr(positions), ops._ptr(out),
                                   ops._ptr(status), ops._stream(qkv)))
    return out


def qkv_rope_append(qkv: torch.Tensor, params: torch.Tensor, positions: torch.Tensor, arena: kv_cache.Int8KvArena,
                    offsets: torch.Tensor, max_context: int, *, commit: bool = True,
                    q_out: torch.Tensor | None = None, scratch_k: torch.Tensor | None = None,
                    scratch_v: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """Rotated q [rows*heads, d] (model dtype) and the f32 scratch k, v of the
    current token; its int8 K/V are appended to `arena` at offsets[row]."""
    ops._require_cuda(qkv, params, positions, offsets, arena.k)
    heads, d = arena.heads, arena.head_dim
    g = _geometry(qkv, heads, d, max_context)
    _check_params(params, qkv, d, max_context)
    _positions(positions, g.rows, "graph positions")
    _positions(offsets, g.rows, "append offsets")
    n = g.rows * heads
    if q_out is None:
        q_out = torch.empty((n, d), dtype=qkv.dtype, device=qkv.device)
    if scratch_k is None:
        scratch_k = torch.empty((n, d), dtype=torch.float32, device=qkv.device)
    if scratch_v is None:
        scratch_v = torch.empty((n, d), dtype=torch.float32, device=qkv.device)
    a = arena.struct()
    N.check(N.lib.pp_b200_qkv_rope_append(C.byref(g), ops._ptr(qkv), ops._ptr(params), ops._ptr(positions),
                                          C.byref(a), ops._ptr(offsets), int(commit), ops._ptr(q_out),
                                          ops._ptr(scratch_k), ops._ptr(scratch_v), ops._ptr(status),
                                          ops._stream(qkv)))
    return q_out, scratch_k, scratch_v


def swiglu(x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up of x = [rows, 2*hidden] (gate | up)."""
    ops._require_cuda(x)
    if x.dim() != 2 or x.shape[1] % 2 or not x.is_contiguous():
        raise N.PreconditionError("graph FFN width must be even")
    rows, hidden = x.shape[0], x.shape[1] // 2
    if out is None:
        out = torch.empty((rows, hidden), dtype=x.dtype, device=x.device)
    N.check(N.lib.pp_b200_swiglu(ops._ptr(x), ops._ptr(out), rows, hidden, _dtype_code(x), ops._stream(x)))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *, residual: torch.Tensor | None = None,
            x_sum: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the last dim of a 2-D x; with `residual`, x + residual is
    normalised and (if given) stored to x_sum, which may be x itself."""
    ops._require_cuda(x, weight, residual, x_sum)
    if x.dim() != 2 or not x.is_contiguous() or weight.numel() != x.shape[1] or weight.dtype != x.dtype:
        raise N.PreconditionError("rms_norm geometry differs")
    for t in (residual, x_sum):
        if t is not None and (t.shape != x.shape or t.dtype != x.dtype or not t.is_contiguous()):
            raise N.PreconditionError("rms_norm residual geometry differs")
    if out is None:
        out = torch.empty_like(x)
    N.check(N.lib.pp_b200_rmsnorm(ops._ptr(x), ops._ptr(residual), ops._ptr(x_sum), ops._ptr(weight), ops._ptr(out),
                                  x.shape[0], x.shape[1], float(eps), _dtype_code(x), ops._stream(x)))
    return out


@dataclass
class DecoderConfig:
    """BASELINE config 3 by default: 24 layers, width 2048, 16 heads x 128,
    SwiGLU hidden 5632, RoPE base 10000, int8 KV."""
    layers: int = 24
    width: int = 2048
    heads: int = 16
    head_dim: int = 128
    ffn_hidden: int = 5632
    max_context: int = 4096

    def parameters(self) -> int:
        w, f = self.width, self.ffn_hidden
        per = 3 * w * w + w * w + 2 * f * w + f * w + 2 * w + 2 * self.head_dim
        return self.layers * per + w


class SyntheticDecoder:
    """Random-init bf16 decoder with per-layer int8 KV arenas for `branches`
    independent branches of up to `capacity` tokens."""

    def __init__(self, cfg: DecoderConfig, branches: int, capacity: int, device, seed: int = 0,
                 dtype: torch.dtype = torch.bfloat16, split_tokens: int = 0):
        self.cfg, self.branches, self.capacity = cfg, branches, capacity
        self.prefetch = True  # see PP_ATTN_PREFETCH_HISTORY
        # 0: stream-K plan balanced over the SMs; > 0: fixed splits of that many tokens, which make every
        # branch's result independent of the other branches in the batch
        self.split_tokens = split_tokens
        self.device = torch.device(device)
        self.dtype = dtype
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        w, f, h, d = cfg.width, cfg.ffn_hidden, cfg.heads, cfg.head_dim

        def lin(out_f: int, in_f: int) -> torch.Tensor:
            return (torch.randn(out_f, in_f, device=self.device, generator=g) / math.sqrt(in_f)).to(dtype)

        def norm(n: int) -> torch.Tensor:
            return (1.0 + 0.1 * torch.randn(n, device=self.device, generator=g)).to(dtype)

        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append(dict(
                norm1=norm(w), qkv=lin(3 * w, w), rope=rope_parameters(norm(d), norm(d), cfg.max_context),
                proj=lin(w, w), norm2=norm(w), gate_up=lin(2 * f, w), down=lin(w, f)))
        self.final_norm = norm(w)
        self.arenas = [kv_cache.Int8KvArena.zeros(branches, h, d, capacity, self.device) for _ in range(cfg.layers)]
        a0 = self.arenas[0].struct()
        self._params = ops.attn_params(q_dtype=dtype, out_dtype=dtype, split_tokens=split_tokens)
        self.workspace = ops.new_workspace(a0, self._params, self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        rows = branches * h
        self._buf = dict(
            x=torch.empty(branches, w, dtype=dtype, device=self.device),
            normed=torch.empty(branches, w, dtype=dtype, device=self.device),
            q=torch.empty(rows, d, dtype=dtype, device=self.device),
            sk=torch.empty(rows, d, dtype=torch.float32, device=self.device),
            sv=torch.empty(rows, d, dtype=torch.float32, device=self.device),
            att=torch.empty(rows, d, dtype=dtype, device=self.device),
            act=torch.empty(branches, f, dtype=dtype, device=self.device),
            out=torch.empty(branches, w, dtype=dtype, device=self.device),
        )

    def fill_history(self, lengths: torch.Tensor, seed: int = 1) -> None:
        """Random int8 history (codes and scales) for every layer, as if
        `lengths[b]` tokens had been decoded already."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for a in self.arenas:
            a.k.random_(0, 256, generator=g)
            a.v.random_(0, 256, generator=g)
            a.k_scale.uniform_(0.005, 0.05, generator=g)
            a.v_scale.uniform_(0.005, 0.05, generator=g)

    def weight_bytes(self) -> int:
        n = sum(t.numel() * t.element_size() for L in self.layers for t in L.values())
        return n + self.final_norm.numel() * self.final_norm.element_size()

    def capture(self, past: torch.Tensor, advance: bool = True) -> "CapturedStep":
        """Records one step into a CUDA graph (all launches of the step, cuBLAS
        included) so that a decode loop costs one graph launch per token.  The
        graph reads its input from `CapturedStep.x` and the per-branch history
        length from `past` (a device tensor that stays in place); with
        `advance`, the graph also adds 1 to `past` after the step, so each
        replay decodes the next position.  Call once the step has run eagerly
        (library and cuBLAS set-up happen on first use)."""
        return CapturedStep(self, past, advance)

    def _linear(self, x: torch.Tensor, li: int, name: str) -> torch.Tensor:
        return torch.matmul(x, self.layers[li][name].t())

    def step(self, x: torch.Tensor, past: torch.Tensor, positions: torch.Tensor | None = None, *,
             commit: bool = True, lengths: torch.Tensor | None = None, probe=None) -> torch.Tensor:
        """One decode token for every branch.  x [branches, width] (the input
        embedding), past u32/i32 [branches] (tokens already in each branch's
        cache; the new K/V go to slot past[b]); returns the final-normed
        hidden state [branches, width].  x is consumed (used as the residual).
        commit=False is the reference's partial query (int8_cache.rs:305-310):
        slot past[b] receives the placeholder (zero codes, scale 1) and the
        attention still sees the current token through the f32 scratch.
        lengths (default: past) is the history each branch's attention reads;
        0 makes a branch attend to its current token only, with no history
        traffic (a retired lane riding along in the batch).
        probe(layer, q, scratch_k, scratch_v, arena, attention_out), when
        given, is called after each layer's attention is enqueued (eager
        steps only; it may synchronise and read the tensors)."""
        cfg, b = self.cfg, self._buf
        H, d = cfg.heads, cfg.head_dim
        pos = past if positions is None else positions
        hist = past if lengths is None else lengths
        a0 = self.arenas[0]
        # one plan per step for every layer's attention (reference mode: history + scratch token)
        ops.plan_ragged(a0.k, a0.v, a0.k_scale, a0.v_scale, hist, H, self.workspace, scratch=True,
                        split_tokens=self.split_tokens)
        xr = x
        residual = None
        for li, (L, arena) in enumerate(zip(self.layers, self.arenas)):
            rmsnorm(xr, L["norm1"], residual=residual, x_sum=xr if residual is not None else None, out=b["normed"])
            qkv = self._linear(b["normed"], li, "qkv")
            qkv_rope_append(qkv, L["rope"], pos, arena, past, cfg.max_context, commit=commit, q_out=b["q"],
                            scratch_k=b["sk"], scratch_v=b["sv"], status=self.status)
            # qkv_rope_append writes slot past[b], after the history: the attention may stream
            # the history while it finishes
            ops.decode_attention(b["q"], arena.k, arena.v, arena.k_scale, arena.v_scale, hist, H,
                                 scratch_k=b["sk"], scratch_v=b["sv"], out_dtype=self.dtype,
                                 split_tokens=self.split_tokens, workspace=self.workspace, plan_ready=True,
                                 status=self.status, out=b["att"], prefetch_history=self.prefetch)
            if probe is not None:
                probe(li, b["q"], b["sk"], b["sv"], arena, b["att"])
            proj = self._linear(b["att"].view(self.branches, H * d), li, "proj")
            rmsnorm(xr, L["norm2"], residual=proj, x_sum=xr, out=b["normed"])
            gate_up = self._linear(b["normed"], li, "gate_up")
            swiglu(gate_up, out=b["act"])
            residual = self._linear(b["act"], li, "down")
        return rmsnorm(xr, self.final_norm, residual=residual, x_sum=xr, out=b["out"])


class CapturedStep:
    """A SyntheticDecoder step recorded in a CUDA graph (see capture())."""

    def __init__(self, model: SyntheticDecoder, past: torch.Tensor, advance: bool):
        self.model, self.past = model, past
        self.x = torch.zeros(model.branches, model.cfg.width, dtype=model.dtype, device=model.device)
        side = torch.cuda.Stream(device=model.device)
        side.wait_stream(torch.cuda.current_stream(model.device))
        with torch.cuda.stream(side):  # warm the capture stream (cuBLAS handles, workspaces)
            keep = past.clone()
            model.step(self.x.clone(), past)
            past.copy_(keep)
        torch.cuda.current_stream(model.device).wait_stream(side)
        torch.cuda.synchronize(model.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = model.step(self.x, past)
            if advance:
                past.add_(1)

    def replay(self, x: torch.Tensor | None = None) -> torch.Tensor:
        """Runs the step on x (copied into the graph's input first when given);
        returns the graph's output buffer (overwritten by the next replay)."""
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.out
