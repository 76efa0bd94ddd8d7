"""Runs the reference's own CUDA kernels (compiled from its sources into
oracle/_ref/ by oracle/Makefile) on device tensors, with the launch geometry
of the reference's CustomOps (app/src/model/int8_kv_ops.rs:120-161).

TEST INFRASTRUCTURE ONLY: used to pin the oracle (tests/golden/make_golden.py)
and by GPU parity tests that compare against the reference kernels directly.
Nothing here reads the reference tree at run time; it needs only the cubins.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
INT8_CUBIN = os.path.join(HERE, "_ref", "int8_kv_ref.cubin")


def available() -> bool:
    return os.path.exists(INT8_CUBIN)


class _Driver:
    def __init__(self):
        self.cu = C.CDLL("libcuda.so.1")
        self.cu.cuModuleLoadData.argtypes = [C.POINTER(C.c_void_p), C.c_void_p]
        self.cu.cuModuleGetFunction.argtypes = [C.POINTER(C.c_void_p), C.c_void_p, C.c_char_p]
        self.cu.cuLaunchKernel.argtypes = [C.c_void_p, C.c_uint, C.c_uint, C.c_uint, C.c_uint, C.c_uint, C.c_uint,
                                           C.c_uint, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]
        self.cu.cuFuncSetAttribute.argtypes = [C.c_void_p, C.c_int, C.c_int]

    def check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what} failed: CUresult {rc}")


class RefInt8Kernels:
    """pp_i8_scale / pp_i8_pack / pp_i8_unpack / pp_i8_attention / pp_i8_merge."""

    def __init__(self, cubin: str = INT8_CUBIN):
        torch.cuda.init()
        torch.empty(1, device="cuda")  # make the primary context current
        self.d = _Driver()
        with open(cubin, "rb") as f:
            self._image = f.read()
        self._buf = C.create_string_buffer(self._image, len(self._image))
        self.mod = C.c_void_p()
        self.d.check(self.d.cu.cuModuleLoadData(C.byref(self.mod), C.cast(self._buf, C.c_void_p)), "cuModuleLoadData")
        self.fn = {}
        for name in ("pp_i8_scale", "pp_i8_pack", "pp_i8_unpack", "pp_i8_attention", "pp_i8_merge"):
            f = C.c_void_p()
            self.d.check(self.d.cu.cuModuleGetFunction(C.byref(f), self.mod, name.encode()), name)
            self.fn[name] = f

    def _launch(self, name, grid, block, smem, args):
        holders = []
        for a in args:
            if isinstance(a, torch.Tensor):
                holders.append(C.c_void_p(a.data_ptr()))
            else:
                holders.append(a)
        params = (C.c_void_p * len(holders))(*[C.cast(C.pointer(h), C.c_void_p) for h in holders])
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        if smem > 48 * 1024:
            self.d.check(self.d.cu.cuFuncSetAttribute(self.fn[name], 8, smem), "cuFuncSetAttribute")
        self.d.check(self.d.cu.cuLaunchKernel(self.fn[name], grid[0], grid[1], 1, block, 1, 1, smem, stream, params,
                                              None), name)

    def quantize(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """x f32 [..., 64] contiguous -> (u8 codes, f32 scales [...])."""
        assert x.dtype == torch.float32 and x.is_contiguous() and x.shape[-1] == 64
        rows = x.numel() // 64
        scale = torch.empty(rows, dtype=torch.float32, device=x.device)
        packed = torch.empty(x.numel(), dtype=torch.uint8, device=x.device)
        self._launch("pp_i8_scale", (rows, 1), 64, 0, [x, scale, C.c_uint64(rows)])
        n = x.numel()
        self._launch("pp_i8_pack", ((n + 255) // 256, 1), 256, 0, [x, scale, packed, C.c_uint64(n)])
        return packed.reshape(x.shape), scale.reshape(x.shape[:-1])

    def dequantize(self, packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
        n = packed.numel()
        out = torch.empty(n, dtype=torch.float32, device=packed.device)
        self._launch("pp_i8_unpack", ((n + 255) // 256, 1), 256, 0, [packed, scale, out, C.c_uint64(n)])
        return out.reshape(packed.shape)

    def attention(self, q, k, v, ks, vs, sk, sv, past, heads: int, split_tokens: int) -> torch.Tensor:
        """Reference-mode attention exactly as cuda::Attention launches it."""
        rows, cap, d = k.shape
        assert d == 64 and cap <= 1024
        split = 128 if split_tokens == 0 else max(32, min(1024, split_tokens))
        splits = (cap + 1 + split - 1) // split
        partial = torch.empty(rows * splits * 66, dtype=torch.float32, device=q.device)
        out = torch.empty(rows * 64, dtype=torch.float32, device=q.device)
        self._launch("pp_i8_attention", (rows, splits), 128, (split + 128) * 4,
                     [q, k, v, ks, vs, sk, sv, past, partial, C.c_uint32(heads), C.c_uint32(cap), C.c_uint32(split),
                      C.c_uint32(splits)])
        self._launch("pp_i8_merge", (rows, 1), 64, 0, [partial, out, C.c_uint32(splits)])
        return out.reshape(rows, 1, 64)


GRAPH_CUBIN = os.path.join(HERE, "_ref", "graph_ops_ref.cubin")


class RefGraphKernels(RefInt8Kernels):
    """pp_graph_qkv / pp_graph_swiglu with the launch geometry of
    graph_ops.rs:355-395 (QKV: one 32-thread block per (row, head);
    element kernels: 1024-thread blocks over the elements)."""

    def __init__(self, cubin: str = GRAPH_CUBIN):
        torch.cuda.init()
        torch.empty(1, device="cuda")
        self.d = _Driver()
        with open(cubin, "rb") as f:
            self._image = f.read()
        self._buf = C.create_string_buffer(self._image, len(self._image))
        self.mod = C.c_void_p()
        self.d.check(self.d.cu.cuModuleLoadData(C.byref(self.mod), C.cast(self._buf, C.c_void_p)), "cuModuleLoadData")
        self.fn = {}
        for name in ("pp_graph_qkv", "pp_graph_swiglu"):
            f = C.c_void_p()
            self.d.check(self.d.cu.cuModuleGetFunction(C.byref(f), self.mod, name.encode()), name)
            self.fn[name] = f

    def qkv(self, qkv: torch.Tensor, params: torch.Tensor, positions: torch.Tensor, heads: int, dim: int,
            max_context: int) -> torch.Tensor:
        rows = qkv.shape[0]
        bf = qkv.dtype == torch.bfloat16
        out = torch.zeros(3 * rows * heads * dim, dtype=qkv.dtype, device=qkv.device)
        self._launch("pp_graph_qkv", (rows * heads, 1), 32, 0,
                     [qkv, params, positions, out, C.c_uint32(rows), C.c_uint32(heads), C.c_uint32(dim),
                      C.c_uint32(max_context), C.c_uint32(1 if bf else 0)])
        return out.reshape(3, rows * heads, dim)

    def swiglu(self, x: torch.Tensor) -> torch.Tensor:
        rows, cols = x.shape
        hidden = cols // 2
        bf = x.dtype == torch.bfloat16
        out = torch.empty(rows, hidden, dtype=x.dtype, device=x.device)
        n = rows * hidden
        self._launch("pp_graph_swiglu", ((n + 1023) // 1024, 1), 1024, 0,
                     [x, out, C.c_uint32(rows), C.c_uint32(hidden), C.c_uint32(1 if bf else 0)])
        return out


RENYI_CUBIN = os.path.join(HERE, "_ref", "renyi_ref.cubin")


class RefRenyiKernel(RefInt8Kernels):
    """pp_renyi_sample with the launch of fused_sampling.rs:147-162 (one
    256-thread block per logical row, padded * 8 + 256 * 16 shared bytes)."""

    def __init__(self, cubin: str = RENYI_CUBIN):
        torch.cuda.init()
        torch.empty(1, device="cuda")
        self.d = _Driver()
        with open(cubin, "rb") as f:
            self._image = f.read()
        self._buf = C.create_string_buffer(self._image, len(self._image))
        self.mod = C.c_void_p()
        self.d.check(self.d.cu.cuModuleLoadData(C.byref(self.mod), C.cast(self._buf, C.c_void_p)), "cuModuleLoadData")
        f = C.c_void_p()
        self.d.check(self.d.cu.cuModuleGetFunction(C.byref(f), self.mod, b"pp_renyi_sample"), "pp_renyi_sample")
        self.fn = {"pp_renyi_sample": f}

    def sample(self, raw: torch.Tensor, uniforms: torch.Tensor, bounds: torch.Tensor, guidance: int, alpha: float,
               cfg: float, offset: int) -> torch.Tensor:
        batch, choices = bounds.shape[0], raw.shape[1]
        padded = 1
        while padded < choices:
            padded <<= 1
        out = torch.zeros(3 * batch, dtype=torch.int32, device=raw.device)
        self._launch("pp_renyi_sample", (batch, 1), 256, padded * 8 + 256 * 16,
                     [raw, uniforms, bounds, out, C.c_uint32(batch), C.c_uint32(choices), C.c_uint32(guidance),
                      C.c_float(alpha), C.c_float(cfg), C.c_uint32(offset), C.c_uint32(padded)])
        return out.reshape(3, batch)


FLOAT_CUBIN = os.path.join(HERE, "_ref", "decode_attention_ref.cubin")


class RefFloatAttention(RefInt8Kernels):
    """pp_attention_f32 / pp_attention_bf16 / pp_attention_merge with the
    launch of fused_attention.rs:46-83: grid (rows, splits), 128 threads,
    (split + 128) * 4 shared bytes; partials [rows, splits, 66] and a 64-thread
    merge when there is more than one split."""

    def __init__(self, cubin: str = FLOAT_CUBIN):
        torch.cuda.init()
        torch.empty(1, device="cuda")
        self.d = _Driver()
        with open(cubin, "rb") as f:
            self._image = f.read()
        self._buf = C.create_string_buffer(self._image, len(self._image))
        self.mod = C.c_void_p()
        self.d.check(self.d.cu.cuModuleLoadData(C.byref(self.mod), C.cast(self._buf, C.c_void_p)), "cuModuleLoadData")
        self.fn = {}
        for name in ("pp_attention_f32", "pp_attention_bf16", "pp_attention_merge"):
            f = C.c_void_p()
            self.d.check(self.d.cu.cuModuleGetFunction(C.byref(f), self.mod, name.encode()), name)
            self.fn[name] = f

    def attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lengths: torch.Tensor | None,
                  heads: int, split_tokens: int, size: int | None = None) -> torch.Tensor:
        """q f32 [rows, qs]; k, v [rows, cap, 64] f32 or bf16 (the first `size`
        tokens are the tensor's key length); lengths int32/uint32 [rows/heads]."""
        rows, cap, d = k.shape
        size = cap if size is None else size
        split = size if split_tokens == 0 else min(max(split_tokens, 32), 1024)
        splits = (size + split - 1) // split
        out = torch.empty(rows * 64, dtype=torch.float32, device=q.device)
        part = torch.empty(rows * splits * 66, dtype=torch.float32, device=q.device) if splits > 1 else None
        name = "pp_attention_bf16" if k.dtype == torch.bfloat16 else "pp_attention_f32"
        self._launch(name, (rows, splits), 128, (split + 128) * 4,
                     [q, k, v, lengths if lengths is not None else C.c_uint64(0), part if part is not None else out,
                      C.c_uint32(heads), C.c_uint32(size), C.c_uint32(split), C.c_uint32(splits),
                      C.c_uint32(1 if lengths is not None else 0), C.c_uint64(q.stride(0)), C.c_uint64(cap * d),
                      C.c_uint64(cap * d)])
        if part is not None:
            self._launch("pp_attention_merge", (rows, 1), 64, 0, [part, out, C.c_uint32(splits)])
        return out.reshape(rows, 64)
