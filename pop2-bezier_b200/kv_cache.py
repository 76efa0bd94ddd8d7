"""Caller-owned int8 KV arenas and the ragged per-branch bookkeeping around them.

Layout (the reference's shared batch arena, app/src/model/cache.rs:301-478 and
int8_cache.rs:326-359): per layer, u8 codes [rows, capacity, d] for K and for V
and f32 scales [rows, capacity] for each; row = branch * heads + head.  The
arena never moves rows: a branch's history lives in rows [b*heads, (b+1)*heads).

Device memory is allocated by torch (the caller side of the C ABI); the
library only reads and writes it.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _native as N
from . import int8_kv_ops as ops


def checked_batch_rows(logical_rows: int, guidance: int) -> int:
    """Physical rows for `logical_rows` branches with CFG `guidance` in {1,2}
    (app/src/model/batch_geometry.rs:4-16)."""
    out = C.c_uint64(0)
    if logical_rows < 0 or logical_rows >= 2**64 or guidance < 0 or guidance >= 2**32:
        raise N.PreconditionError("parallel row count must be non-zero and CFG branches 1 or 2")
    N.check(N.lib.pp_b200_checked_batch_rows(logical_rows, guidance, C.byref(out)))
    return int(out.value)


class BatchWritePlan:
    """Validated per-branch write offsets, shared by every layer of one step.

    Mirrors BatchWritePlan (app/src/model/write_plan.rs:48-93): built once from
    the host-side past lengths, validated before any device write, reused
    across layers and the partial queries of one primitive.  The reference
    expands offsets to a U32[B*H,1,D] scatter index; the append kernel reads one
    u32 per branch instead.
    """

    def __init__(self, past_lens: list[int], heads: int, width: int, capacity: int, device: torch.device):
        self._check(past_lens, heads, width, capacity)
        self.offsets = tuple(int(x) for x in past_lens)
        self.heads, self.width, self.capacity = heads, width, capacity
        self.device = torch.device(device)
        self.indices = torch.tensor(self.offsets, dtype=torch.int32, device=self.device)

    @staticmethod
    def _check(past_lens, heads, width, capacity):
        arr = (C.c_uint64 * max(1, len(past_lens)))(*[int(x) for x in past_lens])
        N.check(N.lib.pp_b200_check_write_offsets(arr, len(past_lens), heads, width, capacity))

    def validate(self, past_lens: list[int], heads: int, width: int, device: torch.device) -> None:
        """write_plan.rs:71-93: geometry and key must match; never reads the device."""
        self._check(past_lens, heads, width, self.capacity)
        if tuple(int(x) for x in past_lens) != self.offsets or heads != self.heads or width != self.width:
            raise N.PreconditionError("write plan key does not match the current row offsets and head shape")
        if torch.device(device) != self.device:
            raise N.PreconditionError("write plan device differs from the current KV device")
        if self.indices.dtype != torch.int32 or self.indices.numel() != len(self.offsets) \
                or not self.indices.is_contiguous():
            raise N.PreconditionError("write plan indices must be contiguous U32 [B]")


@dataclass
class Int8KvArena:
    """One layer's int8 K/V arena for `rows = branches * heads` head rows."""

    k: torch.Tensor
    v: torch.Tensor
    k_scale: torch.Tensor
    v_scale: torch.Tensor
    heads: int

    @classmethod
    def zeros(cls, branches: int, heads: int, head_dim: int, capacity: int, device) -> "Int8KvArena":
        rows = checked_batch_rows(branches, 1) * heads
        dev = torch.device(device)
        return cls(k=torch.zeros((rows, capacity, head_dim), dtype=torch.uint8, device=dev),
                   v=torch.zeros((rows, capacity, head_dim), dtype=torch.uint8, device=dev),
                   k_scale=torch.zeros((rows, capacity), dtype=torch.float32, device=dev),
                   v_scale=torch.zeros((rows, capacity), dtype=torch.float32, device=dev),
                   heads=heads)

    @property
    def rows(self) -> int:
        return self.k.shape[0]

    @property
    def capacity(self) -> int:
        return self.k.shape[1]

    @property
    def head_dim(self) -> int:
        return self.k.shape[2]

    @property
    def branches(self) -> int:
        return self.rows // self.heads

    def struct(self) -> N.PpKvArena:
        return ops.arena_struct(self.k, self.v, self.k_scale, self.v_scale, self.heads)

    def reserved_bytes(self) -> int:
        """Codes plus scales: 2*d + 8 bytes per token and head (136 at d=64,
        app/src/model/int8_cache.rs:47-50)."""
        return sum(t.numel() * t.element_size() for t in (self.k, self.v, self.k_scale, self.v_scale))

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, offsets: torch.Tensor, *, commit: bool = True,
               status: torch.Tensor | None = None) -> None:
        """Quantize-and-append one token per row at offsets[branch]
        (int8_cache.rs:293-359 + cache.rs:415-459).  k_new, v_new: F32/BF16
        [rows, d] (any shape with rows*d elements, e.g. [B,H,1,d])."""
        ops._require_cuda(k_new, v_new, offsets, self.k)
        n = self.rows * self.head_dim
        if k_new.numel() != n or v_new.numel() != n or k_new.dtype != v_new.dtype \
                or not k_new.is_contiguous() or not v_new.is_contiguous():
            raise N.PreconditionError("INT8 batch requires [B,H,1,D] scratch and matching row histories")
        if offsets.numel() != self.branches or offsets.dtype not in (torch.int32, torch.uint32) \
                or not offsets.is_contiguous():
            raise N.PreconditionError("batch KV rows and cache/length counts differ")
        code = ops._dtype_code(k_new, "K/V input")
        a = self.struct()
        N.check(N.lib.pp_b200_quant_append(C.byref(a), ops._ptr(k_new), ops._ptr(v_new), code, ops._ptr(offsets),
                                           int(commit), ops._ptr(status), ops._stream(k_new)))

    def attention(self, q: torch.Tensor, lengths: torch.Tensor, **kw) -> torch.Tensor:
        """History-mode decode attention over this arena (see int8_kv_ops.decode_attention)."""
        return ops.decode_attention(q, self.k, self.v, self.k_scale, self.v_scale, lengths, self.heads, **kw)

    def grown(self, capacity: int, lengths: torch.Tensor) -> "Int8KvArena":
        """A new arena of larger capacity holding each row's committed prefix
        (the growth copy of LayerCache::query, cache.rs:246-266)."""
        if capacity < self.capacity:
            raise N.PreconditionError("KV metadata truncation cannot extend committed history")
        dst = Int8KvArena.zeros(self.branches, self.heads, self.head_dim, capacity, self.k.device)
        a, b = self.struct(), dst.struct()
        N.check(N.lib.pp_b200_copy_prefix(C.byref(a), C.byref(b), ops._ptr(lengths), ops._stream(self.k)))
        return dst


def partition_branches(costs: list[int], shards: int) -> tuple[list[int], list[int]]:
    """Longest-processing-time assignment of independent branches to shards
    (GPUs).  Returns (shard_of_branch, shard_cost)."""
    n = len(costs)
    arr = (C.c_uint64 * max(1, n))(*[int(c) for c in costs])
    out = (C.c_uint32 * max(1, n))()
    cost = (C.c_uint64 * max(1, shards))()
    N.check(N.lib.pp_b200_sched_partition(arr, n, shards, out, cost))
    return [int(out[i]) for i in range(n)], [int(cost[s]) for s in range(shards)]


class BranchShards:
    """The branches one rank owns, and the gather of their outputs to rank 0.

    Branches are independent (app/src/inference/batch.rs:241-558 runs each
    branch's decode on its own cache), so a step needs no collective: each rank
    decodes its shard of the LPT partition above, and only the final outputs
    travel, once, to rank 0.  Shards may hold different numbers of branches;
    the gather pads every shard to the largest and rank 0 puts the rows back
    in global branch order.
    """

    def __init__(self, costs: list[int], world: int, rank: int):
        if not 0 <= rank < world:
            raise N.PreconditionError(f"rank {rank} outside world of {world}")
        self.world, self.rank = world, rank
        self.shard_of, self.shard_cost = partition_branches(costs, world)
        self.members = [[b for b, s in enumerate(self.shard_of) if s == r] for r in range(world)]
        self.mine = self.members[rank]
        self.widest = max(len(m) for m in self.members)

    def gather(self, dist, out: torch.Tensor, group=None) -> torch.Tensor | None:
        """`out` is this rank's output, leading dim = len(self.mine) branches.
        Every rank must call this (it is one collective, over `group`, the
        default group when None); rank 0 gets the outputs of all branches in
        global order, the other ranks get None."""
        if out.shape[0] != len(self.mine):
            raise N.PreconditionError(f"gather: {out.shape[0]} branch outputs for a shard of {len(self.mine)}")
        padded = out.new_zeros((self.widest, *out.shape[1:]))
        padded[: len(self.mine)] = out
        parts = [torch.empty_like(padded) for _ in range(self.world)] if self.rank == 0 else None
        dist.gather(padded, parts, dst=0, group=group)
        if self.rank != 0:
            return None
        full = out.new_empty((len(self.shard_of), *out.shape[1:]))
        for r, branches in enumerate(self.members):
            if branches:
                full[torch.tensor(branches, device=out.device)] = parts[r][: len(branches)]
        return full
