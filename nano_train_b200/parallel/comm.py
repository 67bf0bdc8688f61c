"""Autograd-aware collectives for tensor and sequence parallelism.

Every function degrades to the identity for a group of size 1. The NCCL
calls here are the plumbing baseline; the fused compute+collective kernels
(``nano_train_b200.parallel.fused``) replace the AG->GEMM and GEMM->RS pairs
on GPUs that share NVLink.

Reference parity: src/layers.py:1195-1233 (_ReduceFromTensorParallelRegion,
_CopyToTensorParallelRegion) and 1499-1597 (sequence scatter / gather).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


def group_size(group) -> int:
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def min_fused_ranks() -> int:
    """Smallest group on which the peer-memory kernels (fused EP dispatch / combine, fused ZeRO
    step) replace NCCL: 2, or 1 with NTB_FUSED_ONE_RANK=1. In a one-rank group every "peer"
    pointer is this GPU's own memory, so the kernels run their whole protocol (slabs, epochs,
    bounded waits, canaries) on one GPU; tests use it to check them where only one GPU is present."""
    return 1 if os.environ.get("NTB_FUSED_ONE_RANK", "0") == "1" else 2


def group_rank(group) -> int:
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 0
    return dist.get_rank(group)


def all_gather_dim0(x: torch.Tensor, group) -> torch.Tensor:
    n = group_size(group)
    if n == 1:
        return x
    x = x.contiguous()
    out = torch.empty((n * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)
    return out


def reduce_scatter_dim0(x: torch.Tensor, group) -> torch.Tensor:
    n = group_size(group)
    if n == 1:
        return x
    x = x.contiguous()
    assert x.shape[0] % n == 0, "reduce_scatter_dim0: leading dim must divide the group"
    out = torch.empty((x.shape[0] // n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x, group=group)
    return out


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        if group_size(ctx.group) > 1:
            g = g.contiguous()
            dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        if group_size(group) > 1:
            x = x.contiguous().clone()
            dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherSeq(torch.autograd.Function):
    """Forward all-gather along ``dim``; backward reduce-scatter (Megatron SP)."""

    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        if group_size(group) == 1:
            return x
        xt = x.movedim(dim, 0)
        out = all_gather_dim0(xt, group)
        return out.movedim(0, dim).contiguous()

    @staticmethod
    def backward(ctx, g):
        if group_size(ctx.group) == 1:
            return g, None, None
        gt = g.movedim(ctx.dim, 0)
        out = reduce_scatter_dim0(gt, ctx.group)
        return out.movedim(0, ctx.dim).contiguous(), None, None


class _ReduceScatterSeq(torch.autograd.Function):
    """Forward reduce-scatter along ``dim``; backward all-gather (Megatron SP)."""

    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        if group_size(group) == 1:
            return x
        out = reduce_scatter_dim0(x.movedim(dim, 0), group)
        return out.movedim(0, dim).contiguous()

    @staticmethod
    def backward(ctx, g):
        if group_size(ctx.group) == 1:
            return g, None, None
        out = all_gather_dim0(g.movedim(ctx.dim, 0), ctx.group)
        return out.movedim(0, ctx.dim).contiguous(), None, None


class _ScatterSeq(torch.autograd.Function):
    """Forward keep own chunk along ``dim``; backward all-gather (reference semantics)."""

    @staticmethod
    def forward(ctx, x, rank, size, group, dim):
        ctx.group, ctx.dim, ctx.size = group, dim, size
        if size == 1:
            return x
        n = x.size(dim)
        if n % size != 0:
            raise ValueError("sequence length must be divisible by tp_size for sequence scatter")
        chunk = n // size
        return x.narrow(dim, rank * chunk, chunk).contiguous()

    @staticmethod
    def backward(ctx, g):
        if ctx.size == 1:
            return g, None, None, None, None
        out = all_gather_dim0(g.movedim(ctx.dim, 0), ctx.group)
        return out.movedim(0, ctx.dim).contiguous(), None, None, None, None


class _GatherSeqNarrowBwd(torch.autograd.Function):
    """Forward all-gather along ``dim``; backward keep own chunk (reference semantics)."""

    @staticmethod
    def forward(ctx, x, rank, size, group, dim):
        ctx.rank, ctx.size, ctx.dim = rank, size, dim
        if size == 1:
            return x
        out = all_gather_dim0(x.movedim(dim, 0), group)
        return out.movedim(0, dim).contiguous()

    @staticmethod
    def backward(ctx, g):
        if ctx.size == 1:
            return g, None, None, None, None
        n = g.size(ctx.dim)
        if n % ctx.size != 0:
            raise ValueError("sequence length must be divisible by tp_size for sequence gather")
        chunk = n // ctx.size
        return g.narrow(ctx.dim, ctx.rank * chunk, chunk).contiguous(), None, None, None, None


def copy_to_tensor_parallel_region(x, group):
    return _CopyToTP.apply(x, group)


def reduce_from_tensor_parallel_region(x, group):
    return _ReduceFromTP.apply(x, group)


def gather_along_seq(x, group, dim=0):
    return _GatherSeq.apply(x, group, dim)


def reduce_scatter_along_seq(x, group, dim=0):
    return _ReduceScatterSeq.apply(x, group, dim)


def scatter_to_sequence_parallel_region(x, tp_rank, tp_size, tp_group=None, seq_dim=1):
    group = tp_group if tp_group is not None else (dist.group.WORLD if dist.is_initialized() else None)
    return _ScatterSeq.apply(x, tp_rank, tp_size, group, seq_dim)


def gather_from_sequence_parallel_region(x, tp_rank, tp_size, tp_group=None, seq_dim=1):
    group = tp_group if tp_group is not None else (dist.group.WORLD if dist.is_initialized() else None)
    return _GatherSeqNarrowBwd.apply(x, tp_rank, tp_size, group, seq_dim)
