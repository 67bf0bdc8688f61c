"""Tensor-parallel linear math with Megatron sequence parallelism.

Column-parallel (SP):  x_shard [T/tp, K] --all-gather--> [T, K] . W_shard^T -> [T, N/tp]
Row-parallel (SP):     x [T, K/tp] . W_shard^T -> partial [T, N] --reduce-scatter--> [T/tp, N]

Each pair (all-gather -> GEMM, GEMM -> reduce-scatter) is one fused
compute+collective kernel over NVLink peer memory when a symmetric-memory
communicator is attached to the group (``nano_train_b200.parallel.fused``),
otherwise NCCL + the tcgen05 GEMM (the baseline path, also the CPU/gloo
path). Backward mirrors it: column dgrad is GEMM -> reduce-scatter, row
backward all-gathers dY then runs dgrad/wgrad.

Reference parity: src/layers.py:1235-1496 (Column/RowParallelLinear with
all-reduce, no SP form around linears) - this module adds the SP form the
Llama TP=8 configuration needs.
"""
from __future__ import annotations

import torch

from ..ops.linear import accumulate_weight_grad
from . import comm
from . import fused


def _flat(x):
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.is_contiguous() else x2.contiguous()


class ColumnParallelSPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, group):
        x2 = _flat(x)
        y, x_full = fused.all_gather_gemm(x2, weight, group, bias=bias)
        ctx.save_for_backward(x_full, weight)
        ctx.group = group
        ctx.has_bias = bias is not None
        ctx.lead = x.shape[:-1]
        return y

    @staticmethod
    def backward(ctx, gy):
        x_full, weight = ctx.saved_tensors
        g2 = _flat(gy)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = fused.gemm_reduce_scatter(g2, weight, ctx.group, b_mn=True)
            dx = dx.view(*ctx.lead, -1)
        dw = accumulate_weight_grad(weight, g2, x_full) if ctx.needs_input_grad[1] else None
        db = g2.float().sum(0).to(gy.dtype) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
        return dx, dw, db, None


class RowParallelSPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, group):
        x2 = _flat(x)
        y = fused.gemm_reduce_scatter(x2, weight, group)
        if bias is not None:
            y = y + bias
        ctx.save_for_backward(x2, weight)
        ctx.group = group
        ctx.has_bias = bias is not None
        ctx.in_shape = x.shape
        return y

    @staticmethod
    def backward(ctx, gy):
        x2, weight = ctx.saved_tensors
        g_shard = _flat(gy)
        if ctx.needs_input_grad[0]:
            dx, g_full = fused.all_gather_gemm(g_shard, weight, ctx.group, b_mn=True)
            dx = dx.view(ctx.in_shape)
        else:
            dx, g_full = None, comm.all_gather_dim0(g_shard, ctx.group)
        dw = accumulate_weight_grad(weight, g_full, x2) if ctx.needs_input_grad[1] else None
        db = g_shard.float().sum(0).to(gy.dtype) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
        return dx, dw, db, None


def column_parallel_linear_sp(x, weight, bias, group):
    """x: [T_local, K] sequence shard -> [T, N_local]."""
    return ColumnParallelSPFn.apply(x, weight, bias, group)


def row_parallel_linear_sp(x, weight, bias, group):
    """x: [T, K_local] -> [T_local, N] sequence shard (bias added once, after the reduction)."""
    return RowParallelSPFn.apply(x, weight, bias, group)
