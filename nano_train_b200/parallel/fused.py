"""Dispatch of the fused compute+collective paths.

``all_gather_gemm`` and ``gemm_reduce_scatter`` run as single sm_100a
kernels over NVLink peer memory when the process group has a symmetric-memory
communicator registered (``register_communicator``); otherwise they run the
NCCL collective and the tcgen05 GEMM back to back (the baseline).
"""
from __future__ import annotations

import torch

from ..ops.linear import gemm
from . import comm

_COMMUNICATORS: dict = {}


def register_communicator(group, communicator) -> None:
    _COMMUNICATORS[id(group)] = communicator


def get_communicator(group):
    return _COMMUNICATORS.get(id(group))


def clear_communicators() -> None:
    for c in list(_COMMUNICATORS.values()):
        close = getattr(c, "close", None)
        if close is not None:
            close()
    _COMMUNICATORS.clear()


def all_gather_gemm(x_shard: torch.Tensor, weight: torch.Tensor, group, bias=None, *, b_mn: bool = False):
    """Returns (AG(x_shard) . op(W)^T (+ bias), AG(x_shard)); op(W) = W^T when b_mn (dgrad form)."""
    if comm.group_size(group) == 1:
        return gemm(x_shard, weight, bias=bias, b_mn=b_mn), x_shard
    c = get_communicator(group)
    if c is not None and c.supports(x_shard, weight):
        return c.all_gather_gemm(x_shard, weight, bias, b_mn=b_mn)
    x_full = comm.all_gather_dim0(x_shard, group)
    return gemm(x_full, weight, bias=bias, b_mn=b_mn), x_full


def gemm_reduce_scatter(x: torch.Tensor, weight: torch.Tensor, group, *, b_mn: bool = False):
    """Returns RS(x . op(W)^T) along dim 0, op(W) = W^T when b_mn (dgrad form)."""
    if comm.group_size(group) == 1:
        return gemm(x, weight, b_mn=b_mn)
    c = get_communicator(group)
    if c is not None and c.supports(x, weight):
        return c.gemm_reduce_scatter(x, weight, b_mn=b_mn)
    return comm.reduce_scatter_dim0(gemm(x, weight, b_mn=b_mn), group)
