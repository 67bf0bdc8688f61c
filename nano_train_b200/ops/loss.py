"""Fused cross-entropy (plain and vocab-parallel).

One row kernel computes max / sum-exp / target logit per row; the backward
kernel writes softmax - onehot scaled by the upstream gradient directly,
optionally in place over the logits buffer, so the [T, V] fp32 probabilities
are never materialised. For a vocab-sharded LM head the three per-row
statistics are all-reduced (MAX, SUM, SUM) over the tensor-parallel group.

Reference parity: src/losses.py:95-133 (log_softmax + NLL, ignore_index
-100, mean over valid rows), examples/train_4d.py:725-730.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ._ext import ext


class _CEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index, reduction, vstart, group, inplace_grad):
        lab = labels.reshape(-1).contiguous()
        lg = logits.reshape(-1, logits.shape[-1])
        mx, sm, tg = ext().ce_stats(lg, lab, vstart, ignore_index)
        if group is not None and dist.get_world_size(group) > 1:
            gmx = mx.clone()
            dist.all_reduce(gmx, op=dist.ReduceOp.MAX, group=group)
            sm = sm * torch.exp(mx - gmx)
            dist.all_reduce(sm, group=group)
            dist.all_reduce(tg, group=group)
            mx = gmx
        lse = mx + torch.log(sm)
        valid = lab != ignore_index
        loss_rows = torch.where(valid, lse - tg, torch.zeros_like(lse))
        if reduction == "mean":
            count = valid.sum().clamp_min(1).to(torch.float32)
            out = loss_rows.sum() / count
        elif reduction == "sum":
            count = None
            out = loss_rows.sum()
        else:
            count = None
            out = loss_rows.view(labels.shape)
        ctx.save_for_backward(lg, lab, lse, count if count is not None else lse.new_ones(()))
        ctx.meta = (ignore_index, reduction, vstart, logits.shape, inplace_grad)
        return out

    @staticmethod
    def backward(ctx, gout):
        lg, lab, lse, count = ctx.saved_tensors
        ignore_index, reduction, vstart, shape, inplace_grad = ctx.meta
        if reduction == "mean":
            scale = (gout.float() / count).reshape(1)
        elif reduction == "sum":
            scale = gout.float().reshape(1)
        else:
            scale = gout.float().reshape(-1).contiguous()
        grad = lg if inplace_grad else torch.empty_like(lg)
        ext().ce_bwd(lg, lab, lse, scale.contiguous(), vstart, ignore_index, grad)
        return grad.view(shape), None, None, None, None, None, None


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100, reduction: str = "mean",
                  *, vocab_start: int = 0, group=None, inplace_grad: bool = False) -> torch.Tensor:
    """Cross-entropy over the last dim of ``logits``.

    With ``group`` set, ``logits`` hold columns [vocab_start, vocab_start + V_local)
    of a vocab sharded across that group. ``inplace_grad=True`` lets the
    backward overwrite the logits buffer with the gradient (saves one [T, V]).
    """
    if logits.is_cuda and logits.dtype in (torch.bfloat16, torch.float32):
        return _CEFn.apply(logits, labels, ignore_index, reduction, vocab_start, group, inplace_grad)
    if group is not None and dist.get_world_size(group) > 1:
        return _vocab_parallel_ce_reference(logits, labels, ignore_index, reduction, vocab_start, group)
    lg, lab = logits.reshape(-1, logits.shape[-1]).float(), labels.reshape(-1)
    rows = F.cross_entropy(lg, lab, ignore_index=ignore_index, reduction="none")  # 0 on ignored rows
    if reduction == "none":
        return rows
    total = rows.sum()  # "sum" and "mean" reduce the same per-row values in the same order
    if reduction == "sum":
        return total
    return total / (lab != ignore_index).sum().clamp_min(1).to(total.dtype)  # 0, not NaN, if all ignored


class _VPCERef(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index, vstart, group):
        lg = logits.reshape(-1, logits.shape[-1]).float()
        lab = labels.reshape(-1)
        mx = lg.max(-1).values
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(lg - mx[:, None])
        sm = ex.sum(-1)
        dist.all_reduce(sm, group=group)
        V = lg.shape[-1]
        local = lab - vstart
        inside = (local >= 0) & (local < V) & (lab != ignore_index)
        tg = torch.zeros_like(mx)
        idx = local.clamp(0, V - 1)
        tg[inside] = lg[inside, idx[inside]]
        dist.all_reduce(tg, group=group)
        lse = mx + torch.log(sm)
        valid = lab != ignore_index
        loss = torch.where(valid, lse - tg, torch.zeros_like(lse))
        ctx.save_for_backward(lg, lse, local, inside, valid)
        ctx.shape = logits.shape
        ctx.dtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, g):
        lg, lse, local, inside, valid = ctx.saved_tensors
        p = torch.exp(lg - lse[:, None])
        p[inside, local[inside]] -= 1.0
        p = p * (g * valid)[:, None]
        return p.view(ctx.shape).to(ctx.dtype), None, None, None, None


def _vocab_parallel_ce_reference(logits, labels, ignore_index, reduction, vstart, group):
    rows = _VPCERef.apply(logits, labels, ignore_index, vstart, group)
    valid = labels.reshape(-1) != ignore_index
    if reduction == "mean":
        return rows.sum() / valid.sum().clamp_min(1)
    if reduction == "sum":
        return rows.sum()
    return rows.view(labels.shape)
