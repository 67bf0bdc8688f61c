"""Flat-buffer optimizer kernels: fused AdamW and gradient statistics.

Parameters, fp32 master weights, moments and fp32 gradients live in
contiguous per-domain buffers, so one launch updates every parameter of a
bucket (the reference loops over parameters in Python:
src/runtime/optimizer_runtime.py:68-116, src/distributed/zero.py:451-474).
"""
from __future__ import annotations

import math

import torch

from ._ext import ext


def adamw_flat_(param: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, grad: torch.Tensor, *,
                lr: float, beta1: float, beta2: float, eps: float, weight_decay: float, step: int,
                param_bf16: torch.Tensor | None = None, grad_scale: torch.Tensor | None = None,
                skip: torch.Tensor | None = None) -> None:
    """In-place torch.optim.AdamW step on flat fp32 tensors.

    ``grad_scale`` (fp32 [1], device) multiplies the gradient (unscale and DP
    averaging folded in); ``skip`` (int32 [1], device) non-zero turns the call
    into a no-op without a host sync; ``param_bf16`` receives a bf16 copy.
    """
    if param.is_cuda:
        ext().adamw_flat_(param, exp_avg, exp_avg_sq, grad, param_bf16, lr, beta1, beta2, eps, weight_decay, step,
                          grad_scale, skip)
        return
    if skip is not None and int(skip.item()) != 0:
        return
    g = grad.float()
    if grad_scale is not None:
        g = g * grad_scale.float()
    param.mul_(1.0 - lr * weight_decay)
    exp_avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    denom = (exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)
    if param_bf16 is not None:
        param_bf16.copy_(param)


def grad_stats_(grad: torch.Tensor, out: torch.Tensor, inv_scale: torch.Tensor | None = None) -> None:
    """Optionally unscale ``grad`` in place; add sum(g^2) to out[0]; set out[1]=1 on non-finite."""
    if grad.is_cuda:
        ext().grad_stats_(grad, inv_scale, out)
        return
    if inv_scale is not None:
        grad.mul_(inv_scale)
    g = grad.float()
    out[0] += (g * g).sum()
    if not bool(torch.isfinite(g).all()):
        out[1] = 1.0
