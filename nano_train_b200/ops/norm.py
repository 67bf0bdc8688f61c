"""RMSNorm / LayerNorm (fused residual add) on sm_100a row kernels.

Reference parity: RMSNorm src/models/deepseek.py:386-438 (x * rsqrt(mean(x^2)
+ eps) * w); LayerNorm src/layers.py:639-781 (biased variance). The CUDA path
accumulates in fp32 whatever the storage dtype.
"""
from __future__ import annotations

import torch

from ._ext import ext


def _native(t):
    return t.is_cuda and t.dtype in (torch.bfloat16, torch.float32)


def _rmsnorm_bwd(dy, h, weight, rstd, dres):
    """(dx, dw) of the RMSNorm; when the weight carries an fp32 ``main_grad`` view of a gradient
    bucket, dW is added into it by the column-sum kernel and dw is None (as for the linears)."""
    mg = getattr(weight, "main_grad", None)
    into = mg if (mg is not None and mg.dtype == torch.float32 and mg.is_cuda and mg.is_contiguous()) else None
    dx, dw = ext().rmsnorm_bwd(dy.contiguous(), h, weight.contiguous(), rstd, dres, into)
    if into is not None:
        hook = getattr(weight, "_ntb_grad_ready_hook", None)
        if hook is not None:
            hook(weight)
        return dx, None
    return dx, dw


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        xc = x.contiguous()
        y, h, rstd = ext().rmsnorm_fwd(xc, None, weight.contiguous(), eps)
        ctx.save_for_backward(h, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        h, weight, rstd = ctx.saved_tensors
        dx, dw = _rmsnorm_bwd(dy, h, weight, rstd, None)
        return dx, dw, None


class _AddRMSNormFn(torch.autograd.Function):
    """h = x + residual; y = rmsnorm(h). Returns (y, h)."""

    @staticmethod
    def forward(ctx, x, residual, weight, eps):
        y, h, rstd = ext().rmsnorm_fwd(x.contiguous(), residual.contiguous(), weight.contiguous(), eps)
        ctx.save_for_backward(h, weight, rstd)
        return y, h

    @staticmethod
    def backward(ctx, dy, dh):
        h, weight, rstd = ctx.saved_tensors
        dx, dw = _rmsnorm_bwd(dy, h, weight, rstd, dh.contiguous() if dh is not None else None)
        return dx, dx, dw, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if _native(x) and weight.dtype == x.dtype:
        return _RMSNormFn.apply(x, weight, eps)
    var = x.float().pow(2).mean(-1, keepdim=True)
    return (x.float() * torch.rsqrt(var + eps)).to(x.dtype) * weight


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """Returns (rmsnorm(x + residual), x + residual)."""
    if _native(x) and weight.dtype == x.dtype and residual.dtype == x.dtype:
        return _AddRMSNormFn.apply(x, residual, weight, eps)
    h = x + residual
    return rms_norm(h, weight, eps), h


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        xc = x.contiguous()
        y, mean, rstd = ext().layernorm_fwd(xc, weight.contiguous(), bias, eps)
        ctx.save_for_backward(xc, weight, mean, rstd)
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, mean, rstd = ctx.saved_tensors
        dx, dw, db = ext().layernorm_bwd(dy.contiguous(), x, weight.contiguous(), mean, rstd)
        return dx, dw, (db if ctx.has_bias else None), None


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, eps: float = 1e-5):
    if _native(x) and weight.dtype == x.dtype:
        return _LayerNormFn.apply(x, weight, bias, eps)
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    y = (x - mean) / torch.sqrt(var + eps) * weight
    return y + bias if bias is not None else y
