"""Linear layer math on the tcgen05 GEMM.

forward  Y  = X W^T (+ b)            -> gemm(A=X K-major, B=W K-major)
dgrad    dX = dY W                   -> gemm(A=dY K-major, B=W N-major)
wgrad    dW = dY^T X (+= main_grad)  -> gemm(A=dY M-major, B=X N-major), fp32
                                        accumulation fused into the epilogue

When the weight carries a ``main_grad`` fp32 buffer (a view into the flat
gradient bucket of the optimizer) the weight gradient is accumulated straight
into it and autograd receives ``None`` for the weight; the optimizer reads the
bucket. Otherwise a regular ``.grad`` is produced.

Reference parity: src/layers.py:628-632 (Linear.forward), 1358-1360 and 1484
(Column/RowParallelLinear), whose backward is torch's autograd of F.linear.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext

_GEMM_DTYPES = (torch.bfloat16,)


def _native(t: torch.Tensor) -> bool:
    return t.is_cuda and t.dtype in _GEMM_DTYPES


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *, bias=None, a_mn=False, b_mn=False,
         accumulate=False, alpha=1.0, out_dtype=None) -> torch.Tensor:
    """``out = alpha * op(a) @ op(b)^T (+ bias) (+ out)``.

    ``a`` is [M, K] (``a_mn=False``) or [K, M] (``a_mn=True``); ``b`` is [N, K]
    (``b_mn=False``) or [K, N] (``b_mn=True``).
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype or a.dtype, device=a.device)
    if _native(a):
        ext().gemm_bf16(a, b, out, bias, a_mn, b_mn, accumulate, float(alpha))
        return out
    A = a.t() if a_mn else a
    B = b if b_mn else b.t()
    r = (A.float() @ B.float()) * alpha
    if bias is not None:
        r = r + bias.float()
    if accumulate:
        out.add_(r.to(out.dtype))
    else:
        out.copy_(r.to(out.dtype))
    return out


def accumulate_weight_grad(weight: torch.Tensor, dy2: torch.Tensor, x2: torch.Tensor):
    """Add dY^T X into ``weight.main_grad`` when present; otherwise return dW."""
    mg = getattr(weight, "main_grad", None)
    if mg is not None:
        gemm(dy2, x2, mg, a_mn=True, b_mn=True, accumulate=True)
        hook = getattr(weight, "_ntb_grad_ready_hook", None)
        if hook is not None:
            hook(weight)
        return None
    if _native(dy2):
        return gemm(dy2, x2, a_mn=True, b_mn=True, out_dtype=weight.dtype)
    return (dy2.t().float() @ x2.float()).to(weight.dtype)


class LinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        out = torch.empty(*shape[:-1], weight.shape[0], dtype=x.dtype, device=x.device)
        gemm(x2, weight, out.view(-1, weight.shape[0]), bias=bias)
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        ctx.in_shape = shape
        return out

    @staticmethod
    def backward(ctx, gout):
        x2, weight = ctx.saved_tensors
        g2 = gout.reshape(-1, gout.shape[-1])
        if not g2.is_contiguous():
            g2 = g2.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(g2, weight, b_mn=True).view(ctx.in_shape)
        dw = None
        if ctx.needs_input_grad[1]:
            dw = accumulate_weight_grad(weight, g2, x2)
        db = None
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = g2.float().sum(0).to(gout.dtype)
        return dx, dw, db


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Y = X W^T + b, on tcgen05 for CUDA bf16, torch otherwise."""
    if _native(x) and weight.dtype == x.dtype and x.shape[-1] % 8 == 0:
        return LinearFunction.apply(x, weight, bias)
    return F.linear(x, weight, bias)
