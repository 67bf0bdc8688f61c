"""SwiGLU and exact GELU.

SwiGLU works on the packed [.., 2I] output of one fused gate|up GEMM
(reference: src/models/moe.py:146-193 computes silu(gate(x)) * up(x) with two
GEMMs). GELU is the exact erf form (src/layers.py:1017-1095).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


def _native(t):
    return t.is_cuda and t.dtype in (torch.bfloat16, torch.float32)


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ctx.save_for_backward(gu)
        return ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dout):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(dout, gu)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """silu(gu[..., :I]) * gu[..., I:]."""
    if _native(gu):
        return _SwiGLUFn.apply(gu)
    g, u = gu.chunk(2, dim=-1)
    return F.silu(g) * u


class _GeluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        xc = x.contiguous()
        ctx.save_for_backward(xc)
        return ext().gelu_fwd(xc)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return ext().gelu_bwd(dy, x)


def gelu(x: torch.Tensor) -> torch.Tensor:
    if _native(x):
        return _GeluFn.apply(x)
    return F.gelu(x)
