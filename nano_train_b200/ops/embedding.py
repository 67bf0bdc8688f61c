"""Embedding gather / scatter-add (vocab-parallel aware).

Reference parity: src/layers.py:788-900 (F.embedding). The backward
accumulates in fp32 with atomics, into ``weight.main_grad`` when the weight
has one.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, vstart):
        ctx.save_for_backward(ids)
        ctx.meta = (weight, vstart)
        return ext().embedding_fwd(ids, weight, vstart)

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        weight, vstart = ctx.meta
        mg = getattr(weight, "main_grad", None)
        if mg is not None:
            ext().embedding_bwd_(ids, dout, mg, vstart)
            hook = getattr(weight, "_ntb_grad_ready_hook", None)
            if hook is not None:
                hook(weight)
            return None, None, None
        dw = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        ext().embedding_bwd_(ids, dout, dw, vstart)
        return None, dw.to(weight.dtype), None


def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0) -> torch.Tensor:
    """Rows of ``weight`` for ``ids``; ids outside [vocab_start, vocab_start+V) give zeros."""
    if weight.is_cuda and weight.dtype in (torch.bfloat16, torch.float32):
        return _EmbeddingFn.apply(ids, weight, vocab_start)
    if vocab_start == 0 and weight.shape[0] > 0 and (ids.numel() == 0 or int(ids.max()) < weight.shape[0]):
        return F.embedding(ids, weight)
    local = ids - vocab_start
    mask = (local < 0) | (local >= weight.shape[0])
    out = F.embedding(local.clamp(0, weight.shape[0] - 1), weight)
    return out.masked_fill(mask[..., None], 0.0)
