"""Cross-entropy loss module (reference: src/losses.py:9-133).

``CrossEntropyLoss(ignore_index=-100, reduction="mean")`` over the last
dimension of ``logits`` against integer ``targets`` of the leading shape.
On CUDA it runs the fused sm_100a cross-entropy kernels (row statistics +
in-place gradient); on CPU the fp32 PyTorch formulation.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops


class CrossEntropyLoss(nn.Module):
    def __init__(self, ignore_index: int = -100, reduction: str = "mean"):
        super().__init__()
        if reduction not in ("mean", "sum", "none"):
            raise ValueError(f"reduction must be 'mean', 'sum' or 'none', got {reduction!r}")
        self.ignore_index = ignore_index
        self.reduction = reduction

    def forward(self, logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        if logits.shape[:-1] != targets.shape:
            raise ValueError(f"logits {tuple(logits.shape)} and targets {tuple(targets.shape)} disagree")
        out = ops.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1),
                                ignore_index=self.ignore_index, reduction=self.reduction)
        return out.view(targets.shape) if self.reduction == "none" else out
