"""Optimizer factory (reference: src/optimizer.py:12-55).

``create_optimizer(model, learning_rate, weight_decay)`` groups parameters
the reference's way (names containing ``bias``, ``ln_`` or ``layer_norm``
get no weight decay) and returns the flat-buffer fused AdamW
(betas (0.9, 0.95), eps 1e-8): one fused kernel per parameter group instead
of a per-parameter loop.
"""
from __future__ import annotations

import torch.nn as nn

from .parallel.flat_optimizer import FlatAdamW


def create_optimizer(model: nn.Module, learning_rate: float, weight_decay: float, *, max_grad_norm=None,
                     dp_group=None, strategy: str = "no_shard") -> FlatAdamW:
    if learning_rate <= 0:
        raise ValueError("learning_rate must be positive")
    if weight_decay < 0:
        raise ValueError("weight_decay must be non-negative")
    decay, no_decay, seen = [], [], set()
    for name, p in model.named_parameters():
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        low = name.lower()
        (no_decay if ("bias" in low or "ln_" in low or "layer_norm" in low) else decay).append(p)
    groups = [dict(params=decay, weight_decay=weight_decay, name="decay"),
              dict(params=no_decay, weight_decay=0.0, name="no_decay")]
    return FlatAdamW(groups, lr=learning_rate, betas=(0.9, 0.95), eps=1e-8, weight_decay=weight_decay,
                     max_grad_norm=max_grad_norm, dp_group=dp_group, strategy=strategy)
