"""Optimizer factory (reference: src/optimizer.py:12-55).

``create_optimizer(model, learning_rate, weight_decay)`` groups parameters
the reference's way (names containing ``bias``, ``ln_`` or ``layer_norm``
get no weight decay) and returns the flat-buffer fused AdamW
(betas (0.9, 0.95), eps 1e-8): one fused kernel per parameter group instead
of a per-parameter loop.
"""
from __future__ import annotations

import torch
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


class AdamW(torch.optim.Optimizer):
    """Per-parameter AdamW with torch.optim.AdamW's interface, defaults and update rule
    (decoupled weight decay, bias-corrected moments; ``state[p]`` holds ``step``, ``exp_avg``,
    ``exp_avg_sq``). The reference exposes torch's class under this name (src/optimizer.py);
    here each fp32 CUDA parameter is updated by the fused AdamW kernel in one launch, and other
    parameters (CPU, or low-precision dtypes, which keep fp32 moments) use the same math in
    PyTorch. For many parameters the flat-buffer ``create_optimizer`` path is faster."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2) -> None:
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if eps < 0.0:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameters: {betas}")
        if weight_decay < 0.0:
            raise ValueError(f"Invalid weight_decay value: {weight_decay}")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        from .ops.optim import adamw_flat_

        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("AdamW does not support sparse gradients")
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32,
                                                        memory_format=torch.contiguous_format)
                st["step"] += 1
                fused = p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()
                target = p if p.dtype == torch.float32 else p.float()
                flat = target.view(-1) if fused else target
                grad = p.grad.float()
                adamw_flat_(flat, st["exp_avg"].view(-1) if fused else st["exp_avg"],
                            st["exp_avg_sq"].view(-1) if fused else st["exp_avg_sq"],
                            grad.contiguous().view(-1) if fused else grad, lr=group["lr"], beta1=beta1,
                            beta2=beta2, eps=group["eps"], weight_decay=group["weight_decay"], step=st["step"])
                if target is not p:
                    p.copy_(target)
        return loss
