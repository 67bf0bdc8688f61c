"""Learning-rate schedule: linear warm-up, then cosine decay to ``min_lr``.

Same public interface as the reference's scheduler (src/scheduler.py:11-83):
``CosineAnnealingScheduler(optimizer, warmup_steps, max_steps, min_lr)`` with
``step() -> lr``, ``get_lr()``, ``state_dict()`` / ``load_state_dict()``. The
base LR is the optimizer's LR at construction. Works with any optimizer that
exposes ``param_groups`` (torch optimizers and ``FlatAdamW``).
"""
from __future__ import annotations

import math
from typing import Any


class CosineAnnealingScheduler:
    def __init__(self, optimizer, warmup_steps: int, max_steps: int, min_lr: float = 0.0) -> None:
        if warmup_steps < 0:
            raise ValueError("warmup_steps must be >= 0")
        if max_steps <= 0:
            raise ValueError("max_steps must be > 0")
        if warmup_steps >= max_steps:
            raise ValueError("warmup_steps must be smaller than max_steps")
        if min_lr < 0:
            raise ValueError("min_lr must be >= 0")
        self.optimizer = optimizer
        self.warmup_steps = int(warmup_steps)
        self.max_steps = int(max_steps)
        self.min_lr = float(min_lr)
        self.base_lrs = [float(g["lr"]) for g in optimizer.param_groups]
        self.current_step = 0

    def get_lr(self) -> float:
        peak = self.base_lrs[0]
        s = self.current_step
        if self.warmup_steps > 0 and s <= self.warmup_steps:
            return peak * s / self.warmup_steps
        frac = (s - self.warmup_steps) / float(self.max_steps - self.warmup_steps)
        frac = 0.0 if frac < 0 else (1.0 if frac > 1 else frac)
        return self.min_lr + 0.5 * (peak - self.min_lr) * (1.0 + math.cos(math.pi * frac))

    def _apply(self, lr: float) -> None:
        for g in self.optimizer.param_groups:
            g["lr"] = lr

    def step(self) -> float:
        self.current_step += 1
        lr = self.get_lr()
        self._apply(lr)
        return lr

    def state_dict(self) -> dict[str, Any]:
        return {"current_step": self.current_step, "base_lrs": list(self.base_lrs)}

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        self.current_step = int(state_dict["current_step"])
        if "base_lrs" in state_dict:
            self.base_lrs = [float(x) for x in state_dict["base_lrs"]]
        self._apply(self.get_lr())
