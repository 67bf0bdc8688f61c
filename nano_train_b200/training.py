"""Public single-call training API for language models.

``LMTrainer(model, ...)`` owns the flat-buffer AdamW and runs one optimizer
step per ``train_step(input_ids, labels)`` call: host->device copy of the
batch (pinned host tensors are copied asynchronously), gradient accumulation
over micro-batches, fused optimizer update, and the mean loss as a device
scalar (read it with ``float(loss)``). For a tensor-parallel model the TP
group and sequence-parallel flag are read from the model, so replicated
parameters get their gradients summed over TP and count once in the
clipping norm.
"""
from __future__ import annotations

from typing import Optional

import torch

from .parallel.flat_optimizer import FlatAdamW, split_decay_groups
from .utils.nvtx import nvtx_range


class LMTrainer:
    def __init__(self, model: torch.nn.Module, *, lr: float = 3e-4, weight_decay: float = 0.1,
                 betas=(0.9, 0.95), eps: float = 1e-8, max_grad_norm: Optional[float] = 1.0,
                 micro_batch_size: int = 1, dp_group=None, strategy: str = "no_shard", grad_norm_group=None,
                 device: Optional[torch.device] = None, bucket_mb: Optional[float] = None,
                 overlap_grad_reduce: bool = True):
        self.model = model
        self.micro_batch_size = micro_batch_size
        self.device = device or next(model.parameters()).device
        tp_enabled = bool(getattr(model, "tp_enabled", False))
        tp_group = getattr(model, "tp_group", None) if tp_enabled else None
        self.optimizer = FlatAdamW(split_decay_groups(model, weight_decay, split_tp_replicated=tp_enabled), lr=lr,
                                   betas=betas, eps=eps, weight_decay=weight_decay, dp_group=dp_group,
                                   strategy=strategy, max_grad_norm=max_grad_norm,
                                   grad_norm_group=grad_norm_group if grad_norm_group is not None else tp_group,
                                   tp_group=tp_group,
                                   sequence_parallel=bool(getattr(model, "sequence_parallel", False)),
                                   bucket_mb=bucket_mb)
        # With the peer-memory ZeRO step, the last micro-batch's backward reduce-scatters every
        # gradient bucket as soon as it is complete (FlatAdamW.overlap_next_backward).
        self.overlap_grad_reduce = overlap_grad_reduce

    def train_step(self, input_ids: torch.Tensor, labels: torch.Tensor, lr: Optional[float] = None) -> torch.Tensor:
        with nvtx_range("h2d"):
            ids = input_ids.to(self.device, non_blocking=True)
            lab = labels.to(self.device, non_blocking=True)
        self.optimizer.zero_grad()
        B = ids.shape[0]
        mb = self.micro_batch_size
        n_mb = max(1, B // mb)
        total = torch.zeros((), dtype=torch.float32, device=self.device)
        for i in range(n_mb):
            with nvtx_range(f"forward mb{i}"):
                loss = self.model.forward_loss(ids[i * mb:(i + 1) * mb], lab[i * mb:(i + 1) * mb])
            if i == n_mb - 1 and self.overlap_grad_reduce:
                self.optimizer.overlap_next_backward()
            with nvtx_range(f"backward mb{i}"):
                (loss / n_mb).backward()
            total += loss.detach().float()
        with nvtx_range("optimizer"):
            self.optimizer.step(lr=lr)
        return total / n_mb
