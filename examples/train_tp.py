"""Tensor-parallel tutorial: a column -> row parallel MLP inside a small regression model.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/train_tp.py --tensor-model-parallel-size 2
    python examples/launch.py --world-size 2 --backend gloo --script examples/train_tp.py

TutorialModel = Linear(input -> hidden) -> GELU -> [ColumnParallel(hidden ->
intermediate) -> GELU -> RowParallel(intermediate -> hidden)] -> Linear(hidden -> 1),
MSE on a synthetic regression target. Ranks outside a TP group form the
data-parallel axis; gradients of replicated layers are all-reduced over it.
(reference: examples/train_tp.py)
"""
import argparse
import datetime
import os
import sys

import torch
import torch.distributed as dist
import torch.nn as nn

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.distributed.topology import initialize_model_parallel  # noqa: E402
from nano_train_b200.layers import ColumnParallelLinear, Linear, RowParallelLinear  # noqa: E402
from nano_train_b200 import ops  # noqa: E402
from nano_train_b200.parallel.flat_optimizer import FlatAdamW  # noqa: E402
from nano_train_b200.precision.mixed_precision import (dtype_alias_to_torch,  # noqa: E402
                                                       finalize_module_precision_resolver,
                                                       refresh_persistent_lowbit_params)
from nano_train_b200.precision.precision_args import add_mixed_precision_args, build_precision_runtime  # noqa: E402


class ParallelMLP(nn.Module):
    def __init__(self, hidden, inter, tp_rank, tp_size, tp_group, **kw):
        super().__init__()
        self.fc1 = ColumnParallelLinear(hidden, inter, tp_rank, tp_size, tp_group=tp_group, module_path="mlp.fc1", **kw)
        self.fc2 = RowParallelLinear(inter, hidden, tp_rank, tp_size, tp_group=tp_group, module_path="mlp.fc2", **kw)

    def forward(self, x):
        return self.fc2(ops.gelu(self.fc1(x)))


class TutorialModel(nn.Module):
    def __init__(self, input_size, hidden, inter, tp_rank, tp_size, tp_group, **kw):
        """``kw``: param_dtype / param_device / precision_resolver of every layer."""
        super().__init__()
        self.inp = Linear(input_size, hidden, module_path="inp", **kw)
        self.mlp = ParallelMLP(hidden, inter, tp_rank, tp_size, tp_group, **kw)
        self.out = Linear(hidden, 1, module_path="out", **kw)

    def forward(self, x):
        return self.out(self.mlp(ops.gelu(self.inp(x))))


def main():
    ap = argparse.ArgumentParser(description="Canonical TP/DP tutorial script")
    ap.add_argument("--tensor-model-parallel-size", type=int, default=None)
    ap.add_argument("--tp_size", type=int, default=None, help=argparse.SUPPRESS)
    ap.add_argument("--batch_size", type=int, default=32)
    ap.add_argument("--num_samples", type=int, default=1024)
    ap.add_argument("--epochs", type=int, default=3)
    ap.add_argument("--max_steps", type=int, default=100)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--weight_decay", type=float, default=0.01)
    ap.add_argument("--input_size", type=int, default=10)
    ap.add_argument("--hidden_size", type=int, default=256)
    ap.add_argument("--intermediate_size", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--log_every", type=int, default=10)
    add_mixed_precision_args(ap)
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp = a.tensor_model_parallel_size or a.tp_size or world
    topo = initialize_model_parallel(tensor_model_parallel_size=tp, pipeline_model_parallel_size=1,
                                     expert_model_parallel_size=1, timeout=datetime.timedelta(seconds=300))
    dev = topo.device
    torch.manual_seed(a.seed + topo.dp_rank)  # same replicated init within a TP group
    pc, resolver, pcc = build_precision_runtime(a, dev)
    model = TutorialModel(a.input_size, a.hidden_size, a.intermediate_size, topo.tp_rank, tp, topo.tp_group,
                          param_dtype=dtype_alias_to_torch(pc.params_dtype), param_device=dev,
                          precision_resolver=resolver)
    finalize_module_precision_resolver(resolver)
    opt = FlatAdamW([dict(params=list(model.parameters()), weight_decay=a.weight_decay)], lr=a.lr,
                    dp_group=topo.dp_group)
    g = torch.Generator().manual_seed(a.seed)
    X = torch.randn(a.num_samples, a.input_size, generator=g)
    Y = (X.sin().sum(-1, keepdim=True) + 0.1 * torch.randn(a.num_samples, 1, generator=g))
    shard = slice(topo.dp_rank, None, topo.dp_size)
    X, Y = X[shard].to(dev), Y[shard].to(dev)
    step = 0
    for epoch in range(a.epochs):
        for i in range(0, X.shape[0], a.batch_size):
            if step >= a.max_steps:
                break
            opt.zero_grad()
            with pcc.autocast_context():
                pred = model(X[i:i + a.batch_size].to(dtype_alias_to_torch(pc.params_dtype)))
            loss = torch.nn.functional.mse_loss(pred.float(), Y[i:i + a.batch_size])
            pcc.backward(loss)
            applied = pcc.prepare_optimizer_step(model) if pcc.uses_loss_scaling else True
            if applied:
                opt.step()
                refresh_persistent_lowbit_params(model)
            pcc.update_after_step(step_applied=applied)
            if topo.rank == 0 and a.log_every and step % a.log_every == 0:
                print(f"epoch {epoch} step {step} loss {float(loss.detach()):.6f}", flush=True)
            step += 1
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
