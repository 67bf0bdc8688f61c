"""Data-parallel tutorial with torch DistributedDataParallel (reference: examples/train_ddp.py).

    python examples/launch.py --world-size 2 --backend gloo --script examples/train_ddp.py
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/train_ddp.py

SimpleModel = 3 x Linear with ReLU (the framework's Linear, so the shared precision flags apply: --fp8 /
--fp4 with their backends, loss scaling where the mode needs it), MSE on a synthetic regression task,
DistributedSampler sharding, DDP gradient all-reduce (NCCL on GPUs, gloo on CPU).
"""
import argparse
import datetime
import os
import sys

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.nn.parallel import DistributedDataParallel as DDP
from torch.utils.data import DataLoader, DistributedSampler, TensorDataset

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.distributed.device import get_backend, get_device  # noqa: E402
from nano_train_b200.layers import Linear  # noqa: E402
from nano_train_b200.precision.mixed_precision import (dtype_alias_to_torch,  # noqa: E402
                                                       finalize_module_precision_resolver,
                                                       refresh_persistent_lowbit_params)
from nano_train_b200.precision.precision_args import add_mixed_precision_args, build_precision_runtime  # noqa: E402


class SimpleModel(nn.Module):
    def __init__(self, input_size=10, hidden=128, **kw):
        """``kw``: param_dtype / param_device / precision_resolver of the three linears."""
        super().__init__()
        self.net = nn.Sequential(Linear(input_size, hidden, module_path="net.0", **kw), nn.ReLU(),
                                 Linear(hidden, hidden, module_path="net.2", **kw), nn.ReLU(),
                                 Linear(hidden, 1, module_path="net.4", **kw))

    def forward(self, x):
        return self.net(x)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch_size", type=int, default=32)
    ap.add_argument("--num_samples", type=int, default=1000)
    ap.add_argument("--epochs", type=int, default=3)
    ap.add_argument("--max_steps", type=int, default=1_000_000)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--hidden_size", type=int, default=128)
    ap.add_argument("--log_every", type=int, default=0)
    add_mixed_precision_args(ap)
    a = ap.parse_args()
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    backend = get_backend()
    dev = get_device("cuda" if backend == "nccl" else "cpu", local)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    torch.manual_seed(0)
    pc, resolver, pcc = build_precision_runtime(a, dev)
    pdt = dtype_alias_to_torch(pc.params_dtype)
    model = SimpleModel(10, a.hidden_size, param_dtype=pdt, param_device=dev, precision_resolver=resolver)
    finalize_module_precision_resolver(resolver)
    ddp = DDP(model, device_ids=[dev.index] if dev.type == "cuda" else None) if world > 1 else model
    g = torch.Generator().manual_seed(1)
    X = torch.randn(a.num_samples, 10, generator=g)
    Y = X.pow(2).sum(-1, keepdim=True)
    ds = TensorDataset(X, Y)
    sampler = DistributedSampler(ds, num_replicas=world, rank=rank) if world > 1 else None
    loader = DataLoader(ds, batch_size=a.batch_size, sampler=sampler, shuffle=sampler is None)
    opt = torch.optim.AdamW(ddp.parameters(), lr=a.lr)
    step = 0
    for epoch in range(a.epochs):
        if sampler is not None:
            sampler.set_epoch(epoch)
        total = 0.0
        for x, y in loader:
            if step >= a.max_steps:
                break
            opt.zero_grad()
            with pcc.autocast_context():
                pred = ddp(x.to(dev, pdt))
            loss = nn.functional.mse_loss(pred.float(), y.to(dev))
            pcc.backward(loss)
            applied = pcc.prepare_optimizer_step(model) if pcc.uses_loss_scaling else True
            if applied:
                opt.step()
                refresh_persistent_lowbit_params(model)
            pcc.update_after_step(step_applied=applied)
            total += float(loss.detach())
            if rank == 0 and a.log_every and step % a.log_every == 0:
                print(f"step {step} loss {float(loss.detach()):.5f}", flush=True)
            step += 1
        if rank == 0:
            print(f"epoch {epoch} mean loss {total / max(1, len(loader)):.5f}", flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
