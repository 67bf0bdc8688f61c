"""Sharded optimizer step (ZeRO-2): fused peer-memory kernels vs NCCL reduce-scatter + AdamW + all-gather.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/bench_zero.py [--params 1.3e9]

A flat set of bf16 parameters (GPT-1.3B size by default, split in two buffers: matrices with decay, the
rest without) with fp32 gradients already in place; the timed region is ``FlatAdamW.step()`` alone
(CUDA events, max over ranks). Roofline of the fused step per rank: the slower of the peer traffic over
NVLink, (n-1)/n * P * 4 bytes of gradients in, at the measured 770 GB/s per direction, and the rank's HBM
traffic at the measured copy bandwidth (6548 GB/s): per shard element 4 + 4 bytes (own gradient read,
reduced gradient written), 16 + 12 (master, moments, reduced gradient read; master and moments written)
and 2 (own parameter); per element of the peers' shards 4 (gradients the peers read) + 2 (parameters the
peers write). Clipping needs the global norm before any update, so the reduction and the update are two
passes that cannot overlap.
"""
import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.parallel.flat_optimizer import FlatAdamW  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=float, default=1.3e9)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--clip", type=float, default=1.0)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    n_mat = int(a.params * 0.98) // 4096 * 4096
    n_vec = int(a.params) - n_mat
    res = {}
    for mode in ("nccl", "fused"):
        torch.manual_seed(0)
        mats = [torch.nn.Parameter(torch.randn(n_mat // 4096 // 16, 4096, device="cuda", dtype=torch.bfloat16) * 0.02)
                for _ in range(16)]
        vecs = [torch.nn.Parameter(torch.zeros(n_vec, device="cuda", dtype=torch.bfloat16))]
        opt = FlatAdamW([{"params": mats, "weight_decay": 0.1}, {"params": vecs, "weight_decay": 0.0}], lr=1e-4,
                        dp_group=dist.group.WORLD, strategy="optim_grads", max_grad_norm=a.clip,
                        fused_dp=(mode == "fused"))
        for b in opt.buffers:
            b.grad_data.normal_(0, 1e-3)

        for _ in range(a.warmup):
            opt.step()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            opt.step()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[mode] = {"ms": round(float(t), 3), "fused": opt.fused_dp}
        if opt._zsym is not None:
            opt._zsym.close()
        del opt, mats, vecs
        torch.cuda.empty_cache()
    P = n_mat + n_vec
    link = (world - 1) / world * P * 4 / 770e9
    hbm_bytes = P / world * (4 + 4 + 16 + 12 + 2) + (world - 1) / world * P * (4 + 2)
    res["roofline_ms"] = round(max(link, hbm_bytes / 6.548e12) * 1e3, 3)
    res["fused_fraction_of_roofline"] = round(res["roofline_ms"] / res["fused"]["ms"], 3)
    res["speedup"] = round(res["nccl"]["ms"] / res["fused"]["ms"], 3)
    res["config"] = {"params": P, "dp": world, "clip": a.clip}
    if rank == 0:
        print(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
