"""Expert-parallel MoE layer, forward + backward: fused peer-memory dispatch/combine vs NCCL all-to-all.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/bench_moe_ep.py [--tokens 8192] [--fp8]

DeepSeek-V2-Lite MoE shape by default (hidden 2048, 64 routed experts top-6, expert FFN 1408, 2 shared
experts), bf16, synthetic tokens. Device time per layer call (CUDA events, max over ranks) and the
NVLink roofline of the exchange: each rank sends and receives T*K*(n-1)/n rows of H values twice
(dispatch and combine) in the forward and twice in the backward.
"""
import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.models.moe import ExpertParallelMoE  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=6)
    ap.add_argument("--ffn", type=int, default=1408)
    ap.add_argument("--shared", type=int, default=2)
    ap.add_argument("--capacity-factor", type=float, default=1.25)
    ap.add_argument("--fp8", action="store_true", help="e4m3 1x128 payload (native comm quant)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--fused-first", action="store_true")
    ap.add_argument("--no-main-grad", action="store_true", help="per-parameter .grad instead of flat fp32 main_grad")
    ap.add_argument("--breakdown", action="store_true",
                    help="print the top kernels of two fused iterations (torch.profiler; diagnosis only, not timing)")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    torch.manual_seed(rank)
    moe = ExpertParallelMoE(a.hidden, a.ffn, a.experts, a.topk, ep_rank=rank, ep_size=world,
                            ep_group=dist.group.WORLD, param_dtype=torch.bfloat16, param_device="cuda",
                            n_shared_experts=a.shared, scoring_func="softmax", capacity_factor=a.capacity_factor,
                            comm_quant_granularity="tile_1x128" if a.fp8 else None, comm_quant_backend="native")
    if not a.no_main_grad:
        # as under the flat optimizer: fp32 main_grad views of one buffer, weight gradients accumulate there
        from nano_train_b200.parallel.flat_optimizer import FlatParamBuffer

        FlatParamBuffer(list(moe.parameters()))
    x = torch.randn(1, a.tokens, a.hidden, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    dy = torch.randn(1, a.tokens, a.hidden, device="cuda", dtype=torch.bfloat16)
    res = {}
    for mode in (("fused", "all_to_all") if a.fused_first else ("all_to_all", "fused")):
        os.environ["NTB_FUSED_EP"] = "1" if mode == "fused" else "0"

        def step():
            out = moe(x)
            out.backward(dy)

        for _ in range(a.warmup):
            step()
        dist.barrier()
        torch.cuda.synchronize()
        m0 = torch.cuda.memory_stats()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.iters + 1)]
        import time

        host = 0.0
        s.record()
        ev[0].record()
        for i in range(a.iters):
            h0 = time.perf_counter()
            step()
            host += time.perf_counter() - h0
            ev[i + 1].record()
        e.record()
        torch.cuda.synchronize()
        per_iter = [round(ev[i].elapsed_time(ev[i + 1]), 2) for i in range(a.iters)]
        t = torch.tensor([s.elapsed_time(e) / a.iters], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        m1 = torch.cuda.memory_stats()
        res[mode] = {"ms": round(float(t), 3), "path": moe.last_path, "host_enqueue_ms": round(host * 1e3 / a.iters, 2),
                     "per_iter_ms_rank0": per_iter,
                     "allocator": {k: m1.get(k, 0) - m0.get(k, 0)
                                   for k in ("num_device_alloc", "num_device_free", "num_alloc_retries")}}
    if a.breakdown:
        os.environ["NTB_FUSED_EP"] = "1"
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
            for _ in range(2):
                out = moe(x)
                out.backward(dy)
            torch.cuda.synchronize()
        if rank == 0:
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=60))
            print(prof.key_averages().table(sort_by="self_cpu_time_total", row_limit=25, max_name_column_width=60))
            if os.environ.get("NTB_TRACE_OUT"):
                prof.export_chrome_trace(os.environ["NTB_TRACE_OUT"])
    elem = 1 if a.fp8 else 2
    rows = a.tokens * a.topk * (world - 1) / world
    link_bytes = 4 * rows * a.hidden * elem  # dispatch + combine, forward + backward (bwd in bf16)
    if a.fp8:
        link_bytes = 2 * rows * a.hidden * 1 + 2 * rows * a.hidden * 2
    res["exchange_roofline_ms_at_770GBps"] = round(link_bytes / 770e9 * 1e3, 3)
    res["speedup"] = round(res["all_to_all"]["ms"] / res["fused"]["ms"], 3)
    res["config"] = {k: v for k, v in vars(a).items()} | {"ep": world}
    if rank == 0:
        print(json.dumps(res))
    from nano_train_b200.parallel.ep_fused import clear_workspaces

    clear_workspaces()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
