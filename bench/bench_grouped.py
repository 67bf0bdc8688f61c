"""Grouped expert MLP (one grouped tcgen05 GEMM per matrix) vs one GEMM launch per expert.

    python bench/bench_grouped.py [--experts 64] [--hidden 2048] [--inter 1408] [--tokens 8192] [--topk 6]

DeepSeek-V2-Lite expert shapes by default; balanced random routing; forward +
backward timed with CUDA events (median).
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.models.moe import ExpertMLP, run_experts_grouped  # noqa: E402
from nano_train_b200.ops._ext import check_status  # noqa: E402
from nano_train_b200.ops.grouped import _StackCache, grouped_swiglu_experts  # noqa: E402


def t_ms(fn, iters=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    return sorted(ts)[len(ts) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=1408)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--topk", type=int, default=6)
    a = ap.parse_args()
    dev = torch.device("cuda")
    torch.manual_seed(0)
    E, H, I = a.experts, a.hidden, a.inter
    experts = torch.nn.ModuleList([ExpertMLP(H, I, param_dtype=torch.bfloat16, param_device=dev) for _ in range(E)])
    n = a.tokens * a.topk
    counts = torch.bincount(torch.randint(0, E, (n,), device=dev), minlength=E)
    x = torch.randn(n, H, device=dev, dtype=torch.bfloat16, requires_grad=True)
    cache = _StackCache()

    def grouped():
        y = grouped_swiglu_experts(x, counts, experts, cache, max_rows=n + E * 127)
        y.sum().backward()

    cl = counts.tolist()

    def loop():
        y = run_experts_grouped(experts, x, cl)
        y.sum().backward()

    flops = 3 * 2 * n * 3 * H * I
    tg, tl = t_ms(grouped), t_ms(loop)
    check_status(0)
    print(json.dumps(dict(experts=E, hidden=H, inter=I, rows=n, grouped_ms=tg, loop_ms=tl, speedup=tl / tg,
                          grouped_tflops=flops / tg / 1e9, loop_tflops=flops / tl / 1e9)))


if __name__ == "__main__":
    main()
