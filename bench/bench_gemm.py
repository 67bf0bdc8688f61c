"""Device-timed throughput of the tcgen05 GEMM against torch.matmul (cuBLAS).

    python bench/bench_gemm.py [--shapes llama8b]

Times each GEMM with CUDA events after warm-up; inputs of the large shapes
exceed the 126 MB L2, and an L2 flush buffer is written between iterations.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.ops._ext import check_status, ext  # noqa: E402

LLAMA8B = [
    # (name, M, N, K, a_mn, b_mn)
    ("qkv_fwd", 4096, 6144, 4096, False, False),
    ("o_fwd", 4096, 4096, 4096, False, False),
    ("gateup_fwd", 4096, 28672, 4096, False, False),
    ("down_fwd", 4096, 4096, 14336, False, False),
    ("lmhead_fwd", 4096, 128256, 4096, False, False),
    ("down_dgrad", 4096, 14336, 4096, False, True),
    ("down_wgrad", 4096, 14336, 4096, True, True),
    ("gateup_wgrad", 28672, 4096, 4096, True, True),
    ("sq8192", 8192, 8192, 8192, False, False),
    # weight gradients as training runs them: accumulated into the fp32 main_grad
    ("down_wgrad_f32acc", 4096, 14336, 4096, True, True),
    ("qkv_wgrad_f32acc", 6144, 4096, 4096, True, True),
]


def time_fn(fn, iters=20, warmup=5, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    C = ext()
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)
    rows = []
    for name, M, N, K, a_mn, b_mn in LLAMA8B:
        A = torch.randn(K, M, device="cuda", dtype=torch.bfloat16) if a_mn else torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        B = torch.randn(K, N, device="cuda", dtype=torch.bfloat16) if b_mn else torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        acc = name.endswith("_f32acc")
        out = torch.zeros(M, N, device="cuda", dtype=torch.float32 if acc else torch.bfloat16)
        t_ours = time_fn(lambda: C.gemm_bf16(A, B, out, None, a_mn, b_mn, acc, 1.0), args.iters, flush=flush)
        Aop = A.t() if a_mn else A
        Bop = B if b_mn else B.t()
        if acc:  # cuBLAS bf16 GEMM into a bf16 temporary + fp32 accumulate (what eager PyTorch does)
            t_cublas = time_fn(lambda: out.add_(torch.matmul(Aop, Bop)), args.iters, flush=flush)
            out.zero_()
        else:
            t_cublas = time_fn(lambda: torch.matmul(Aop, Bop, out=out), args.iters, flush=flush)
        ref = Aop.float() @ Bop.float() if M * N * K <= 4096 * 6144 * 4096 else None
        C.gemm_bf16(A, B, out, None, a_mn, b_mn, False, 1.0)
        if acc:
            C.gemm_bf16(A, B, out, None, a_mn, b_mn, True, 1.0)
            ref = 2 * ref if ref is not None else None
        err = None
        if ref is not None:
            err = ((out.float() - ref).norm() / ref.norm()).item()
        flops = 2.0 * M * N * K
        row = dict(name=name, M=M, N=N, K=K, a_mn=a_mn, b_mn=b_mn, ours_ms=t_ours, cublas_ms=t_cublas,
                   ours_tflops=flops / t_ours / 1e9, cublas_tflops=flops / t_cublas / 1e9, rel_err=err)
        rows.append(row)
        print(json.dumps(row), flush=True)
        del A, B, out
    check_status(0)
    if args.out:
        with open(args.out, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
