"""Block-scaled fp8 GEMM (e4m3, 1x128 / 128x128 fp32 scales) vs the bf16 tcgen05 GEMM, device-timed.

    python bench/bench_fp8_gemm.py
"""
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.ops._ext import check_status, ext  # noqa: E402


def t_ms(fn, iters=20, warm=5):
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
    C = ext()
    for M, N, K in ((4096, 4096, 4096), (8192, 2048, 7168), (4096, 14336, 4096), (16384, 2816, 2048)):
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        xq, sx = C.fp8_quantize(x, 1, False, 0)
        wq, sw = C.fp8_quantize(w, 128, False, 0)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        tf = t_ms(lambda: C.gemm_fp8_blockscaled(xq, sx, wq, sw, y))
        tb = t_ms(lambda: C.gemm_bf16(x, w, y, None, False, False, False, 1.0))
        tq = t_ms(lambda: C.fp8_quantize(x, 1, False, 0))
        fl = 2.0 * M * N * K
        print(json.dumps(dict(M=M, N=N, K=K, fp8_ms=tf, bf16_ms=tb, act_quant_ms=tq, fp8_tflops=fl / tf / 1e9,
                              bf16_tflops=fl / tb / 1e9, speedup=tb / tf)), flush=True)
    check_status(0)


if __name__ == "__main__":
    main()
