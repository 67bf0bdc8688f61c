"""NVFP4 GEMM (e2m1, e4m3 scales per 1x16 group, tcgen05 kind::mxf4nvf4) vs the bf16 and
block-scaled e4m3 tcgen05 GEMMs, device-timed (CUDA events, median of 20 after 5 warm-ups;
operands of 64-300 MB, larger than L2 for the big shapes).

    python bench/bench_fp4_gemm.py
"""
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.ops import fp4  # noqa: E402
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
    shapes = ((4096, 4096, 4096), (16384, 2048, 8192), (16384, 8192, 2048), (16384, 6144, 2048), (8192, 8192, 8192))
    for M, N, K in shapes:
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        a, b = fp4.quantize(x), fp4.quantize(w)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t4 = t_ms(lambda: fp4.gemm(a, b, out=y))
        tb = t_ms(lambda: C.gemm_bf16(x, w, y, None, False, False, False, 1.0))
        xq, sx = C.fp8_quantize(x, 1, False, 0)
        wq, sw = C.fp8_quantize(w, 128, False, 0)
        t8 = t_ms(lambda: C.gemm_fp8_blockscaled(xq, sx, wq, sw, y))
        tq = t_ms(lambda: fp4.quantize(x))
        fl = 2.0 * M * N * K
        print(json.dumps(dict(M=M, N=N, K=K, fp4_ms=round(t4, 4), fp8_ms=round(t8, 4), bf16_ms=round(tb, 4),
                              act_quant_ms=round(tq, 4), fp4_tflops=round(fl / t4 / 1e9, 1),
                              fp8_tflops=round(fl / t8 / 1e9, 1), bf16_tflops=round(fl / tb / 1e9, 1),
                              fp4_vs_bf16=round(tb / t4, 2))), flush=True)
        del x, w, a, b, y, xq, wq
    check_status(0)


if __name__ == "__main__":
    main()
