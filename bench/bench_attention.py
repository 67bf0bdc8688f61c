"""Device-timed flash attention forward: tcgen05 kernel vs the mma.sync kernel (and backward for context).

    python bench/bench_attention.py [--seq 4096] [--heads 32] [--kv-heads 8]

FLOPs counted as 4 * S^2 * D * H (halved for causal); CUDA events, median of
iterations after warm-up; inputs are reused (K/V per head fit in L2, as in training).
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.ops._ext import check_status, ext  # noqa: E402


def t_ms(fn, iters=20, warm=3):
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
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    a = ap.parse_args()
    C = ext()
    B, S, H, HK, D = a.batch, a.seq, a.heads, a.kv_heads, 128
    qkv = torch.randn(B, S, H + 2 * HK, D, device="cuda", dtype=torch.bfloat16)
    q, k, v = qkv[:, :, :H], qkv[:, :, H:H + HK], qkv[:, :, H + HK:]
    sc = D ** -0.5
    fl = 4.0 * S * S * D * H * B / 2
    rows = []
    for causal in (True, False):
        f = fl * (1 if causal else 2)
        t_tc = t_ms(lambda: C.flash_attn_fwd_tc(q, k, v, sc, causal))
        t_old = t_ms(lambda: C.flash_attn_fwd(q, k, v, sc, causal))
        rows.append(dict(kind="fwd", causal=causal, S=S, H=H, HK=HK, tc_ms=t_tc, mma_sync_ms=t_old,
                         tc_tflops=f / t_tc / 1e9, mma_sync_tflops=f / t_old / 1e9, speedup=t_old / t_tc))
        print(json.dumps(rows[-1]), flush=True)
        o, lse = C.flash_attn_fwd_tc(q, k, v, sc, causal)
        do = torch.randn_like(o)
        t_tc = t_ms(lambda: C.flash_attn_bwd(do, q, k, v, o, lse, sc, causal))
        os.environ["NTB_ATTN_BWD_LEGACY"] = "1"
        t_old = t_ms(lambda: C.flash_attn_bwd(do, q, k, v, o, lse, sc, causal))
        del os.environ["NTB_ATTN_BWD_LEGACY"]
        fb = 2.5 * f
        rows.append(dict(kind="bwd", causal=causal, S=S, H=H, HK=HK, tc_ms=t_tc, mma_sync_ms=t_old,
                         tc_tflops=fb / t_tc / 1e9, mma_sync_tflops=fb / t_old / 1e9, speedup=t_old / t_tc))
        print(json.dumps(rows[-1]), flush=True)
    check_status(0)


if __name__ == "__main__":
    main()
