"""Small, self-contained launches of the hot kernels for Nsight Compute captures.

    python bench/profile_kernels.py <case> [--iters N]

Each case allocates a few hundred MB at most (inputs larger than the 126 MB
L2 where the kernel is bandwidth-bound), runs 2 warm-up launches and then
``--iters`` launches, and checks the kernel status word. Cases:

  gemm          any dense tcgen05 GEMM (--mnk M,N,K --layout fwd|dgrad|wgrad; --cublas for torch.matmul);
                NTB_GEMM_BN=128|256 forces the tile width
  gemm_fwd      tcgen05 GEMM 4096 x 6144 x 4096 (Llama-8B QKV, K-major A and B)
  gemm_wgrad    4096 x 14336 x 4096 with M-major A / N-major B (weight gradient)
  attn_fwd      flash attention fwd, B=1 S=4096 32q/8kv heads d=128 causal
  attn_bwd      flash attention bwd, same shape
  attn_fwd_tc   tcgen05 flash attention fwd, same shape
  attn_bwd_tc   tcgen05 flash attention bwd (the default backward for head dim 128), same shape
  attn_{fwd,bwd}_{tc128,tc128_tp8,mla}  tcgen05 attention on the Llama shape, one TP = 8 rank of it
                (4 q / 1 kv heads) and the DeepSeek-V2-Lite MLA shape (--time reports TFLOP/s)
  fp8_gemm      block-scaled e4m3 GEMM 8192 x 2048 x 7168 (DeepSeek-V3 recipe scales)
  fp4_gemm      NVFP4 GEMM 16384 x 8192 x 2048 (GPT-1.3B MLP fc1 shape, e2m1 with e4m3 1x16 scales)
  grouped_fwd   grouped expert GEMM, 64 experts, 49152 routed rows x 2816 x 2048 (DeepSeek-V2-Lite gate|up)
  rmsnorm_bwd   RMSNorm backward 8192 x 4096 bf16
  adamw         fused flat AdamW over 64M fp32 elements
  swiglu        SwiGLU fwd 8192 x 14336
  mla_k         MLA key assembly [k_nope | rope(k_rope)], DeepSeek-V2-Lite micro-batch (8192 tokens, 16 heads,
                nope 128 / rope 64 / v 128, kv_lora 512); mla_k_bwd its backward
  ce            vocab cross-entropy stats+bwd 4096 x 32064
  router        fused top-k router fwd, 16384 tokens x 64 experts, top-6 softmax (bf16)
  router_bwd    its backward
  ep_layer      expert-parallel dispatch -> receive plan -> gather -> pull-combine of one MoE layer
                (8192 tokens x 2048, top-6 of 64 experts), run as a 1-rank group: every "peer" pointer
                is this GPU's own memory, so the kernels' code and memory behaviour are captured on one GPU
  zero_step     fused ZeRO step (reduce-scatter pull + AdamW + parameter stores) over 64M parameters,
                1-rank group (same reason)
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.ops._ext import check_status, ext  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", type=int, default=0,
                    help="also time this many launches with CUDA events (after the warm-up) and print ms / GB/s")
    ap.add_argument("--mnk", default="4096,4096,4096", help="gemm case: M,N,K")
    ap.add_argument("--layout", default="fwd", choices=("fwd", "dgrad", "wgrad"), help="gemm case: operand layout")
    ap.add_argument("--cublas", action="store_true", help="gemm case: time torch.matmul instead")
    a = ap.parse_args()
    nbytes = 0  # algorithmic DRAM bytes of one launch, where the case defines them
    nflops = 0  # algorithmic FLOPs of one launch, where the case defines them
    C = ext()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    bf = dict(device=dev, dtype=torch.bfloat16)
    if a.case == "gemm":
        # any dense GEMM: --mnk M,N,K and --layout fwd (a [M,K], b [N,K]), dgrad (b [K,N]) or
        # wgrad (a [K,M], b [K,N], fp32 accumulate); --cublas times torch.matmul of the same product
        M, N, K = (int(v) for v in a.mnk.split(","))
        nflops = 2 * M * N * K
        if a.layout == "wgrad":
            x, w = torch.randn(K, M, **bf), torch.randn(K, N, **bf)
            y = torch.zeros(M, N, device=dev, dtype=torch.float32)
            fn = lambda: C.gemm_bf16(x, w, y, None, True, True, True, 1.0)  # noqa: E731
            yb = torch.empty(M, N, **bf)
            ref = lambda: torch.matmul(x.t(), w, out=yb)  # noqa: E731  (bf16 out: cuBLAS has no fp32-accumulate form here)
        else:
            x = torch.randn(M, K, **bf)
            w = torch.randn(K, N, **bf) if a.layout == "dgrad" else torch.randn(N, K, **bf)
            y = torch.empty(M, N, **bf)
            bmn = a.layout == "dgrad"
            fn = lambda: C.gemm_bf16(x, w, y, None, False, bmn, False, 1.0)  # noqa: E731
            ref = lambda: torch.matmul(x, w if bmn else w.t(), out=y)  # noqa: E731
        if a.cublas:
            fn = ref
    elif a.case == "gemm_fwd":
        x, w = torch.randn(4096, 4096, **bf), torch.randn(6144, 4096, **bf)
        y = torch.empty(4096, 6144, **bf)
        fn = lambda: C.gemm_bf16(x, w, y, None, False, False, False, 1.0)  # noqa: E731
    elif a.case == "gemm_wgrad":
        dy, x = torch.randn(4096, 14336, **bf), torch.randn(4096, 4096, **bf)
        dw = torch.zeros(14336, 4096, device=dev, dtype=torch.float32)
        fn = lambda: C.gemm_bf16(dy, x, dw, None, True, True, True, 1.0)  # noqa: E731
    elif a.case == "attn_fwd_tc":
        qkv = torch.randn(1, 4096, 48, 128, **bf)
        q, k, v = qkv[:, :, :32], qkv[:, :, 32:40], qkv[:, :, 40:]
        fn = lambda: C.flash_attn_fwd_tc(q, k, v, 128 ** -0.5, True)  # noqa: E731
    elif a.case == "fp8_gemm":
        x = torch.randn(8192, 7168, **bf)
        w = torch.randn(2048, 7168, **bf)
        xq, sx = C.fp8_quantize(x, 1, False, 0)
        wq, sw = C.fp8_quantize(w, 128, False, 0)
        y = torch.empty(8192, 2048, **bf)
        fn = lambda: C.gemm_fp8_blockscaled(xq, sx, wq, sw, y)  # noqa: E731
    elif a.case in ("quant_tile", "quant_tile_sr"):
        # 1x128 e4m3 activation quantiser of the DeepSeek recipe, 16384 x 2048 bf16 (the MoE payload shape)
        x = torch.randn(16384, 2048, **bf)
        sr = a.case.endswith("sr")
        nbytes = x.numel() * (2 + 1) + x.numel() // 128 * 4  # read bf16, write codes and scales
        fn = lambda: C.fp8_quantize(x, 1, sr, 7)  # noqa: E731
    elif a.case == "fp4_gemm":
        from nano_train_b200.ops import fp4

        a4 = fp4.quantize(torch.randn(16384, 2048, **bf))
        b4 = fp4.quantize(torch.randn(8192, 2048, **bf))
        y = torch.empty(16384, 8192, **bf)
        fn = lambda: fp4.gemm(a4, b4, out=y)  # noqa: E731
    elif a.case == "grouped_fwd":
        from nano_train_b200.ops.grouped import pad_segments

        counts = torch.bincount(torch.randint(0, 64, (49152,), device=dev), minlength=64)
        off, rows = pad_segments(counts)
        x = torch.randn(rows, 2048, **bf)
        w = torch.randn(64 * 2816, 2048, **bf)
        y = torch.empty(rows, 2816, **bf)
        fn = lambda: C.gemm_grouped_bf16(x, w, y, off, 1)  # noqa: E731
    elif a.case == "attn_bwd_tc":
        qkv = torch.randn(1, 4096, 48, 128, **bf)
        q, k, v = qkv[:, :, :32], qkv[:, :, 32:40], qkv[:, :, 40:]
        o, lse = C.flash_attn_fwd_tc(q, k, v, 128 ** -0.5, True)
        do = torch.randn_like(o)
        fn = lambda: C.flash_attn_bwd(do, q, k, v, o, lse, 128 ** -0.5, True)  # noqa: E731
    elif a.case in ("attn_fwd_mla", "attn_bwd_mla", "attn_fwd_tc128", "attn_bwd_tc128", "attn_fwd_tc128_tp8",
                    "attn_bwd_tc128_tp8"):
        # DeepSeek-V2-Lite MLA shape (2 x 4096 tokens, 16 heads, q/k 192, v 128), the Llama shape
        # (1 x 4096, 32 q / 8 kv heads, 128) or its TP = 8 rank (4 q / 1 kv heads), causal; tcgen05 kernels
        mla = a.case.endswith("mla")
        Bq, Sq, hq, hkv, dqk, dvv = (2, 4096, 16, 16, 192, 128) if mla else (1, 4096, 32, 8, 128, 128)
        if a.case.endswith("tp8"):
            hq, hkv = 4, 1
        buf = torch.randn(Bq, Sq, hq * dqk + hkv * (dqk + dvv), **bf)
        q = buf[..., : hq * dqk].view(Bq, Sq, hq, dqk)
        k = buf[..., hq * dqk: (hq + hkv) * dqk].view(Bq, Sq, hkv, dqk)
        v = buf[..., (hq + hkv) * dqk:].view(Bq, Sq, hkv, dvv)
        sc = dqk ** -0.5
        o, lse = C.flash_attn_fwd_tc(q, k, v, sc, True)
        fwd_flops = Bq * hq * Sq * Sq * (dqk + dvv)  # causal: half of 2 * S^2 * (dqk + dv) per head
        if "fwd" in a.case:
            nflops = fwd_flops
            fn = lambda: C.flash_attn_fwd_tc(q, k, v, sc, True)  # noqa: E731
        else:
            nflops = fwd_flops * 5 // 2  # S recompute, dP, dV, dK, dQ
            do = torch.randn_like(o)
            fn = lambda: C.flash_attn_bwd(do, q, k, v, o, lse, sc, True)  # noqa: E731
    elif a.case in ("attn_fwd", "attn_bwd"):
        q = torch.randn(1, 4096, 32, 128, **bf)
        k = torch.randn(1, 4096, 8, 128, **bf)
        v = torch.randn(1, 4096, 8, 128, **bf)
        scale = 128 ** -0.5
        o, lse = C.flash_attn_fwd(q, k, v, scale, True)
        if a.case == "attn_fwd":
            fn = lambda: C.flash_attn_fwd(q, k, v, scale, True)  # noqa: E731
        else:
            os.environ["NTB_ATTN_BWD_LEGACY"] = "1"  # the mma.sync kernel
            do = torch.randn_like(o)
            fn = lambda: C.flash_attn_bwd(do, q, k, v, o, lse, scale, True)  # noqa: E731
    elif a.case == "rmsnorm_bwd":
        h = torch.randn(8192, 4096, **bf)
        w = torch.randn(4096, **bf)
        dy = torch.randn(8192, 4096, **bf)
        rstd = torch.rand(8192, device=dev) + 0.5
        nbytes = 3 * 8192 * 4096 * 2 + 8192 * 4 + 4096 * (2 + 4 + 2)  # dy, h, dx; rstd; w, dw (fp32 + bf16)
        fn = lambda: C.rmsnorm_bwd(dy, h, w, rstd, None)  # noqa: E731
    elif a.case == "adamw":
        n = 64 * 1024 * 1024
        p, m, v, g = (torch.randn(n, device=dev) for _ in range(4))
        m.zero_()
        v.zero_()
        pb = torch.empty(n, **bf)
        sc = torch.ones(1, device=dev)
        fn = lambda: C.adamw_flat_(p, m, v, g, pb, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1, sc, None)  # noqa: E731
    elif a.case in ("swiglu", "swiglu_bwd"):
        gu = torch.randn(8192, 2 * 14336, **bf)
        if a.case == "swiglu":
            nbytes = gu.numel() * 2 + gu.numel()  # read gate|up, write the activation
            fn = lambda: C.swiglu_fwd(gu)  # noqa: E731
        else:
            dy = torch.randn(8192, 14336, **bf)
            nbytes = gu.numel() * 2 * 2 + dy.numel() * 2  # read gate|up and dY, write d(gate|up)
            fn = lambda: C.swiglu_bwd(dy, gu)  # noqa: E731
    elif a.case in ("mla_k", "mla_k_bwd"):
        from nano_train_b200.ops.rope import rope_table

        T, h, Dn, Dv, R, lat, S = 8192, 16, 128, 128, 64, 512, 4096
        table = rope_table(S, R, 1e4, dev)
        if a.case == "mla_k":
            kv = torch.randn(T, h, Dn + Dv, **bf)
            kr = torch.randn(T, lat + R, **bf)[:, lat:]
            nbytes = T * h * Dn * 2 + T * R * 2 + T * h * (Dn + R) * 2  # read nope + rope part, write keys
            fn = lambda: C.mla_k_assemble(kv, kr, table, Dn, S)  # noqa: E731
        else:
            dk = torch.randn(T, h, Dn + R, **bf)
            dkv = torch.empty(T, h, Dn + Dv, **bf)
            nbytes = T * h * (Dn + R) * 2 + T * h * Dn * 2 + T * R * 2  # read dK, write nope grads + dk_rope
            fn = lambda: C.mla_k_assemble_bwd(dk, dkv, table, Dn, S)  # noqa: E731
    elif a.case == "ce":
        logits = torch.randn(4096, 32064, **bf)
        labels = torch.randint(0, 32064, (4096,), device=dev)
        fn = lambda: C.ce_stats(logits, labels, 0, -100)  # noqa: E731
    elif a.case in ("router", "router_bwd"):
        logits = torch.randn(16384, 64, **bf)
        cfg = (6, True, 1, 1, True, 1.0)
        idx, w, _, _ = C.router_fwd(logits, *cfg)
        dw = torch.randn_like(w)
        dps = torch.randn(64, device=dev)
        if a.case == "router":
            fn = lambda: C.router_fwd(logits, *cfg)  # noqa: E731
        else:
            fn = lambda: C.router_bwd(logits, idx, dw, dps, *cfg)  # noqa: E731
    elif a.case in ("ep_layer", "zero_step"):
        import torch.distributed as dist

        dist.init_process_group("nccl", rank=0, world_size=1, init_method="tcp://127.0.0.1:29561",
                                device_id=dev)
        if a.case == "ep_layer":
            from nano_train_b200.parallel.ep_fused import EPWorkspace

            T, H, K, E = 8192, 2048, 6, 64
            ws = EPWorkspace(dist.group.WORLD, max_tokens=T, hidden=H, top_k=K, experts_per_rank=E,
                             fp8_payload=False, device=dev)
            tokens = torch.randn(T, H, **bf)
            w, idx = torch.topk(torch.softmax(torch.randn(T, E, device=dev), -1), K, dim=-1)
            wf = w.reshape(-1).contiguous()
            host_cap = int(1.25 * T * K / E) + 1

            def fn():
                dest, slot = ws.dispatch(tokens, idx, w, stochastic=False, seed=0)
                rp = ws.plan(num_experts=E, capacity_factor=1.25, host_cap=host_cap)
                x = ws.gather(rp)
                ws.y(rp.rows).copy_(x)
                ws.publish_y(rp, stochastic=False, seed=0)
                ws.pull_combine(dest, slot, wf, T, save=True)
        else:
            from nano_train_b200.parallel.zero_fused import ZeroSymm

            P = 64 * 2 ** 20
            zs = ZeroSymm(dist.group.WORLD, [P], dev)
            pv, gv = zs.views(0)
            pv.normal_(0, 0.02)
            gv.normal_(0, 1e-3)
            sh = dict(lo=0, hi=P, master=pv.float(), exp_avg=torch.zeros(P, device=dev),
                      exp_avg_sq=torch.zeros(P, device=dev))
            it = [0]

            def fn():
                it[0] += 1
                zs.step([sh], [1e-4], [0.1], [0], step=it[0], betas=(0.9, 0.95), eps=1e-8, inv_dp=1.0,
                        max_norm=1.0)
    else:
        raise SystemExit(f"unknown case {a.case}")
    for _ in range(2 + a.iters):
        fn()
    torch.cuda.synchronize()
    check_status(0)
    print(f"{a.case}: ok")
    if a.time:
        # Each launch is timed on its own between two events, with a 256 MB write before it so the
        # inputs are not served from the 126 MB L2; the median is reported.
        flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)
        ts = []
        for _ in range(a.time):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            ts.append(s.elapsed_time(e))
        ts.sort()
        ms = ts[len(ts) // 2]
        line = f"{a.case}: median {ms * 1e3:.1f} us over {a.time} launches"
        if nbytes:
            line += f", {nbytes / ms / 1e6:.0f} GB/s algorithmic"
        if nflops:
            line += f", {nflops / ms / 1e9:.0f} TFLOP/s algorithmic"
        print(line)


if __name__ == "__main__":
    main()
