"""Fused TP paths vs NCCL + GEMM at the Llama-3-8B-shape sequence-parallel shapes.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/bench_tp_fused.py [--seq 4096]

For each op (forward and backward forms of the column-parallel AG->GEMM and
row-parallel GEMM->RS linears of one layer) it reports, with CUDA events on
the launching stream, max over ranks, median of iterations:
  fused_ms   the single fused kernel
  nccl_ms    NCCL collective + the tcgen05 GEMM (baseline)
  gemm_ms    the GEMM alone on local data (no communication)
  roof_ms    max(FLOPs / measured bf16 peak, NVLink bytes / 770 GB/s)
  frac       roof_ms / fused_ms (fraction of roofline)
and for the reduce-scatter ops also the GEMM + pull kernel (pull_*) and the progressive-pull
single kernel (overlap_*).
"""
import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.ops._ext import check_status, ext  # noqa: E402
from nano_train_b200.ops.linear import gemm  # noqa: E402
from nano_train_b200.parallel import comm  # noqa: E402
from nano_train_b200.parallel.symm import TPCommunicator  # noqa: E402

NVLINK_GBS = 770.0


def peak_tflops():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def timeit(fn, iters, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        dist.barrier()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    t = torch.tensor([ts[len(ts) // 2]], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


EVENTS = ["start", "copy_done", "first_tile", "first_remote_ready", "producer_done", "last_store",
          "reduce_wait_done", "end"]


def trace_report(c, fn, name, rank, n):
    """Runs fn once with per-CTA globaltimer stamps; prints min/median/max (us since the earliest start)."""
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    c.trace = torch.zeros(sms, 8, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    dist.barrier()
    fn()
    torch.cuda.synchronize()
    tr = c.trace.cpu()
    c.trace = None
    t0 = int(tr[:, 0][tr[:, 0] > 0].min())
    out = {"op": name, "rank": rank}
    for e, ev in enumerate(EVENTS):
        col = tr[:, e]
        col = col[col > 0]
        if col.numel() == 0:
            continue
        us = (col - t0).double() / 1e3
        out[ev] = [round(float(us.min()), 1), round(float(us.median()), 1), round(float(us.max()), 1)]
    for r in range(n):
        dist.barrier()
        if r == rank:
            print("TRACE", json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--out", default=None)
    ap.add_argument("--trace", action="store_true", help="print per-CTA timeline of one fused call per op")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    n, rank = dist.get_world_size(), dist.get_rank()
    T, H, I, HQ, HKV, D = args.seq, 4096, 14336, 32, 8, 128
    Tl = T // n
    c = TPCommunicator(dist.group.WORLD, max_local_rows=Tl, max_k=H, max_rs_n=H)
    g = dist.group.WORLD
    peak, peak_kind = peak_tflops()
    qkv_n = (HQ + 2 * HKV) * D // n
    ops_ = [
        ("qkv_ag_fwd", "ag", H, qkv_n, False),
        ("gateup_ag_fwd", "ag", H, 2 * I // n, False),
        ("o_rs_fwd", "rs", HQ * D // n, H, False),
        ("down_rs_fwd", "rs", I // n, H, False),
        ("down_ag_bwd_dgrad", "ag", H, I // n, True),     # dX = AG(dY) . W_row
        ("gateup_rs_bwd_dgrad", "rs", 2 * I // n, H, True),  # dX = RS(dY . W_col)
    ]
    rows = []
    for name, kind, K, N, b_mn in ops_:
        torch.manual_seed(rank)
        if kind == "ag":
            x = torch.randn(Tl, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(K, N, device="cuda", dtype=torch.bfloat16) if b_mn else \
                torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
            xf = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
            fused = lambda: c.all_gather_gemm(x, w, b_mn=b_mn)
            nccl = lambda: gemm(comm.all_gather_dim0(x, g), w, b_mn=b_mn)
            alone = lambda: gemm(xf, w, b_mn=b_mn)
            flops = 2.0 * T * N * K
            nvl_bytes = (n - 1) * Tl * K * 2
        else:
            x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(K, N, device="cuda", dtype=torch.bfloat16) if b_mn else \
                torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
            fused = lambda: c.gemm_reduce_scatter(x, w, b_mn=b_mn)
            pull = lambda: c.gemm_reduce_scatter_pull(x, w, b_mn=b_mn)
            ovl = lambda: c.gemm_reduce_scatter_overlap(x, w, b_mn=b_mn)
            nccl = lambda: comm.reduce_scatter_dim0(gemm(x, w, b_mn=b_mn), g)
            alone = lambda: gemm(x, w, b_mn=b_mn)
            flops = 2.0 * T * N * K
            nvl_bytes = (n - 1) * Tl * N * 2
        fused()
        torch.cuda.synchronize()
        st0 = ext().read_and_clear_status(local)
        tf = timeit(fused, args.iters)
        torch.cuda.synchronize()
        st1 = ext().read_and_clear_status(local)
        if st0 or st1:
            print(f"rank {rank} op {name}: kernel status after first call {st0}, after timing {st1}", flush=True)
        if args.trace:
            trace_report(c, fused, name, rank, n)
        tn = timeit(nccl, args.iters)
        ta = timeit(alone, args.iters)
        roof = max(flops / (peak * 1e12), nvl_bytes / (NVLINK_GBS * 1e9)) * 1e3
        row = dict(op=name, n=n, T=T, K=K, N=N, fused_ms=tf, nccl_ms=tn, gemm_ms=ta, roof_ms=roof,
                   frac=roof / tf, speedup_vs_nccl=tn / tf, peak=f"{peak} TFLOP/s ({peak_kind})")
        if kind == "rs":
            ref = nccl().float()
            rel = ((pull().float() - ref).norm() / ref.norm()).item()
            tp = timeit(pull, args.iters)
            row.update(pull_ms=tp, pull_frac=roof / tp, pull_speedup_vs_nccl=tn / tp, pull_rel_err_vs_nccl=rel)
            rel_o = ((ovl().float() - ref).norm() / ref.norm()).item()
            to = timeit(ovl, args.iters)
            row.update(overlap_ms=to, overlap_frac=roof / to, overlap_speedup_vs_nccl=tn / to,
                       overlap_rel_err_vs_nccl=rel_o)
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    check_status(local)
    c.close()
    if rank == 0 and args.out:
        with open(args.out, "w") as f:
            json.dump(rows, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
