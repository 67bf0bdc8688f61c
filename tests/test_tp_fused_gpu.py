"""Fused all-gather->GEMM and GEMM->reduce-scatter kernels vs NCCL + fp32 math (one rank on one GPU; 2+ GPUs)."""
import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from nano_train_b200.ops._ext import check_status
        from nano_train_b200.parallel.symm import TPCommunicator

        c = TPCommunicator(dist.group.WORLD, max_local_rows=256, max_k=512, max_rs_n=512)
        errs = []
        for it in range(3):
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            T_local, K, N = 256, 512, 384
            x = torch.randn(T_local, K, device="cuda", dtype=torch.bfloat16, generator=g)
            w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(7 + it))
            y, full = c.all_gather_gemm(x, w)
            ref_full = torch.empty(world * T_local, K, device="cuda", dtype=torch.bfloat16)
            dist.all_gather_into_tensor(ref_full, x)
            errs.append(("ag_full", float((full.float() - ref_full.float()).abs().max())))
            errs.append(("ag", _rel(y, ref_full.float() @ w.float().t())))
            # dgrad form: B stored [K_out, N] (b_mn)
            wt = torch.randn(K, 256, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(11 + it))
            y2, _ = c.all_gather_gemm(x, wt, b_mn=True)
            errs.append(("ag_bmn", _rel(y2, ref_full.float() @ wt.float())))
            # GEMM + reduce-scatter
            xr = torch.randn(world * T_local, K, device="cuda", dtype=torch.bfloat16, generator=g)
            wr = torch.randn(512, K, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(13 + it))
            out = c.gemm_reduce_scatter(xr, wr)
            part = (xr.float() @ wr.float().t()).contiguous()
            ref = torch.empty(T_local, 512, device="cuda", dtype=torch.float32)
            dist.reduce_scatter_tensor(ref, part)
            errs.append(("rs", _rel(out, ref)))
            errs.append(("rs_pull", _rel(c.gemm_reduce_scatter_pull(xr, wr), ref)))
            errs.append(("rs_overlap", _rel(c.gemm_reduce_scatter_overlap(xr, wr), ref)))
            wrt = torch.randn(K, 512, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(17 + it))
            out2 = c.gemm_reduce_scatter(xr, wrt, b_mn=True)
            part2 = (xr.float() @ wrt.float()).contiguous()
            ref2 = torch.empty(T_local, 512, device="cuda", dtype=torch.float32)
            dist.reduce_scatter_tensor(ref2, part2)
            errs.append(("rs_bmn", _rel(out2, ref2)))
            errs.append(("rs_overlap_bmn", _rel(c.gemm_reduce_scatter_overlap(xr, wrt, b_mn=True), ref2)))
        torch.cuda.synchronize()
        check_status(rank)
        bad = c.check_canaries()
        assert not bad, f"canaries overwritten after {bad}"
        c.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, None, repr(e)))


# "one": a one-rank group on one GPU (every peer pointer is this GPU's memory), so the kernels'
# protocol is checked where only one GPU is present; "multi": 2 ranks, or NTB_TEST_WORLD=4 (or 8).
@pytest.mark.parametrize("ranks", ["one", "multi"])
def test_fused_ag_gemm_and_gemm_rs(ranks, monkeypatch):
    if ranks == "multi" and torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if ranks == "one":
        monkeypatch.setenv("NTB_FUSED_ONE_RANK", "1")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    world = 1 if ranks == "one" else max(2, min(int(os.environ.get("NTB_TEST_WORLD", "2")),
                                                torch.cuda.device_count()))
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, exc in results:
        assert exc is None, f"rank {rank}: {exc}"
        for name, e in errs:
            if name == "ag_full":
                assert e == 0.0, (rank, name, e)
            else:
                assert e < 1e-2, (rank, name, e)
