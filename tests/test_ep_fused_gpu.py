"""Fused expert-parallel dispatch / combine (peer-memory kernels) vs the all-to-all path (one rank on one GPU; 2+ GPUs).

Same module, same inputs: forward output, input gradient, router and expert
gradients and the dropped fraction must agree with the NCCL all-to-all
implementation, for a bf16 and an e4m3 (1x128, nearest) payload.
"""
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


def _run(moe, x, fused: bool):
    os.environ["NTB_FUSED_EP"] = "1" if fused else "0"
    moe.zero_grad(set_to_none=True)
    xi = x.detach().clone().requires_grad_(True)
    out = moe(xi)
    g = torch.Generator(device="cuda").manual_seed(99 + dist.get_rank())
    dy = torch.randn(out.shape, device="cuda", dtype=out.dtype, generator=g)
    (out.float() * dy.float()).sum().backward()
    grads = {n: p.grad.detach().clone() for n, p in moe.named_parameters() if p.grad is not None}
    return out.detach(), xi.grad.detach(), grads, moe.last_dropped_fraction, moe.last_path


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from nano_train_b200.models.moe import ExpertParallelMoE
        from nano_train_b200.ops._ext import check_status
        from nano_train_b200.parallel.ep_fused import clear_workspaces

        results = []
        for gran, cf in ((None, 1.0), ("tile_1x128", 0.75)):
            torch.manual_seed(1234 + rank)
            moe = ExpertParallelMoE(256, 128, 8, 2, ep_rank=rank, ep_size=world, ep_group=dist.group.WORLD,
                                    param_dtype=torch.bfloat16, param_device="cuda", n_shared_experts=1,
                                    scoring_func="softmax", capacity_factor=cf, comm_quant_granularity=gran,
                                    comm_quant_rounding="nearest", comm_quant_backend="native")
            # identical router / shared expert on every rank (the reference broadcasts replicated params)
            for name, p in moe.named_parameters():
                if "experts." in name and "shared" not in name:
                    continue
                dist.broadcast(p.data, 0)
            g = torch.Generator(device="cuda").manual_seed(7 + rank)
            x = torch.randn(2, 128, 256, device="cuda", dtype=torch.bfloat16, generator=g)
            for rep in range(2):  # second call reuses the workspace (epochs advance)
                o0, dx0, g0, d0, p0 = _run(moe, x, fused=False)
                o1, dx1, g1, d1, p1 = _run(moe, x, fused=True)
                assert p0 == "all_to_all" and p1 == "fused", (p0, p1)
                errs = {"out": _rel(o1, o0), "dx": _rel(dx1, dx0), "drop": abs(d1 - d0)}
                for k in g0:
                    errs["grad:" + k] = _rel(g1[k], g0[k])
                results.append((str(gran), rep, errs))
        torch.cuda.synchronize()
        check_status(rank)
        from nano_train_b200.parallel.ep_fused import workspaces

        for ws in workspaces():
            bad = ws.check_canaries()
            assert not bad, f"canaries overwritten after {bad}"
        clear_workspaces()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, repr(e) + traceback.format_exc()))


# "one": a one-rank group on one GPU (every peer pointer is this GPU's memory), so the kernels'
# protocol is checked where only one GPU is present; "multi": 2 ranks, or NTB_TEST_WORLD=4 (or 8).
@pytest.mark.parametrize("ranks", ["one", "multi"])
def test_fused_ep_dispatch_combine(ranks, monkeypatch):
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
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, res, exc in results:
        assert exc is None, f"rank {rank}: {exc}"
        for gran, rep, errs in res:
            print(rank, gran, rep, {k: round(v, 5) for k, v in errs.items()})
            assert errs["drop"] < 1e-6, (rank, gran, errs)
            for k, v in errs.items():
                assert v < 3e-2, (rank, gran, rep, k, v)
