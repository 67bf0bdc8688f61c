"""Router, capacity selection and MoE layers (CPU), plus EP=2 over gloo.

Oracles are plain Python loops over tokens/experts with the reference's
semantics: group-limited top-k, weights renormalised (sigmoid) or
re-softmaxed (softmax) then scaled, capacity ceil(cf * T * K / E) keeping the
highest-weight assignments, output[token] += w * expert(x), shared experts
averaged.
"""
import datetime
import math
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from conftest import free_port
from nano_train_b200.models.moe import ExpertParallelMoE, LocalRoutedMoE, TopKRouter, capacity_select


@pytest.mark.parametrize("scoring", ["sigmoid", "softmax"])
def test_router_group_limited_topk(scoring):
    torch.manual_seed(0)
    E, K, G, TG = 16, 4, 4, 2
    r = TopKRouter(32, E, K, scoring_func=scoring, n_group=G, topk_group=TG, routed_scaling_factor=2.5)
    x = torch.randn(50, 32)
    out = r(x)
    logits = x @ r.router.weight.t()
    scores = (torch.sigmoid(logits) if scoring == "sigmoid" else torch.softmax(logits, -1)).detach()
    for t in range(50):
        gmax = scores[t].view(G, E // G).max(-1).values
        allowed_groups = set(torch.topk(gmax, TG).indices.tolist())
        chosen = out.topk_indices[t].tolist()
        assert all(e // (E // G) in allowed_groups for e in chosen)
        masked = torch.tensor([float(scores[t, e]) if e // (E // G) in allowed_groups else -1.0 for e in range(E)])
        assert set(chosen) == set(torch.topk(masked, K).indices.tolist())
        raw = scores[t, out.topk_indices[t]]
        expect = raw / raw.sum() if scoring == "sigmoid" else torch.softmax(raw, -1)
        torch.testing.assert_close(out.topk_weights[t], 2.5 * expect, rtol=1e-5, atol=1e-6)
    # aux loss: N * sum_i f_i * P_i (P from normalised scores for sigmoid)
    normed = scores / scores.sum(-1, keepdim=True) if scoring == "sigmoid" else scores
    f = torch.bincount(out.topk_indices.reshape(-1), minlength=E).float() / (50 * K)
    torch.testing.assert_close(out.aux_loss, (f * normed.mean(0)).sum() * E, rtol=1e-5, atol=1e-6)


def test_capacity_select_keeps_highest_weights():
    torch.manual_seed(1)
    T, K, E, cap = 40, 2, 5, 7
    idx = torch.stack([torch.randperm(E)[:K] for _ in range(T)])
    w = torch.rand(T, K)
    tok, slot, exp, counts = capacity_select(idx, w, E, cap)
    kept = set(zip(tok.tolist(), slot.tolist()))
    for e in range(E):
        cand = [(float(w[t, s]), t, s) for t in range(T) for s in range(K) if idx[t, s] == e]
        cand.sort(key=lambda c: -c[0])
        expect = {(t, s) for _, t, s in cand[:cap]}
        got = {(t, s) for (t, s) in kept if idx[t, s] == e}
        assert got == expect
        assert counts[e] == len(expect)
    assert torch.all(exp[:-1] <= exp[1:])  # grouped by expert


def _moe_oracle(moe, x):
    tokens = x.reshape(-1, x.shape[-1])
    ro = moe.router(tokens)
    T, K = ro.topk_indices.shape
    cap = max(int(math.ceil(moe.capacity_factor * T * K / moe.num_experts)), 1)
    out = torch.zeros_like(tokens)
    for e in range(moe.num_experts):
        w = ro.topk_weights.detach()
        cand = [(float(w[t, s]), t, s) for t in range(T) for s in range(K) if ro.topk_indices[t, s] == e]
        cand.sort(key=lambda c: -c[0])
        for _, t, s in cand[:cap]:
            ex = moe.experts[e]
            h = F.silu(tokens[t] @ ex.gate_proj.weight.t()) * (tokens[t] @ ex.up_proj.weight.t())
            out[t] += ro.topk_weights[t, s] * (h @ ex.down_proj.weight.t())
    if len(moe.shared_experts):
        out = out + sum(se(tokens) for se in moe.shared_experts) / len(moe.shared_experts)
    return out.view_as(x)


@pytest.mark.parametrize("cf", [0.5, 4.0])
def test_local_moe_matches_loop_oracle(cf):
    torch.manual_seed(2)
    moe = LocalRoutedMoE(16, 24, 8, 2, n_shared_experts=2, n_group=4, topk_group=2, capacity_factor=cf)
    x = torch.randn(2, 6, 16)
    y = moe(x)
    torch.testing.assert_close(y, _moe_oracle(moe, x), rtol=1e-5, atol=1e-5)
    assert (moe.last_dropped_fraction > 0) == (cf < 1.0)
    y.sum().backward()
    assert moe.router.router.weight.grad is not None


def _ep_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        torch.manual_seed(3)
        local = LocalRoutedMoE(16, 24, 8, 2, n_shared_experts=1, capacity_factor=0.75)
        ep = ExpertParallelMoE(16, 24, 8, 2, ep_rank=rank, ep_size=world, ep_group=dist.group.WORLD,
                               n_shared_experts=1, capacity_factor=0.75)
        sd = local.state_dict()
        mine = {}
        for k, v in sd.items():
            if k.startswith("experts."):
                e = int(k.split(".")[1])
                if e // 4 == rank:
                    mine[k.replace(f"experts.{e}.", f"experts.{e - 4 * rank}.", 1)] = v
            else:
                mine[k] = v
        ep.load_state_dict(mine)
        g = torch.Generator().manual_seed(4)
        xs = [torch.randn(2, 5, 16, generator=g) for _ in range(world)]
        full = torch.cat(xs, 0)
        ref = local(full)[rank * 2:(rank + 1) * 2]
        x = xs[rank].clone().requires_grad_(True)
        y = ep(x)
        err = float((y - ref).abs().max())
        y.square().sum().backward()
        ok_grad = x.grad is not None and bool(torch.isfinite(x.grad).all())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err, ok_grad, None))
    except Exception:
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


def test_expert_parallel_matches_local_over_concatenated_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err, ok_grad, exc in res:
        assert exc is None, f"rank {rank}:\n{exc}"
        assert err < 1e-5, (rank, err)
        assert ok_grad
