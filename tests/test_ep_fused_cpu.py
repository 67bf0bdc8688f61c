"""Host-side logic of the fused expert-parallel dispatch / combine (no GPU).

The kernels' data movement is emulated in-process (emulate_exchange / gather /
pull); the send / receive plans are the production code. The result must
equal a single-process MoE over every rank's tokens with the reference's
capacity rule (highest-weight assignments per expert, ties in arrival order).
"""
import dataclasses
import math

import pytest
import torch

from nano_train_b200.models.moe import capacity_select
from nano_train_b200.parallel.ep_fused import (_desc_float_key, capacity_tensor, emulate_exchange, emulate_gather,
                                               emulate_pull, plan_receive, plan_send, rows_bound)


def _shuffle_slots(sp, n, K, gen):
    """The kernel reserves slab rows with atomics: any permutation of a destination block is possible."""
    slot = sp.slot.clone()
    for d in range(n):
        sel = (sp.dest == d).nonzero().flatten()
        slot[sel] = slot[sel][torch.randperm(sel.numel(), generator=gen)]
    slot_tk = torch.empty_like(slot)
    order = sp.tok.long() * K + sp.kslot.long()
    slot_tk[order] = slot
    return dataclasses.replace(sp, slot=slot, slot_tk=slot_tk)


def _expert_fn(x: torch.Tensor, e: int) -> torch.Tensor:
    return x * (e + 1) + 0.5 * e


def _route(T, E, K, gen, tie_grid=None):
    logits = torch.randn(T, E, generator=gen)
    w, idx = torch.topk(torch.softmax(logits, -1), K, dim=-1)
    if tie_grid:
        w = torch.round(w * tie_grid) / tie_grid
    return idx, w


@pytest.mark.parametrize("n,E,K,T,cf,tie,shuffle", [(3, 6, 2, 7, 0.5, None, False), (2, 8, 3, 16, 1.0, None, True),
                                                    (4, 8, 2, 9, 0.4, 4, True), (4, 8, 2, 9, 0.4, 4, False),
                                                    (2, 4, 1, 5, 4.0, None, True)])
def test_fused_plan_matches_capacity_semantics(n, E, K, T, cf, tie, shuffle):
    gen = torch.Generator().manual_seed(n * 100 + E + K + T)
    H = 16
    epr = E // n
    tokens = [torch.randn(T, H, generator=gen) for _ in range(n)]
    routes = [_route(T, E, K, gen, tie) for _ in range(n)]
    P = T * K
    host_cap = max(int(math.ceil(cf * (n * T) * K / float(E))), 1)
    plans = [plan_send(idx, w, epr, n) for idx, w in routes]
    if shuffle:
        plans = [_shuffle_slots(sp, n, K, gen) for sp in plans]
    for sp in plans:  # each destination's block is filled by contiguous slots 0..count-1
        for d in range(n):
            sl = sp.slot[sp.dest == d].sort().values
            assert torch.equal(sl, torch.arange(sl.numel(), dtype=torch.int32))
    exch = emulate_exchange(tokens, plans, epr, P)
    rowmaps, ys, stats = [], [], torch.zeros(2)
    for d in range(n):
        counts, meta, payload = exch[d]
        t_all = torch.tensor(n * T)
        cap = capacity_tensor(t_all, cf, K, E, host_cap)
        rp = plan_receive(counts, meta, epr, cap, rows_bound(n, P, epr, host_cap), K)
        x = emulate_gather(payload, rp)
        y = torch.zeros_like(x)
        for e in range(epr):
            a, b = int(rp.offsets[e]), int(rp.offsets[e + 1])
            y[a:b] = _expert_fn(x[a:b], d * epr + e)
            # padding rows are zero on input
            assert torch.all(x[a + int(rp.kept_counts[e]):b] == 0)
        rowmaps.append(rp.rowmap)
        ys.append(y)
        stats += rp.stats
    # reference: one MoE over the concatenation of every rank's tokens
    X = torch.cat(tokens)
    idx_all = torch.cat([r[0] for r in routes])
    w_all = torch.cat([r[1] for r in routes])
    tok, slot, ex, kept_counts = capacity_select(idx_all, w_all, E, host_cap)
    ref = torch.zeros_like(X)
    for t, s, e in zip(tok.tolist(), slot.tolist(), ex.tolist()):
        ref[t] += w_all[t, s] * _expert_fn(X[t], e)
    for s in range(n):
        out = emulate_pull(T, K, plans[s], rowmaps, ys, routes[s][1].reshape(-1), s, P)
        torch.testing.assert_close(out, ref[s * T:(s + 1) * T], rtol=1e-5, atol=1e-5)
    total = n * T * K
    assert int(stats[1]) == total
    assert int(stats[0]) == total - int(kept_counts.sum())


def test_dispatch_backward_pull_sums_k_copies():
    """The dispatch backward (unit weights over saved positions) sums each token's kept copies."""
    gen = torch.Generator().manual_seed(7)
    n, E, K, T, H = 2, 4, 2, 6, 8
    epr, P = E // n, T * K
    tokens = [torch.randn(T, H, generator=gen) for _ in range(n)]
    routes = [_route(T, E, K, gen) for _ in range(n)]
    plans = [plan_send(i, w, epr, n) for i, w in routes]
    exch = emulate_exchange(tokens, plans, epr, P)
    host_cap = 10 ** 6
    rps = [plan_receive(c, m, epr, torch.tensor(host_cap), rows_bound(n, P, epr, host_cap), K) for c, m, _ in exch]
    gx = [emulate_gather(exch[d][2], rps[d]) for d in range(n)]  # gradient rows = the payload itself
    for s in range(n):
        dx = emulate_pull(T, K, plans[s], [rp.rowmap for rp in rps], gx, None, s, P)
        torch.testing.assert_close(dx, tokens[s] * K)


def test_desc_float_key_orders_descending():
    v = torch.tensor([0.5, -1.0, 2.0, 0.0, -0.25, 1e-30, 3.5])
    key = _desc_float_key(v.view(torch.int32))
    assert torch.equal(torch.argsort(key), torch.argsort(v, descending=True))


def test_region_layout_sections_and_canaries_do_not_overlap():
    from nano_train_b200.parallel.region import CANARY_BYTES, RegionLayout

    lay = RegionLayout(4096)
    sizes = {"a": 100, "b": 0, "c": 4096, "d": 7}
    offs = {k: lay.add(k, v) for k, v in sizes.items()}
    spans = [(o, o + sizes[k]) for k, o in offs.items()] + [(c, c + CANARY_BYTES) for _, c in lay.canaries]
    spans.sort()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert all(o % 256 == 0 for o in offs.values()) and all(c % 256 == 0 for _, c in lay.canaries)
    for (name, c), (k, o) in zip(lay.canaries, offs.items()):
        assert name == k and c >= o + sizes[k]
    assert lay.total == lay.canaries[-1][1] + CANARY_BYTES
