"""Point-to-point issue order of the 1F1B schedule, checked with a recording stand-in for
``dist.isend`` / ``dist.irecv``.

NCCL ignores tags: between two ranks it pairs the sends of one direction with the receives of
that direction in the order both sides issued them. gloo honours tags, so a multi-process gloo run
cannot show an order mismatch. Here every stage's schedule runs against a recorder instead, and
for every (source, destination) pair the sender's sequence of messages must equal the receiver's
sequence of posted receives, element by element (tag, element count, dtype). With PP = 2 the
first stage sends both the labels and the activations to the same peer, which is the case that
used to pair an activation receive with a label send.
"""
from types import SimpleNamespace

import pytest
import torch
import torch.nn as nn

import nano_train_b200.parallel.pipeline as pl

B, S, H, V = 2, 6, 8, 11


class _Stage(nn.Module):
    def __init__(self, first, last):
        super().__init__()
        self.is_first_pp_stage, self.is_last_pp_stage = first, last
        self.emb = nn.Embedding(V, H) if first else None
        self.lin = nn.Linear(H, H)
        self.head = nn.Linear(H, V) if last else None

    def forward_stage(self, input_ids=None, hidden_states=None, attention_mask=None):
        x = self.emb(input_ids) if self.is_first_pp_stage else hidden_states
        x = torch.tanh(self.lin(x))
        return self.head(x) if self.is_last_pp_stage else x


class _Req:
    def wait(self):
        return True


def _run_stage(monkeypatch, pp, rank, m, prefetch):
    """Run one stage's whole 1F1B schedule against the recorder; return its message log."""
    log = []

    def isend(t, dst, tag=0, group=None):
        log.append(("send", rank, dst, tag, t.numel(), t.dtype))
        return _Req()

    def irecv(t, src, tag=0, group=None):
        t.zero_()
        log.append(("recv", src, rank, tag, t.numel(), t.dtype))
        return _Req()

    def recv(t, src, tag=0, group=None):
        irecv(t, src, tag, group)

    monkeypatch.setattr(pl.dist, "isend", isend)
    monkeypatch.setattr(pl.dist, "irecv", irecv)
    monkeypatch.setattr(pl.dist, "recv", recv)
    monkeypatch.setattr(pl, "PREFETCH", prefetch)
    torch.manual_seed(0)
    model = _Stage(rank == 0, rank == pp - 1)
    peers = pl.PipelinePeers(prev_rank=rank - 1 if rank > 0 else None, next_rank=rank + 1 if rank + 1 < pp else None,
                             first_stage_rank=0, last_stage_rank=pp - 1)
    state = pl.PipelineStepState()
    ids = torch.randint(0, V, (B * m, S))
    mbs = list(torch.chunk(ids, m, dim=0)) if model.is_first_pp_stage else [None] * m

    def metrics(model, device):
        return torch.zeros(()), torch.zeros(())

    par = SimpleNamespace(pipeline_model_parallel_size=pp, pipeline_model_parallel_rank=rank)
    pl.execute_1f1b_schedule(
        par, m,
        run_forward=lambda i: pl.pipeline_forward_microbatch(i, model, mbs, peers, state, B, S, H, torch.float32,
                                                              torch.device("cpu"), metrics, None, m),
        run_backward=lambda i: pl.pipeline_backward_microbatch(i, model, peers, state, m, 0.01, B, S, H,
                                                                torch.float32, torch.device("cpu")))
    pl.finalize_pipeline_sends(state)
    pl.finalize_pipeline_metrics(state)
    assert isinstance(state.task_loss_sum, float) and isinstance(state.aux_loss_sum, float)
    return log


@pytest.mark.parametrize("pp", [2, 3, 4])
@pytest.mark.parametrize("m", [1, 3, 4])
@pytest.mark.parametrize("prefetch", [False, True])
def test_send_and_receive_issue_order_match_per_peer(monkeypatch, pp, m, prefetch):
    logs = [_run_stage(monkeypatch, pp, r, m, prefetch) for r in range(pp)]
    sends, recvs = {}, {}
    for r, log in enumerate(logs):
        for kind, src, dst, tag, n, dt in log:
            (sends if kind == "send" else recvs).setdefault((src, dst), []).append((tag, n, dt))
    assert set(sends) == set(recvs)
    for pair in sends:
        # NCCL pairs them by position, so position by position they must describe the same message.
        assert sends[pair] == recvs[pair], pair
    # every stage boundary carried one activation and one gradient per micro-batch
    for r in range(pp - 1):
        assert sum(1 for t, _, _ in sends[(r, r + 1)] if 10_000 <= t < 20_000) == m
        assert sum(1 for t, _, _ in sends[(r + 1, r)] if 20_000 <= t < 30_000) == m


def test_two_stage_order_is_label_then_activation(monkeypatch):
    first = [e for e in _run_stage(monkeypatch, 2, 0, 2, False) if e[0] == "send"]
    assert [e[3] for e in first] == [pl.label_tag(0), pl.activation_tag(0), pl.label_tag(1), pl.activation_tag(1)]
