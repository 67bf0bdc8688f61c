"""Tensor + sequence parallel (TP=2, gloo, CPU) against the unsharded model.

Both ranks build the same TP=1 model, load its weights into a TP=2
sequence-parallel model with ``load_full_state_dict`` and compare the loss,
then train both for a few steps with ``LMTrainer`` (gradient clipping active)
and compare every parameter shard. This pins the column/row sharding layout,
the all-gather / reduce-scatter autograd, the vocab-parallel cross-entropy,
the summation of replicated-parameter gradients under sequence parallelism
and the TP-aware clipping norm.
"""
import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port


def _cfg(kind, sp):
    from nano_train_b200.config import ModelConfig, _NoOpPrecisionResolver

    common = dict(param_dtype=torch.float32, param_device=torch.device("cpu"), precision_resolver=_NoOpPrecisionResolver(),
                  hidden_size=64, num_layers=2, num_attention_heads=4, intermediate_size=96, vocab_size=64,
                  max_position_embeddings=64, dropout=0.0, tie_word_embeddings=False, sequence_parallel=sp)
    if kind == "llama":
        common.update(num_key_value_heads=2, norm="rmsnorm", position="rope", mlp="swiglu", bias=False,
                      rope_theta=10000.0)
    return ModelConfig(**common)


def _worker(rank, world, port, kind, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from nano_train_b200.config import TPConfig
        from nano_train_b200.models.transformer import TransformerModel
        from nano_train_b200.training import LMTrainer

        torch.manual_seed(0)
        ref = TransformerModel(_cfg(kind, False))
        tp = TransformerModel(_cfg(kind, True), TPConfig(enabled=True, rank=rank, size=world, group=dist.group.WORLD))
        tp.load_full_state_dict({k: v.clone() for k, v in ref.state_dict().items()})
        g = torch.Generator().manual_seed(1)
        ids = torch.randint(0, 64, (2, 16), generator=g)
        labels = torch.randint(0, 64, (2, 16), generator=g)
        labels[0, :3] = -100
        errs = {}
        with torch.no_grad():
            errs["loss0"] = abs(float(ref.forward_loss(ids, labels)) - float(tp.forward_loss(ids, labels)))
        t_ref = LMTrainer(ref, lr=1e-2, max_grad_norm=0.05, micro_batch_size=1)
        t_tp = LMTrainer(tp, lr=1e-2, max_grad_norm=0.05, micro_batch_size=1)
        for _ in range(3):
            l_ref = float(t_ref.train_step(ids, labels))
            l_tp = float(t_tp.train_step(ids, labels))
            errs["loss_step"] = max(errs.get("loss_step", 0.0), abs(l_ref - l_tp))
        errs["gnorm"] = abs(float(t_ref.optimizer.last_grad_norm) - float(t_tp.optimizer.last_grad_norm))
        expect = tp.shard_full_state_dict(ref.state_dict())
        got = tp.state_dict()
        errs["param"] = max(float((expect[k] - got[k]).abs().max()) for k in got if got[k].numel())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("kind", ["llama", "gpt2"])
def test_tp2_sequence_parallel_matches_unsharded(kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, kind, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, exc in results:
        assert exc is None, f"rank {rank}:\n{exc}"
        assert errs["loss0"] < 1e-5, errs
        assert errs["loss_step"] < 1e-4, errs
        assert errs["gnorm"] < 1e-4, errs
        assert errs["param"] < 1e-4, errs
