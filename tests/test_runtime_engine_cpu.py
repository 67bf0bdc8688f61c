"""RuntimeEngine lifecycle with fake components (single process, no collectives).

Behaviour follows the reference's tests test_runtime_engine.py, test_runtime_bootstrap_contract.py and
test_runtime_checkpoint_lifecycle.py: the bootstrap builds the context before any other component, the
checkpoint is loaded before the first step and its resume state decides where the loop starts, the
plain loop runs epochs over the loader and the pipeline loop refills the first stage's data at the end of
an epoch; ``on_run_end`` runs once."""
import argparse
from types import SimpleNamespace

import pytest
import torch

from nano_train_b200.runtime.context import RunConfig, RuntimeContext
from nano_train_b200.runtime.contracts import (OptimizerState, ParamShardInfo, ResumeState, RuntimeComponents,
                                               StepOutput, TrainDataBundle)
from nano_train_b200.runtime.engine import RuntimeEngine
from nano_train_b200.runtime.schedules import DefaultScheduleSelector


class _Sampler:
    def __init__(self, log):
        self.log = log
        self.epoch_seed = None

    def set_epoch(self, e):
        self.log.append(("set_epoch", e))
        self.epoch_seed = 1000 + e


def _components(log, *, pp=1, n_batches=3, resume=ResumeState(), first_stage=True):
    parallel = SimpleNamespace(rank=0, world_size=1, device=torch.device("cpu"), tensor_model_parallel_size=1,
                               pipeline_model_parallel_size=pp, expert_model_parallel_size=1, data_parallel_size=1,
                               expert_data_parallel_size=1, context_parallel_size=1)

    class Bootstrap:
        def build_context(self, args):
            log.append(("bootstrap",))
            return RuntimeContext(parallel=parallel, mode="pipeline" if pp > 1 else "plain",
                                  run_config=RunConfig(args=args, pp_layer_splits=None))

    class Models:
        def build_model(self, ctx):
            assert log[-1] == ("bootstrap",)
            log.append(("model",))
            m = torch.nn.Linear(2, 2)
            m.is_first_pp_stage = first_stage
            return m

    class Data:
        def build_train_data(self, ctx):
            log.append(("data",))
            return TrainDataBundle(loader=[{"i": torch.tensor(i)} for i in range(n_batches)], sampler=_Sampler(log))

    class Opt:
        def initialize(self, model, ctx):
            log.append(("optimizer",))
            return OptimizerState(optimizer=None, shard_info=ParamShardInfo(set(), set()))

    def step(name):
        def run(sc):
            b = None if sc.batch is None else int(sc.batch["i"])
            log.append((name, sc.train_state.global_step, sc.train_state.epoch, b))
            return StepOutput(task_loss=1.0, aux_loss=0.0, total_loss=1.0, drop_fraction=0.0)
        return SimpleNamespace(run_step=run)

    class Ckpt:
        def load(self, *, model, optimizer_state, ctx):
            log.append(("load",))
            return resume

        def on_step_end(self, *, model, optimizer_state, state, ctx):
            log.append(("step_end", state.global_step))

        def on_run_end(self, *, model, optimizer_state, state, ctx):
            log.append(("run_end", state.global_step))

    return RuntimeComponents(bootstrap=Bootstrap(), model_provider=Models(), data_provider=Data(),
                             optimizer_runtime=Opt(),
                             schedule_selector=DefaultScheduleSelector(non_pipeline_schedule=step("plain"),
                                                                       pipeline_schedule=step("pipe")),
                             checkpoint_manager=Ckpt())


def _args(**kw):
    return argparse.Namespace(**{"epochs": 2, "max_steps": 100, "log_every": 0, **kw})


def test_plain_mode_lifecycle_order_and_epochs():
    log = []
    RuntimeEngine().run(_components(log), _args())
    assert log[:5] == [("bootstrap",), ("model",), ("data",), ("optimizer",), ("load",)]
    steps = [e for e in log if e[0] == "plain"]
    assert steps == [("plain", s, s // 3, s % 3) for s in range(6)]  # two epochs of three batches
    assert [e for e in log if e[0] == "set_epoch"] == [("set_epoch", 0), ("set_epoch", 1)]
    assert log[-1] == ("run_end", 6) and sum(1 for e in log if e[0] == "run_end") == 1
    assert log.index(("load",)) < log.index(("plain", 0, 0, 0))


def test_plain_mode_stops_at_max_steps():
    log = []
    RuntimeEngine().run(_components(log), _args(max_steps=4))
    assert [e[1] for e in log if e[0] == "plain"] == [0, 1, 2, 3]
    assert log[-1] == ("run_end", 4)


def test_resume_state_is_used_before_the_first_step():
    log = []
    RuntimeEngine().run(_components(log, resume=ResumeState(start_global_step=4, start_epoch=1)), _args())
    # step 4 is the second batch of epoch 1: the first batch of that epoch was trained before the checkpoint
    assert [e for e in log if e[0] == "plain"] == [("plain", 4, 1, 1), ("plain", 5, 1, 2)]
    assert ("set_epoch", 0) not in log


def test_pipeline_mode_refills_the_first_stage_across_epochs():
    log = []
    RuntimeEngine().run(_components(log, pp=2, n_batches=2), _args(max_steps=5))
    assert [(e[1], e[3]) for e in log if e[0] == "pipe"] == [(0, 0), (1, 1), (2, 0), (3, 1), (4, 0)]
    assert [e for e in log if e[0] == "set_epoch"] == [("set_epoch", 0), ("set_epoch", 1), ("set_epoch", 2)]
    assert log[-1] == ("run_end", 5)


def test_pipeline_mode_later_stages_get_no_batch():
    log = []
    RuntimeEngine().run(_components(log, pp=2, first_stage=False), _args(max_steps=3))
    assert [e[3] for e in log if e[0] == "pipe"] == [None, None, None]
    assert not any(e[0] == "set_epoch" for e in log)


def test_pipeline_resume_skips_consumed_batches_of_the_epoch():
    log = []
    comps = _components(log, pp=2, n_batches=3, resume=ResumeState(start_global_step=4, pipeline_epoch=1))
    RuntimeEngine().run(comps, _args(max_steps=6))
    assert [(e[1], e[3]) for e in log if e[0] == "pipe"] == [(4, 1), (5, 2)]


def test_a_failing_component_is_not_swallowed():
    log = []
    comps = _components(log)

    def boom(ctx):
        raise RuntimeError("model provider failed")
    comps.model_provider.build_model = boom
    with pytest.raises(RuntimeError, match="model provider failed"):
        RuntimeEngine().run(comps, _args())
    assert ("data",) not in log
