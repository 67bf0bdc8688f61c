"""RuntimeEngine: the fixed training lifecycle.

Lifecycle (the component protocol of the reference, src/runtime/engine.py:20-331): bootstrap ->
model -> train data -> optimizer -> schedule -> checkpoint load -> step loop -> ``on_run_end`` ->
process-group teardown.

Design. There is exactly one step loop (``_drive``). What differs between the training modes is
where batches come from, so that is a strategy object:

* ``_EpochStream`` (no pipeline axis): epochs ``[start, args.epochs)`` over the loader, the sampler
  re-seeded per epoch, batches of an interrupted epoch that were already trained on skipped on
  resume; the end of every epoch is an ``_EpochEnd`` marker in the stream.
* ``_RefillStream`` (first pipeline stage): one endless stream that starts the next pipeline epoch
  when the loader runs dry, so ``max_steps`` alone bounds the run.
* ``_Nothing`` (later pipeline stages): ``None`` batches; activations arrive over the pipeline.

Metrics are kept in a ``_Window`` (sums of the step outputs and their counts). Without a pipeline
the per-step line shows this rank's step and the window is reduced over WORLD at each epoch end;
with a pipeline only the last stage holds the task loss, so every step's window is reduced over
WORLD (float64) before its line is printed. The step line ``step=.. task=.. aux=.. total=..
drop=..`` and the epoch line are a log format other tools parse, kept as the reference prints them.
"""
from __future__ import annotations

import argparse
from dataclasses import dataclass
from typing import Iterator

import torch
import torch.distributed as dist

from ..distributed.failure import fault_point
from ..logging import get_logger
from ..utils.nvtx import nvtx_range
from .context import RuntimeContext, TrainState
from .contracts import RuntimeComponents, StepContext, StepOutput

logger = get_logger(__name__)

STEP_LINE = "step=%d task=%.6f aux=%.6f total=%.6f drop=%.4f"
EPOCH_LINE = "epoch=%d avg_task=%.6f avg_aux=%.6f avg_total=%.6f avg_drop=%.4f"


# ------------------------------------------------------------------------------------------ metrics
@dataclass
class _Window:
    """Running sums of step outputs; means divide by the objective / drop counts."""

    task: float = 0.0
    aux: float = 0.0
    total: float = 0.0
    drop: float = 0.0
    objectives: int = 0
    drops: int = 0

    def add(self, out: StepOutput) -> "_Window":
        self.task += out.task_loss
        self.aux += out.aux_loss
        self.total += out.total_loss
        self.drop += out.drop_fraction
        self.objectives += out.counters.get("objective_count", 1)
        self.drops += out.counters.get("drop_count", 1)
        return self

    def means(self) -> tuple[float, float, float, float]:
        o, d = max(1, self.objectives), max(1, self.drops)
        return self.task / o, self.aux / o, self.total / o, self.drop / d

    def reduced(self, parallel) -> tuple[float, float, float, float]:
        """Means over every rank of the job (sums and counts all-reduced in float64)."""
        if parallel.world_size == 1:
            return self.means()
        v = torch.tensor([self.task, self.aux, self.total, self.drop, self.objectives, self.drops],
                         dtype=torch.float64, device=parallel.device)
        dist.all_reduce(v, op=dist.ReduceOp.SUM)
        t, a, tot, d, o, dc = v.tolist()
        return t / max(1.0, o), a / max(1.0, o), tot / max(1.0, o), d / max(1.0, dc)


# ------------------------------------------------------------------------------------ batch sources
class _EpochEnd:
    def __init__(self, epoch: int):
        self.epoch = epoch


class _EpochStream:
    """Epochs over the loader; resumes inside the interrupted epoch, in that epoch's order."""

    reduce_each_step = False

    def __init__(self, loader, sampler, args, state: TrainState):
        self.loader, self.sampler, self.args, self.state = loader, sampler, args, state

    def __iter__(self) -> Iterator:
        st = self.state
        skip = max(0, st.global_step - st.epoch * len(self.loader)) if st.global_step else 0
        if skip and hasattr(self.sampler, "force_next_seed"):
            self.sampler.force_next_seed(st.data_seed)
        for epoch in range(st.epoch, self.args.epochs):
            st.epoch = epoch
            if hasattr(self.sampler, "set_epoch"):
                self.sampler.set_epoch(epoch)
            for batch in self.loader:
                st.data_seed = getattr(self.sampler, "epoch_seed", None)
                if skip:
                    skip -= 1
                    continue
                yield batch
            yield _EpochEnd(epoch)


class _RefillStream:
    """First pipeline stage: the loader restarted with the next pipeline epoch when it runs dry."""

    reduce_each_step = True

    def __init__(self, loader, sampler, state: TrainState):
        self.loader, self.sampler, self.state = loader, sampler, state

    def _start(self, epoch: int):
        if hasattr(self.sampler, "set_epoch"):
            self.sampler.set_epoch(epoch)
        return iter(self.loader)

    def __iter__(self) -> Iterator:
        st = self.state
        consumed = max(0, st.global_step - st.pipeline_epoch * len(self.loader))
        if consumed and hasattr(self.sampler, "force_next_seed"):
            self.sampler.force_next_seed(st.data_seed)
        it = self._start(st.pipeline_epoch)
        for _ in range(consumed if st.global_step else 0):
            next(it, None)
        while True:
            batch = next(it, _EpochEnd(st.pipeline_epoch))
            if isinstance(batch, _EpochEnd):
                st.pipeline_epoch += 1
                it = self._start(st.pipeline_epoch)
                batch = next(it)
            st.data_seed = getattr(self.sampler, "epoch_seed", None)
            yield batch


class _Nothing:
    """Later pipeline stages train on activations received from the previous stage."""

    reduce_each_step = True

    def __iter__(self) -> Iterator:
        while True:
            yield None


def _batch_source(model, train_data, args, state: TrainState, pipeline: bool):
    if not pipeline:
        return _EpochStream(train_data.loader, train_data.sampler, args, state)
    if getattr(model, "is_first_pp_stage", False):
        return _RefillStream(train_data.loader, train_data.sampler, state)
    return _Nothing()


# --------------------------------------------------------------------------------------- the engine
class RuntimeEngine:
    def run(self, components: RuntimeComponents, args: argparse.Namespace) -> None:
        from ..distributed.debug import enable_from_env

        enable_from_env()  # NTB_CHECK_COLLECTIVES=1: every collective is order-checked across its group
        ctx = components.bootstrap.build_context(args)
        _announce(ctx)
        model = components.model_provider.build_model(ctx)
        train_data = components.data_provider.build_train_data(ctx)
        optimizer_state = components.optimizer_runtime.initialize(model, ctx)
        schedule = components.schedule_selector.select(ctx)
        resume = components.checkpoint_manager.load(model=model, optimizer_state=optimizer_state, ctx=ctx)
        model.train()
        state = TrainState(global_step=resume.start_global_step, epoch=resume.start_epoch,
                           pipeline_epoch=resume.pipeline_epoch, data_seed=getattr(resume, "data_seed", None))
        heartbeat = None
        try:
            heartbeat = _start_heartbeat(args, ctx)
            source = _batch_source(model, train_data, args, state, ctx.parallel.pipeline_model_parallel_size > 1)
            self._drive(source, schedule=schedule, model=model, optimizer_state=optimizer_state, ctx=ctx,
                        state=state, components=components, args=args)
            components.checkpoint_manager.on_run_end(model=model, optimizer_state=optimizer_state, state=state,
                                                     ctx=ctx)
            if ctx.parallel.rank == 0:
                logger.info("Training completed")
            if heartbeat is not None:
                heartbeat.stop(done=True)
                heartbeat = None
        finally:
            if heartbeat is not None:
                heartbeat.stop()
            _teardown()

    def _drive(self, source, *, schedule, model, optimizer_state, ctx: RuntimeContext, state: TrainState,
               components: RuntimeComponents, args) -> None:
        """The step loop: one schedule step per batch while ``global_step < max_steps``. A batch is
        only drawn from the source when a step will run on it."""
        parallel = ctx.parallel
        every = int(getattr(args, "log_every", 0))
        window = _Window()

        def close_epoch(epoch: int) -> None:
            nonlocal window
            if window.objectives:
                means = window.reduced(parallel)
                if parallel.rank == 0:
                    logger.info(EPOCH_LINE, epoch + 1, *means)
            window = _Window()

        it = iter(source)
        while state.global_step < args.max_steps:
            item = next(it, _DONE)
            if item is _DONE:
                break
            if isinstance(item, _EpochEnd):
                close_epoch(item.epoch)
                continue
            with nvtx_range(f"step {state.global_step}"):
                out = schedule.run_step(StepContext(model=model, batch=item, optimizer_state=optimizer_state,
                                                    runtime_context=ctx, train_state=state))
            step = _Window().add(out)
            if source.reduce_each_step:
                means = step.reduced(parallel)
            else:
                means = step.means()
                window.add(out)
            components.checkpoint_manager.on_step_end(model=model, optimizer_state=optimizer_state, state=state,
                                                      ctx=ctx)
            if parallel.rank == 0 and every > 0 and state.global_step % every == 0:
                logger.info(STEP_LINE, state.global_step, *means)
            fault_point("step_end", state.global_step, parallel.rank)
            state.global_step += 1
        if not source.reduce_each_step:
            close_epoch(state.epoch)  # an epoch cut short by max_steps still gets its summary


_DONE = object()


def _start_heartbeat(args, ctx: RuntimeContext):
    """``--heartbeat-timeout-s T`` (> 0, more than one rank): every rank beats into the process group's
    store, and a rank whose peer has been silent for T seconds ends its process with a message naming
    that peer, instead of waiting in a collective for the process-group timeout."""
    t = float(getattr(args, "heartbeat_timeout_s", 0.0) or 0.0)
    if t <= 0 or ctx.parallel.world_size <= 1 or not dist.is_initialized():
        return None
    from ..distributed.failure import fail_fast_monitor

    return fail_fast_monitor(t)


def _announce(ctx: RuntimeContext) -> None:
    """One line with the run's mode and parallel layout (rank 0)."""
    p = ctx.parallel
    if p.rank != 0:
        return
    backend = dist.get_backend() if p.world_size > 1 and dist.is_initialized() else "none"
    logger.info("runtime: mode=%s world=%d tp=%d pp=%d ep=%d dp=%d edp=%d cp=%d backend=%s device=%s", ctx.mode,
                p.world_size, p.tensor_model_parallel_size, p.pipeline_model_parallel_size,
                p.expert_model_parallel_size, p.data_parallel_size, p.expert_data_parallel_size,
                p.context_parallel_size, backend, p.device)


def _teardown() -> None:
    """Release the peer-memory communicators before the process group they were built on."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    try:
        from ..parallel.fused import clear_communicators

        clear_communicators()
    except Exception:  # pragma: no cover - best effort teardown
        pass
    dist.destroy_process_group()


__all__ = ["RuntimeEngine", "STEP_LINE", "EPOCH_LINE"]
