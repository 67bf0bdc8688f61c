"""Schedule strategies (reference: src/runtime/schedules/*.py)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from ..contracts import ScheduleStrategy, StepContext, StepOutput

StepFn = Callable[[StepContext], StepOutput]


@dataclass
class NonPipelineSchedule:
    """Runs one step without pipeline parallelism through ``step_fn``."""

    step_fn: StepFn

    def run_step(self, step_ctx: StepContext) -> StepOutput:
        return self.step_fn(step_ctx)


@dataclass
class Pipeline1F1BSchedule:
    """Runs one non-interleaved 1F1B pipeline step through ``step_fn``."""

    step_fn: StepFn

    def run_step(self, step_ctx: StepContext) -> StepOutput:
        return self.step_fn(step_ctx)


@dataclass
class DefaultScheduleSelector:
    """Pipeline schedule when the pipeline axis is > 1, else the plain schedule."""

    non_pipeline_schedule: ScheduleStrategy
    pipeline_schedule: ScheduleStrategy

    def select(self, ctx) -> ScheduleStrategy:
        if ctx.parallel.pipeline_model_parallel_size > 1:
            return self.pipeline_schedule
        return self.non_pipeline_schedule


__all__ = ["DefaultScheduleSelector", "NonPipelineSchedule", "Pipeline1F1BSchedule"]
