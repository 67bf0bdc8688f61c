"""Plain (no pipeline axis) schedule: one forward / backward / optimizer step per batch.

The step itself is supplied as a function (``step_fn``) by the training script's components, so
the schedule is the policy object the engine selects, not the math. Mirrors the reference's
src/runtime/schedules/non_pipeline.py.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from ..contracts import StepContext, StepOutput

StepFn = Callable[[StepContext], StepOutput]


@dataclass
class NonPipelineSchedule:
    """Runs one step without pipeline parallelism through ``step_fn``."""

    step_fn: StepFn

    def run_step(self, step_ctx: StepContext) -> StepOutput:
        return self.step_fn(step_ctx)
