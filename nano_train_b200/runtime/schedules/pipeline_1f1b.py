"""Non-interleaved 1F1B pipeline schedule.

``one_f_one_b(pp, rank, m)`` is the order in which a stage runs its forward ("F") and backward
("B") micro-batch steps: ``min(pp - rank - 1, m)`` warm-up forwards, then alternating one
forward / one backward, then the remaining backwards. A stage therefore holds at most
``min(pp - rank, m)`` micro-batches of activations. ``parallel/pipeline.py`` executes it with the
send / receive plumbing; ``Pipeline1F1BSchedule`` is the policy object the engine selects, with
the step supplied as ``step_fn``. Mirrors the reference's src/runtime/schedules/pipeline_1f1b.py.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from ..contracts import StepContext, StepOutput

StepFn = Callable[[StepContext], StepOutput]


def one_f_one_b(pp: int, rank: int, m: int) -> list[tuple[str, int]]:
    warm = max(0, min(pp - rank - 1, m))
    order = [("F", i) for i in range(warm)]
    for i in range(m - warm):
        order += [("F", warm + i), ("B", i)]
    order += [("B", m - warm + i) for i in range(warm)]
    return order


@dataclass
class Pipeline1F1BSchedule:
    """Runs one non-interleaved 1F1B pipeline step through ``step_fn``."""

    step_fn: StepFn

    def run_step(self, step_ctx: StepContext) -> StepOutput:
        return self.step_fn(step_ctx)
