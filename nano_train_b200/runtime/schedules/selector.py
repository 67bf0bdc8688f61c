"""Schedule selection: the 1F1B schedule when the pipeline axis is > 1, else the plain one.
Mirrors the reference's src/runtime/schedules/selector.py."""
from __future__ import annotations

from dataclasses import dataclass

from ..contracts import ScheduleStrategy


@dataclass
class DefaultScheduleSelector:
    non_pipeline_schedule: ScheduleStrategy
    pipeline_schedule: ScheduleStrategy

    def select(self, ctx) -> ScheduleStrategy:
        if ctx.parallel.pipeline_model_parallel_size > 1:
            return self.pipeline_schedule
        return self.non_pipeline_schedule
