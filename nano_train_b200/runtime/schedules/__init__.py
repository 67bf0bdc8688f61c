"""Schedule strategies: plain, non-interleaved 1F1B, and the selector between them."""
from .non_pipeline import NonPipelineSchedule
from .pipeline_1f1b import Pipeline1F1BSchedule, one_f_one_b
from .selector import DefaultScheduleSelector

__all__ = ["DefaultScheduleSelector", "NonPipelineSchedule", "Pipeline1F1BSchedule", "one_f_one_b"]
