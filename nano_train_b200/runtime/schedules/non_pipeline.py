from . import DefaultScheduleSelector, NonPipelineSchedule, Pipeline1F1BSchedule  # noqa: F401
