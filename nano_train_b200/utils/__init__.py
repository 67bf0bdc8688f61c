"""Utilities: analytic model report (``dump_model_info``), NVTX ranges, SVG plots, log viewer.

``dump_model_info`` is loaded on first use (the report module is large and pure Python)."""


def __getattr__(name):
    if name == "dump_model_info":
        from .model_info import dump_model_info

        return dump_model_info
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
