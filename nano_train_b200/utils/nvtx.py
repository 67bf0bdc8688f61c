"""NVTX ranges around training phases, for timeline profilers (off unless NTB_NVTX=1).

The ranges cost nothing when off; when on they mark h2d / forward / backward /
optimizer phases (and the engine's per-step phases) so a timeline shows which
kernels belong to which phase.
"""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("NTB_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx_range(name: str):
    if ENABLED and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
