"""Runtime context objects (reference: src/runtime/context.py:16-40)."""
from __future__ import annotations

import argparse
from dataclasses import dataclass
from typing import TYPE_CHECKING, Any, Optional

if TYPE_CHECKING:
    from .contracts import PrecisionConfig


@dataclass
class RunConfig:
    """Resolved run configuration: parsed args, pipeline layer splits, precision."""

    args: argparse.Namespace
    pp_layer_splits: Optional[tuple[int, ...]]
    precision_config: Optional["PrecisionConfig"] = None


@dataclass
class RuntimeContext:
    """Topology of this process, run mode, and run configuration."""

    parallel: Any
    mode: str
    run_config: RunConfig


@dataclass
class TrainState:
    """Train-loop counters."""

    global_step: int = 0
    epoch: int = 0
    pipeline_epoch: int = 0
    data_seed: Optional[int] = None  # shuffle seed of the current epoch (EpochSeedRandomSampler)
