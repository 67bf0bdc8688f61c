"""Runtime package: the engine, its component contracts, context and precision plumbing.

Names are exported lazily (PEP 562 ``__getattr__``): ``from nano_train_b200.runtime import
RuntimeEngine`` imports only the engine's module, so the lightweight contracts stay importable
without pulling in the models, the CUDA extension or torch.distributed set-up. The exported names
are those of the reference's runtime package (src/runtime/__init__.py:13-82); the table below
says which of this framework's modules defines each.
"""
from __future__ import annotations

import importlib

_CONTRACTS = ("CheckpointManager", "DataProvider", "ModelProvider", "OptimizerRuntime", "OptimizerState",
              "ModulePrecisionAssignment", "ModulePrecisionPolicy", "ModelPrecisionPlan", "LowBitKernelSpec",
              "MasterOwnershipMode", "PrecisionConfig", "PrecisionRuntimeState", "ResumeState", "RuntimeBootstrap",
              "RuntimeComponents", "ScheduleSelector", "ScheduleStrategy", "StepContext", "StepOutput",
              "TrainDataBundle", "ParamShardInfo")

# name -> module (relative to this package's parent) that defines it
_EXPORTS: dict[str, str] = {
    **{n: ".runtime.contracts" for n in _CONTRACTS},
    "RunConfig": ".runtime.context",
    "RuntimeContext": ".runtime.context",
    "TrainState": ".runtime.context",
    "NoOpCheckpointManager": ".runtime.checkpoint",
    "RuntimeEngine": ".runtime.engine",
    "MixedPrecisionController": ".precision.mixed_precision",
    "build_module_precision_resolver": ".precision.mixed_precision",
    "dtype_alias_to_torch": ".precision.mixed_precision",
    "finalize_module_precision_resolver": ".precision.mixed_precision",
    "refresh_persistent_lowbit_params": ".precision.mixed_precision",
    "add_mixed_precision_args": ".precision.precision_args",
    "normalize_and_resolve_precision": ".precision.precision_args",
    "materialize_optimizer_owned_masters": ".precision.master_store",
}

__all__ = sorted(_EXPORTS)


def __getattr__(name: str):
    mod = _EXPORTS.get(name)
    if mod is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(importlib.import_module(mod, __package__.rpartition(".")[0]), name)
    globals()[name] = value  # later lookups skip __getattr__
    return value


def __dir__():
    return sorted(set(globals()) | set(_EXPORTS))
