"""Runtime component contracts and shared value objects.

The protocol names, dataclass names and fields are the reference's public
runtime API (src/runtime/contracts.py:25-352) so that component
implementations written for it plug into this engine unchanged.
"""
from __future__ import annotations

import argparse
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Iterable, Literal, Optional, Protocol, Set

import torch

from .context import RuntimeContext, TrainState

if TYPE_CHECKING:  # pragma: no cover
    from ..precision.backends import LowBitBackend

PrecisionMode = Literal["fp32", "bf16", "fp16", "fp8", "fp4"]
PrecisionDType = Literal["fp32", "bf16", "fp16"]
LowBitBackendName = Literal["transformer_engine", "emulated", "native"]
FP8Format = Literal["e4m3", "hybrid"]
FP8AmaxComputeAlgo = Literal["most_recent", "max"]
ModulePatternType = Literal["regex", "glob"]
LowBitComputeMode = Literal["fp8", "fp4"]
PersistentLowBitMode = Literal["off", "fp8", "fp4"]
PersistentScaleGranularity = Literal["per_tensor", "per_channel"]
FP4PersistentFormat = Literal["nf4"]
LowBitCapableModuleType = Literal["linear", "column_parallel_linear", "row_parallel_linear"]
MasterOwnershipMode = Literal["module", "optimizer"]
QuantGranularity = Literal["tensor", "channel", "tile_1x128", "block_128x128"]
RoundingMode = Literal["nearest", "stochastic"]
PrecisionRecipeName = Literal["default", "deepseek_v3"]


@dataclass
class ParamShardInfo:
    """Parameter ids split by sharding domain (tensor-parallel vs expert-parallel)."""

    tensor_model_parallel_sharded_param_ids: Set[int]
    expert_model_parallel_sharded_param_ids: Set[int]


@dataclass(frozen=True)
class DeepSeekV3PrecisionRecipe:
    """DeepSeek-V3 fp8 recipe: 1x128 activation tiles, 128x128 weight blocks,
    stochastic rounding, fp8 MoE payloads, and high-precision exceptions."""

    activation_quant_granularity: QuantGranularity = "tile_1x128"
    weight_quant_granularity: QuantGranularity = "block_128x128"
    rounding_mode: RoundingMode = "stochastic"
    comm_quant_enabled: bool = True
    comm_quant_granularity: QuantGranularity = "block_128x128"
    high_precision_module_patterns: tuple[str, ...] = ()
    high_precision_grad_patterns: tuple[str, ...] = ()


@dataclass(frozen=True)
class LowBitKernelSpec:
    """Shape and quantisation metadata a low-bit backend needs for one linear layer."""

    module_type: LowBitCapableModuleType
    in_features: int
    out_features: int
    has_bias: bool
    activation_quant_granularity: QuantGranularity = "tensor"
    weight_quant_granularity: QuantGranularity = "tensor"
    rounding_mode: RoundingMode = "nearest"


@dataclass
class ModulePrecisionPolicy:
    """Module-pattern policy for low-bit compute, persistent low-bit params and dtype rules."""

    pattern_type: ModulePatternType = "regex"
    compute_lowbit_mode: Optional[LowBitComputeMode] = None
    compute_lowbit_include: tuple[str, ...] = ()
    compute_lowbit_exclude: tuple[str, ...] = ()
    persistent_lowbit_mode: PersistentLowBitMode = "off"
    persistent_lowbit_include: tuple[str, ...] = ()
    persistent_lowbit_exclude: tuple[str, ...] = ()
    persistent_scale_granularity: PersistentScaleGranularity = "per_channel"
    fp4_persistent_format: FP4PersistentFormat = "nf4"
    module_compute_dtype_rules: tuple[str, ...] = ()


@dataclass
class ModulePrecisionAssignment:
    """Resolved precision of one concrete module instance."""

    module_name: str
    module_type: str
    compute_lowbit_mode: Optional[LowBitComputeMode]
    persistent_lowbit_mode: PersistentLowBitMode
    persistent_scale_granularity: PersistentScaleGranularity
    fp4_persistent_format: FP4PersistentFormat
    compute_dtype_override: Optional[PrecisionDType] = None
    master_ownership: MasterOwnershipMode = "module"


@dataclass
class ModelPrecisionPlan:
    assignments: dict[str, ModulePrecisionAssignment] = field(default_factory=dict)
    compute_lowbit_module_count: int = 0
    persistent_lowbit_module_count: int = 0


@dataclass(frozen=True)
class ModulePrecisionInitState:
    assignment: ModulePrecisionAssignment
    lowbit_backend: Optional["LowBitBackend"] = None
    lowbit_capable_type: Optional[LowBitCapableModuleType] = None
    master_ownership_mode: MasterOwnershipMode = "module"


@dataclass(frozen=True)
class ModulePrecisionSummary:
    parameterized_module_count: int = 0
    lowbit_capable_module_count: int = 0
    compute_lowbit_module_count: int = 0
    persistent_lowbit_module_count: int = 0
    high_precision_exception_module_count: int = 0


class ModulePrecisionResolver(Protocol):
    def resolve_module_init_state(self, *, module_path: str, module_type: str,
                                  lowbit_capable_type: Optional[LowBitCapableModuleType],
                                  kernel_spec: Optional[LowBitKernelSpec] = None) -> ModulePrecisionInitState:
        ...

    def finalize(self) -> ModulePrecisionSummary:
        ...

    def deepseek_v3_recipe(self) -> Optional[DeepSeekV3PrecisionRecipe]:
        ...


@dataclass
class PrecisionConfig:
    """Resolved precision settings of a run."""

    mode: PrecisionMode = "fp32"
    params_dtype: PrecisionDType = "fp32"
    main_params_dtype: PrecisionDType = "fp32"
    main_grads_dtype: PrecisionDType = "fp32"
    exp_avg_dtype: PrecisionDType = "fp32"
    exp_avg_sq_dtype: PrecisionDType = "fp32"
    activation_dtype: PrecisionDType = "fp32"
    fp8_backend: LowBitBackendName = "transformer_engine"
    fp8_format: FP8Format = "e4m3"
    fp8_amax_history_len: int = 16
    fp8_amax_compute_algo: FP8AmaxComputeAlgo = "most_recent"
    fp4_backend: str = "emulated"
    module_precision_policy: Optional[ModulePrecisionPolicy] = None
    fp8_param: bool = False
    fp4_param: bool = False
    fp4_param_format: FP4PersistentFormat = "nf4"
    persistent_scale_granularity: PersistentScaleGranularity = "per_channel"
    lowbit_master_ownership: MasterOwnershipMode = "optimizer"
    precision_recipe_name: PrecisionRecipeName = "default"
    deepseek_v3_recipe: Optional[DeepSeekV3PrecisionRecipe] = None
    loss_scale_init: float = 65536.0
    loss_scale_growth_factor: float = 2.0
    loss_scale_backoff_factor: float = 0.5
    loss_scale_growth_interval: int = 2000
    loss_scale_min: float = 1.0
    loss_scale_max: float = 16777216.0


@dataclass
class PrecisionRuntimeState:
    loss_scale: float
    growth_tracker: int = 0
    skipped_steps: int = 0
    found_inf_steps: int = 0


@dataclass
class TrainDataBundle:
    loader: Iterable[dict[str, torch.Tensor]]
    sampler: Optional[object]
    metadata: dict[str, object] = field(default_factory=dict)


@dataclass
class OptimizerState:
    optimizer: object
    shard_info: ParamShardInfo
    extra_state: dict[str, object] = field(default_factory=dict)


@dataclass
class StepContext:
    model: torch.nn.Module
    batch: Optional[dict[str, torch.Tensor]]
    optimizer_state: OptimizerState
    runtime_context: RuntimeContext
    train_state: TrainState


@dataclass
class StepOutput:
    """Local metric numerators of one step and their counts."""

    task_loss: float
    aux_loss: float
    total_loss: float
    drop_fraction: float
    counters: dict[str, int] = field(default_factory=dict)


@dataclass
class ResumeState:
    start_global_step: int = 0
    start_epoch: int = 0
    pipeline_epoch: int = 0
    data_seed: Optional[int] = None


class ModelProvider(Protocol):
    def build_model(self, ctx: RuntimeContext) -> torch.nn.Module:
        ...


class DataProvider(Protocol):
    def build_train_data(self, ctx: RuntimeContext) -> TrainDataBundle:
        ...


class OptimizerRuntime(Protocol):
    def initialize(self, model: torch.nn.Module, ctx: RuntimeContext) -> OptimizerState:
        ...

    def zero_grad(self, state: OptimizerState) -> None:
        ...

    def step(self, *, model: torch.nn.Module, state: OptimizerState, ctx: RuntimeContext) -> None:
        ...


class ScheduleStrategy(Protocol):
    def run_step(self, step_ctx: StepContext) -> StepOutput:
        ...


class ScheduleSelector(Protocol):
    def select(self, ctx: RuntimeContext) -> ScheduleStrategy:
        ...


class CheckpointManager(Protocol):
    def load(self, *, model: torch.nn.Module, optimizer_state: OptimizerState, ctx: RuntimeContext) -> ResumeState:
        ...

    def on_step_end(self, *, model: torch.nn.Module, optimizer_state: OptimizerState, state: TrainState,
                    ctx: RuntimeContext) -> None:
        ...

    def on_run_end(self, *, model: torch.nn.Module, optimizer_state: OptimizerState, state: TrainState,
                   ctx: RuntimeContext) -> None:
        ...


class RuntimeBootstrap(Protocol):
    def build_context(self, args: argparse.Namespace) -> RuntimeContext:
        ...


@dataclass
class RuntimeComponents:
    """The six injected components RuntimeEngine drives."""

    bootstrap: RuntimeBootstrap
    model_provider: ModelProvider
    data_provider: DataProvider
    optimizer_runtime: OptimizerRuntime
    schedule_selector: ScheduleSelector
    checkpoint_manager: CheckpointManager
