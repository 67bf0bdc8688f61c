"""Configuration dataclasses.

Field names and defaults follow the reference's public config objects
(src/config.py:19-352: ModelConfig, TPConfig, TrainingConfig, DataConfig,
MonitoringConfig, AlertThresholdsConfig, DistributedConfig, Config) so that
scripts written against it keep working. ``ModelConfig`` gains optional
architecture switches (RMSNorm, RoPE, SwiGLU, grouped-query attention, untied
head, sequence parallelism) used by the Llama-shape configuration; their
defaults reproduce the reference's GPT-2 block.
"""
from __future__ import annotations

from dataclasses import dataclass, field, fields, is_dataclass
from typing import Literal, Optional, Protocol

import torch
import torch.distributed as dist


class _PrecisionResolverLike(Protocol):
    def resolve_module_init_state(self, *, module_path: str, module_type: str, lowbit_capable_type,
                                  kernel_spec=None):
        ...

    def finalize(self):
        ...

    def deepseek_v3_recipe(self):
        ...


class FullPrecisionResolver:
    """Precision resolver of call sites without a low-bit policy: every module computes in its parameter
    dtype. It answers with the runtime's own contract types (``ModulePrecisionInitState`` holding a
    ``ModulePrecisionAssignment`` with low-bit compute and persistence off), so layers treat it exactly
    like a resolver built from a precision config."""

    def resolve_module_init_state(self, *, module_path: str, module_type: str, lowbit_capable_type,
                                  kernel_spec=None):
        from .runtime.contracts import ModulePrecisionAssignment, ModulePrecisionInitState

        del lowbit_capable_type, kernel_spec
        return ModulePrecisionInitState(assignment=ModulePrecisionAssignment(
            module_name=module_path, module_type=module_type, compute_lowbit_mode=None,
            persistent_lowbit_mode="off", persistent_scale_granularity="per_channel", fp4_persistent_format="nf4"))

    def finalize(self):
        return None

    def deepseek_v3_recipe(self):
        return None


_NoOpPrecisionResolver = FullPrecisionResolver  # name used by earlier scripts and tests


def _default_precision_resolver() -> _PrecisionResolverLike:
    return FullPrecisionResolver()


@dataclass
class ModelConfig:
    """Dense transformer architecture.

    Defaults are the reference's 125M GPT-2 block; the Llama-shape benchmark
    sets ``norm="rmsnorm"``, ``position="rope"``, ``mlp="swiglu"``,
    ``num_key_value_heads`` and ``tie_word_embeddings=False``.
    """

    param_dtype: torch.dtype
    param_device: Optional[torch.device]
    precision_resolver: _PrecisionResolverLike
    hidden_size: int = 768
    num_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    max_position_embeddings: int = 2048
    vocab_size: int = 50257
    dropout: float = 0.1
    # Architecture switches (B200 build additions; defaults = reference GPT-2)
    num_key_value_heads: Optional[int] = None
    norm: Literal["layernorm", "rmsnorm"] = "layernorm"
    norm_eps: float = 1e-5
    position: Literal["learned", "rope"] = "learned"
    rope_theta: float = 10000.0
    mlp: Literal["gelu", "swiglu"] = "gelu"
    bias: bool = True
    tie_word_embeddings: bool = True
    sequence_parallel: bool = False
    init_std: float = 0.02


@dataclass
class TPConfig:
    """Tensor-parallel placement of this process (1/size of every sharded weight)."""

    enabled: bool = False
    rank: int = 0
    size: int = 1
    group: Optional[object] = None

    def __post_init__(self) -> None:
        if self.enabled:
            if self.size <= 1:
                raise ValueError("tp_size must be > 1 when TP is enabled")
            if self.rank < 0 or self.rank >= self.size:
                raise ValueError(f"tp_rank must be in [0, {self.size - 1}]")
            if self.group is None:
                self.group = dist.group.WORLD


@dataclass
class TrainingConfig:
    batch_size: int = 32
    micro_batch_size: int = 32
    learning_rate: float = 3e-4
    weight_decay: float = 0.1
    max_steps: int = 100
    eval_steps: int = 50
    save_steps: int = 50
    log_steps: int = 10
    warmup_steps: int = 10
    clip_grad: float = 1.0
    bf16: bool = True
    gradient_checkpointing: bool = False


@dataclass
class DataConfig:
    dataset_path: str = "examples/tiny_shakespeare.txt"
    max_seq_length: int = 256
    train_split: float = 0.9


@dataclass
class MonitoringConfig:
    """Bounded monitoring: cost scales with depth, not parameter count, except in debug mode."""

    mode: Literal["minimal", "standard", "debug"] = "standard"
    histogram_steps: int = 1000
    activation_sites: Literal["none", "sentinel", "all_lns"] = "sentinel"
    sync_cuda_timing: bool = False
    fail_fast_nonfinite: bool = True
    gpu_metrics_steps: int = 10
    log_memory: bool = True
    grad_norm_per_block_steps: int = 100
    update_ratio_steps: int = 100
    tensorboard_max_queue: int = 1
    tensorboard_flush_secs: int = 1
    tensorboard_flush_on_log: bool = True
    attn_tau: float = 100.0
    loss_ema_beta: float = 0.98
    sentinel_blocks: Optional[tuple[int, int, int]] = None
    opt_state_check_steps: int = 1000
    probe_steps: int = 1000
    probe_topk: int = 10
    peak_tflops: Optional[float] = None
    mfu_flops_multiplier: float = 6.0


@dataclass
class AlertThresholdsConfig:
    loss_spike_warn: float = 3.0
    loss_spike_stop: float = 10.0
    grad_norm_warn_min: float = 1e-2
    grad_norm_warn_max: float = 1e2
    grad_norm_stop_max: float = 1e3
    clip_coef_warn: float = 0.5
    clip_coef_bad: float = 0.1
    update_ratio_warn_low: float = 1e-7
    update_ratio_warn_high: float = 1e-1
    update_ratio_stop_high: float = 3e-1
    depth_ratio_warn: float = 0.05
    depth_ratio_bad: float = 0.01
    ignore_frac_warn: float = 0.2
    ignore_frac_bad: float = 0.3
    activation_rms_warn_low: float = 0.5
    activation_rms_warn_high: float = 2.0
    activation_rms_bad_low: float = 0.25
    activation_rms_bad_high: float = 4.0
    activation_max_abs_warn: float = 20.0
    activation_max_abs_bad: float = 50.0
    max_attn_logit_warn: float = 200.0
    max_attn_logit_crit: float = 1000.0
    attn_entropy_norm_warn: float = 0.1
    residual_outlier_rate_warn: float = 1e-3
    residual_outlier_rate_bad: float = 1e-2
    data_wait_frac_warn: float = 0.3
    data_wait_frac_bad: float = 0.5
    reserved_frac_warn: float = 0.90
    reserved_frac_bad: float = 0.95


@dataclass
class DistributedConfig:
    world_size: Optional[int] = None
    backend: Literal["auto", "gloo", "nccl"] = "auto"
    master_addr: str = "localhost"
    master_port: int = 29500
    device: Optional[Literal["cpu", "cuda"]] = None
    find_unused_parameters: bool = False
    broadcast_buffers: bool = False
    bucket_cap_mb: int = 25
    use_distributed_optimizer: bool = False
    data_parallel_sharding_strategy: Literal["no_shard", "optim", "optim_grads"] = "no_shard"
    num_distributed_optimizer_instances: int = 1


@dataclass
class Config:
    model: ModelConfig = field(default_factory=lambda: ModelConfig(
        param_dtype=torch.float32, param_device=None, precision_resolver=_default_precision_resolver()))
    training: TrainingConfig = field(default_factory=TrainingConfig)
    data: DataConfig = field(default_factory=DataConfig)
    monitoring: MonitoringConfig = field(default_factory=MonitoringConfig)
    alerts: AlertThresholdsConfig = field(default_factory=AlertThresholdsConfig)
    distributed: DistributedConfig = field(default_factory=DistributedConfig)
    output_dir: str = "outputs"
    run_name: str = "nano_train_mvp"
    log_dir: str = "outputs"
    seed: int = 42


def _serialize_config_value(value: object) -> object:
    if isinstance(value, (torch.dtype, torch.device)):
        return str(value)
    if isinstance(value, (str, int, float, bool)) or value is None:
        return value
    if is_dataclass(value):
        return {f.name: _serialize_config_value(getattr(value, f.name)) for f in fields(value)}
    if isinstance(value, dict):
        return {str(k): _serialize_config_value(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_serialize_config_value(v) for v in value]
    return str(value)


def config_to_serializable_dict(config: Config) -> dict[str, object]:
    """JSON-safe dictionary of a Config (dtypes/devices/objects become strings)."""
    out = _serialize_config_value(config)
    if not isinstance(out, dict):
        raise ValueError("Config serialization must produce a dictionary")
    return out
