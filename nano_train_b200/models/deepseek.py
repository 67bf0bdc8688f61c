"""DeepSeek-style decoder LM: MLA attention, RMSNorm, RoPE, dense-first then
routed-MoE blocks, pipeline-stage partitioning.

Public names, config fields (with legacy aliases), module paths and forward
semantics follow the reference's src/models/deepseek.py:47-1095, including
its numerical quirks kept for loss parity: the RoPE layout (interleaved
rotate with a half-split cos/sin cache), q-LoRA always present, the shared
k_rope broadcast to every head, biased TP GatedMLP, averaged shared experts.

On CUDA the attention runs as one flash-attention kernel over
[q_nope | q_rope] / [k_nope | k_rope] heads (d_qk = nope + rope, d_v
separate) instead of materialising [B, h, S, S] scores and an additive mask.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..config import _default_precision_resolver
from ..layers import (ColumnParallelLinear, Dropout, Embedding, Linear, RMSNorm, RowParallelLinear,
                      gather_from_sequence_parallel_region, scatter_to_sequence_parallel_region)
from ..ops.attention import flash_attention
from ..ops.rope import rope_reference
from .moe import ExpertMLP, ExpertParallelMoE, LocalRoutedMoE


@dataclass
class DeepSeekModelConfig:
    param_dtype: torch.dtype
    param_device: Optional[torch.device]
    precision_resolver: object
    module_compute_dtype_overrides: dict = field(default_factory=dict)
    vocab_size: int = 129280
    hidden_size: int = 7168
    num_hidden_layers: int = 61
    num_attention_heads: int = 128
    num_key_value_heads: int = 128
    intermediate_size: int = 18432
    max_position_embeddings: int = 163840
    rms_norm_eps: float = 1e-6
    q_lora_rank: Optional[int] = 1536  # 0 / None: a direct q projection (DeepSeek-V2-Lite)
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    rope_theta: float = 10000.0
    rope_scaling: Dict[str, float] = field(default_factory=lambda: {
        "type": "yarn", "factor": 40.0, "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0,
        "original_max_position_embeddings": 4096.0})
    attention_dropout: float = 0.0
    dropout: float = 0.0
    moe_intermediate_size: int = 2048
    n_routed_experts: int = 256
    n_shared_experts: int = 1
    num_experts_per_tok: int = 8
    first_k_dense_replace: int = 3
    moe_layer_freq: int = 1
    scoring_func: str = "sigmoid"
    topk_method: str = "noaux_tc"
    n_group: int = 8
    topk_group: int = 4
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 2.5
    tie_word_embeddings: bool = False
    # Legacy aliases
    num_layers: Optional[int] = None
    num_kv_heads: Optional[int] = None
    num_experts: Optional[int] = None
    num_shared_experts: Optional[int] = None
    expert_intermediate_size: Optional[int] = None
    top_k: Optional[int] = None
    # B200-build options (defaults keep reference semantics)
    shared_expert_reduction: str = "mean"  # "mean" (reference) or "sum" (DeepSeek paper)
    comm_quant_backend: str = "emulated"

    def __post_init__(self) -> None:
        for alias, target in (("num_layers", "num_hidden_layers"), ("num_kv_heads", "num_key_value_heads"),
                              ("num_experts", "n_routed_experts"), ("num_shared_experts", "n_shared_experts"),
                              ("expert_intermediate_size", "moe_intermediate_size"),
                              ("top_k", "num_experts_per_tok")):
            if getattr(self, alias) is not None:
                setattr(self, target, getattr(self, alias))
        if self.num_attention_heads <= 0:
            raise ValueError("num_attention_heads must be positive")
        if self.n_routed_experts <= 0:
            raise ValueError("n_routed_experts must be positive")
        if self.num_experts_per_tok <= 0:
            raise ValueError("num_experts_per_tok must be positive")
        if self.num_experts_per_tok > self.n_routed_experts:
            raise ValueError("num_experts_per_tok cannot exceed n_routed_experts")
        if self.qk_rope_head_dim <= 0 or self.qk_rope_head_dim % 2 != 0:
            raise ValueError("qk_rope_head_dim must be a positive even number")
        if self.n_group <= 0 or self.n_routed_experts % self.n_group != 0:
            raise ValueError("n_group must divide n_routed_experts")
        if self.topk_group <= 0 or self.topk_group > self.n_group:
            raise ValueError("topk_group must be in [1, n_group]")
        if self.topk_group * (self.n_routed_experts // self.n_group) < self.num_experts_per_tok:
            raise ValueError("topk_group selection exposes fewer experts than num_experts_per_tok")
        if self.first_k_dense_replace < 0:
            raise ValueError("first_k_dense_replace must be non-negative")
        if self.scoring_func not in {"sigmoid", "softmax"}:
            raise ValueError("scoring_func must be 'sigmoid' or 'softmax'")
        for name, dt in self.module_compute_dtype_overrides.items():
            if not name:
                raise ValueError("module_compute_dtype_overrides keys must be non-empty")
            if dt not in {"fp32", "bf16", "fp16"}:
                raise ValueError("module_compute_dtype_overrides values must be one of fp32, bf16, fp16")


class _DeepSeekConfigPrecisionResolver:
    """Applies exact module-path dtype overrides from the config on top of a base resolver."""

    def __init__(self, base, overrides: dict) -> None:
        self._base = base
        self._overrides = dict(overrides)
        self._matched: set[str] = set()

    def resolve_module_init_state(self, *, module_path: str, module_type: str, lowbit_capable_type, kernel_spec=None):
        state = self._base.resolve_module_init_state(module_path=module_path, module_type=module_type,
                                                     lowbit_capable_type=lowbit_capable_type, kernel_spec=kernel_spec)
        dt = self._overrides.get(module_path)
        if dt is None:
            return state
        self._matched.add(module_path)
        return replace(state, assignment=replace(state.assignment, compute_lowbit_mode=None,
                                                 compute_dtype_override=dt), lowbit_backend=None)

    def finalize(self):
        summary = self._base.finalize()
        missing = [n for n in self._overrides if n not in self._matched]
        if missing:
            raise ValueError(f"DeepSeek config module_compute_dtype_overrides matched zero modules: {missing[:5]}")
        return summary

    def deepseek_v3_recipe(self):
        fn = getattr(self._base, "deepseek_v3_recipe", None)
        return fn() if callable(fn) else None


@dataclass
class DeepSeekParallelContext:
    tensor_model_parallel_rank: int = 0
    tensor_model_parallel_size: int = 1
    tensor_model_parallel_group: Optional[object] = None
    expert_model_parallel_rank: int = 0
    expert_model_parallel_size: int = 1
    expert_model_parallel_group: Optional[object] = None
    pipeline_model_parallel_rank: int = 0
    pipeline_model_parallel_size: int = 1
    pipeline_model_parallel_group: Optional[object] = None
    context_parallel_rank: int = 0
    context_parallel_size: int = 1
    context_parallel_group: Optional[object] = None
    pp_layer_splits: Optional[tuple[int, ...]] = None
    capacity_factor: float = 1.0
    expert_tensor_parallel_size: int = 1
    sequence_parallel: bool = True

    def __post_init__(self) -> None:
        for n in ("tensor_model_parallel", "expert_model_parallel", "pipeline_model_parallel"):
            if getattr(self, f"{n}_size") <= 0:
                raise ValueError(f"{n}_size must be positive")
        if self.context_parallel_size <= 0:
            raise ValueError("context_parallel_size must be positive")
        for n in ("tensor_model_parallel", "expert_model_parallel", "pipeline_model_parallel"):
            r, s = getattr(self, f"{n}_rank"), getattr(self, f"{n}_size")
            if r < 0 or r >= s:
                raise ValueError(f"{n}_rank must be in [0, {n}_size)")
        if self.context_parallel_rank < 0 or self.context_parallel_rank >= self.context_parallel_size:
            raise ValueError("context_parallel_rank must be in [0, context_parallel_size)")
        if self.pp_layer_splits is not None:
            if len(self.pp_layer_splits) != self.pipeline_model_parallel_size + 1:
                raise ValueError("pp_layer_splits length must be pipeline_model_parallel_size + 1")
            if self.pp_layer_splits[0] != 0:
                raise ValueError("pp_layer_splits must start with 0")
            for i in range(1, len(self.pp_layer_splits)):
                if self.pp_layer_splits[i] <= self.pp_layer_splits[i - 1]:
                    raise ValueError("pp_layer_splits must be strictly increasing")
        if self.capacity_factor <= 0:
            raise ValueError("capacity_factor must be positive")
        if self.expert_tensor_parallel_size != 1:
            raise ValueError("DeepSeek routed experts currently require expert_tensor_parallel_size=1")

    def resolve_attention_tensor_model_parallel(self) -> Tuple[int, int, Optional[object]]:
        return self.tensor_model_parallel_rank, self.tensor_model_parallel_size, self.tensor_model_parallel_group

    def resolve_expert_model_parallel(self) -> Tuple[int, int, Optional[object]]:
        return self.expert_model_parallel_rank, self.expert_model_parallel_size, self.expert_model_parallel_group

    resolve_attn_tp = resolve_attention_tensor_model_parallel
    resolve_moe_ep = resolve_expert_model_parallel

    def resolve_pp_layer_boundaries(self, num_hidden_layers: int) -> tuple[int, ...]:
        if num_hidden_layers <= 0:
            raise ValueError("num_hidden_layers must be positive")
        if self.pipeline_model_parallel_size == 1:
            return (0, num_hidden_layers)
        if self.pp_layer_splits is not None:
            if self.pp_layer_splits[-1] != num_hidden_layers:
                raise ValueError("pp_layer_splits last value must equal num_hidden_layers")
            return self.pp_layer_splits
        base, rem = divmod(num_hidden_layers, self.pipeline_model_parallel_size)
        b = [0]
        for stage in range(self.pipeline_model_parallel_size):
            b.append(b[-1] + base + (1 if stage < rem else 0))
        return tuple(b)

    def resolve_pp_layer_range(self, num_hidden_layers: int) -> tuple[int, int]:
        b = self.resolve_pp_layer_boundaries(num_hidden_layers)
        r = self.pipeline_model_parallel_rank
        return b[r], b[r + 1]

    tp_rank = property(lambda self: self.tensor_model_parallel_rank)
    tp_size = property(lambda self: self.tensor_model_parallel_size)
    tp_group = property(lambda self: self.tensor_model_parallel_group)
    ep_rank = property(lambda self: self.expert_model_parallel_rank)
    ep_size = property(lambda self: self.expert_model_parallel_size)
    ep_group = property(lambda self: self.expert_model_parallel_group)
    pp_rank = property(lambda self: self.pipeline_model_parallel_rank)
    pp_size = property(lambda self: self.pipeline_model_parallel_size)
    pp_group = property(lambda self: self.pipeline_model_parallel_group)
    expert_tp_size = property(lambda self: self.expert_tensor_parallel_size)
    enable_moe_sequence_parallel = property(lambda self: self.sequence_parallel)


# ------------------------------------------------------------------ RoPE helpers (reference layout)
def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Pairs interleaved elements: (x0, x1, x2, x3, ...) -> (-x1, x0, -x3, x2, ...)."""
    return torch.stack((-x[..., 1::2], x[..., ::2]), dim=-1).flatten(-2)


def _build_rope_cache(seq_len: int, dim: int, device, theta: float):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device).float() / dim))
    freqs = torch.outer(torch.arange(seq_len, device=device).float(), inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def _apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: (B, H, S, D)."""
    return x * cos[None, None] + _rotate_half(x) * sin[None, None]


class GatedMLP(nn.Module):
    """SwiGLU FFN: column(gate), column(up), row(down) with biases under TP; ExpertMLP otherwise."""

    def __init__(self, hidden_size: int, intermediate_size: int, dropout: float, param_dtype, param_device,
                 precision_resolver, module_prefix: str, parallel_context: Optional[DeepSeekParallelContext] = None):
        super().__init__()
        self.parallel_context = parallel_context or DeepSeekParallelContext()
        pc = self.parallel_context
        self.use_tp = pc.tensor_model_parallel_size > 1
        kw = dict(param_dtype=param_dtype, param_device=param_device, precision_resolver=precision_resolver)
        if self.use_tp:
            tp = dict(tp_rank=pc.tensor_model_parallel_rank, tp_size=pc.tensor_model_parallel_size,
                      tp_group=pc.tensor_model_parallel_group, bias=True)
            self.gate_proj = ColumnParallelLinear(hidden_size, intermediate_size, module_path=f"{module_prefix}.gate_proj",
                                                  **tp, **kw)
            self.up_proj = ColumnParallelLinear(hidden_size, intermediate_size, module_path=f"{module_prefix}.up_proj",
                                                **tp, **kw)
            self.down_proj = RowParallelLinear(intermediate_size, hidden_size, module_path=f"{module_prefix}.down_proj",
                                               **tp, **kw)
            self.dropout = Dropout(dropout)
        else:
            self.mlp = ExpertMLP(hidden_size, intermediate_size, dropout, module_prefix=f"{module_prefix}.mlp", **kw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.use_tp:
            return self.dropout(self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x)))
        return self.mlp(x)


class _RopeColumnsInPlace(torch.autograd.Function):
    """RoPE of columns [off, off + R) of every head of x [B, S, h, D], in place (x is a projection's
    output that nothing else keeps); the backward rotates the incoming gradient in place. The q of MLA
    thus stays one [B, S, h, nope | rope] tensor for the attention kernel, with no concatenation in the
    forward and none in the backward."""

    @staticmethod
    def forward(ctx, x, off, R, theta, mode):
        from ..ops.rope import rope_rows_

        B, S, h, D = x.shape
        rope_rows_(x.view(B * S, h, D), off, R, S, theta, mode, False)
        ctx.mark_dirty(x)
        ctx.meta = (off, R, theta, mode)
        return x

    @staticmethod
    def backward(ctx, dy):
        from ..ops.rope import rope_rows_

        off, R, theta, mode = ctx.meta
        dy = dy.contiguous()
        B, S, h, D = dy.shape
        rope_rows_(dy.view(B * S, h, D), off, R, S, theta, mode, True)
        return dy, None, None, None, None


class _MlaAttention(torch.autograd.Function):
    """Causal MLA attention from the projection outputs, without materialising the broadcast rope key.

    q [B, S, h, Dn + R] (rope columns already rotated), kv [B, S, h, Dn + Dv] (the kv up-projection: nope
    keys, then values, per head), k_rope [B, S, R] (rope part of the kv down-projection, not rotated, one
    vector per token shared by every head; reference: src/models/deepseek.py:681-738, where it is
    expanded over heads and concatenated to k_nope). Forward: one kernel writes the keys
    [k_nope | rope(k_rope)] per head, and the tcgen05 attention reads the values as a strided view of kv.
    Backward: the attention backward stores dV straight into the value columns of dkv, and one kernel
    copies dK's nope part into dkv and reduces its rope part over heads into dk_rope (rotated back)."""

    @staticmethod
    def forward(ctx, q, kv, k_rope, Dn, scale, theta):
        from ..ops._ext import ext
        from ..ops.attention import _fwd
        from ..ops.rope import rope_table

        B, S, h, Dkv = kv.shape
        R = k_rope.shape[-1]
        table = rope_table(S, R, theta, kv.device)
        kf = ext().mla_k_assemble(kv.reshape(B * S, h, Dkv), k_rope.reshape(B * S, R), table, Dn, S)
        kf = kf.view(B, S, h, Dn + R)
        v = kv[..., Dn:]
        o, lse = _fwd(q, kf, v, scale, True)
        ctx.save_for_backward(q, kf, v, o, lse)
        ctx.meta = (Dn, scale, theta)
        return o

    @staticmethod
    def backward(ctx, do):
        from ..ops._ext import ext
        from ..ops.rope import rope_table

        q, kf, v, o, lse = ctx.saved_tensors
        Dn, scale, theta = ctx.meta
        B, S, h, Dk = kf.shape
        Dv = v.shape[-1]
        C = ext()
        dkv = torch.empty(B, S, h, Dn + Dv, device=kf.device, dtype=kf.dtype)
        dk = torch.empty_like(kf)
        dq = C.flash_attn_bwd(do.contiguous(), q, kf, v, o, lse, float(scale), True, None, dk, dkv[..., Dn:])[0]
        dkr = C.mla_k_assemble_bwd(dk.view(B * S, h, Dk), dkv.view(B * S, h, Dn + Dv),
                                   rope_table(S, Dk - Dn, theta, kf.device), Dn, S)
        return dq, dkv, dkr.view(B, S, Dk - Dn), None, None, None


def _mla_fused_ok(q: torch.Tensor, kv: torch.Tensor, k_rope: torch.Tensor, Dn: int) -> bool:
    """The fused key assembly applies: bf16 tensors whose rows start on 16-byte boundaries, head dims of
    a tcgen05 attention kernel, rope width R with R / 8 dividing 32."""
    from ..ops._ext import ext
    from ..ops.attention import _KERNEL_HEAD_DIMS

    R = k_rope.shape[-1]
    if not (q.is_cuda and q.dtype == kv.dtype == k_rope.dtype == torch.bfloat16 and hasattr(ext(), "mla_k_assemble")):
        return False
    if (Dn + R, kv.shape[-1] - Dn) not in _KERNEL_HEAD_DIMS or R % 8 or 32 % (R // 8) or Dn % 8:
        return False
    return all(t.stride(-1) == 1 and all(st % 8 == 0 for st in t.stride()[:-1]) and t.data_ptr() % 16 == 0
               for t in (kv, k_rope))


class MultiHeadLatentAttention(nn.Module):
    def __init__(self, config: DeepSeekModelConfig, parallel_context: Optional[DeepSeekParallelContext] = None, *,
                 module_prefix: str):
        super().__init__()
        self.parallel_context = parallel_context or DeepSeekParallelContext()
        (self.attention_tensor_model_parallel_rank, self.attention_tensor_model_parallel_size,
         self.attention_tensor_model_parallel_group) = self.parallel_context.resolve_attention_tensor_model_parallel()
        tp = self.attention_tensor_model_parallel_size
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        if self.num_heads % tp != 0:
            raise ValueError("num_attention_heads must be divisible by attention TP size")
        self.local_num_heads = self.num_heads // tp
        self.qk_nope_head_dim = config.qk_nope_head_dim
        self.qk_rope_head_dim = config.qk_rope_head_dim
        self.v_head_dim = config.v_head_dim
        self.qk_head_dim = self.qk_nope_head_dim + self.qk_rope_head_dim
        self.scale = self.qk_head_dim ** -0.5
        self.rope_theta = config.rope_theta
        kw = dict(param_dtype=config.param_dtype, param_device=config.param_device,
                  precision_resolver=config.precision_resolver)
        tpkw = dict(tp_rank=self.attention_tensor_model_parallel_rank, tp_size=tp,
                    tp_group=self.attention_tensor_model_parallel_group)
        q_out = self.num_heads * self.qk_head_dim
        self.q_proj = self.q_a_proj = self.q_a_norm = self.q_b_proj = None
        if config.q_lora_rank:
            self.q_a_proj = Linear(self.hidden_size, config.q_lora_rank, bias=False,
                                   module_path=f"{module_prefix}.q_a_proj", **kw)
            self.q_a_norm = RMSNorm(config.q_lora_rank, eps=config.rms_norm_eps,
                                    module_path=f"{module_prefix}.q_a_norm", **kw)
            if tp > 1:
                self.q_b_proj = ColumnParallelLinear(config.q_lora_rank, q_out, bias=False,
                                                     module_path=f"{module_prefix}.q_b_proj", **tpkw, **kw)
            else:
                self.q_b_proj = Linear(config.q_lora_rank, q_out, bias=False, module_path=f"{module_prefix}.q_b_proj",
                                       **kw)
        elif tp > 1:  # no q-LoRA (DeepSeek-V2-Lite): one projection to the heads
            self.q_proj = ColumnParallelLinear(self.hidden_size, q_out, bias=False,
                                               module_path=f"{module_prefix}.q_proj", **tpkw, **kw)
        else:
            self.q_proj = Linear(self.hidden_size, q_out, bias=False, module_path=f"{module_prefix}.q_proj", **kw)
        self.kv_a_proj = None
        self.kv_a_proj = Linear(self.hidden_size, config.kv_lora_rank + self.qk_rope_head_dim, bias=False,
                                module_path=f"{module_prefix}.kv_a_proj", **kw)
        self.kv_a_norm = RMSNorm(config.kv_lora_rank, eps=config.rms_norm_eps, module_path=f"{module_prefix}.kv_a_norm",
                                 **kw)
        kv_out = self.num_heads * (self.qk_nope_head_dim + self.v_head_dim)
        if tp > 1:
            self.kv_b_proj = ColumnParallelLinear(config.kv_lora_rank, kv_out, bias=False,
                                                  module_path=f"{module_prefix}.kv_b_proj", **tpkw, **kw)
            self.out_proj = RowParallelLinear(self.num_heads * self.v_head_dim, self.hidden_size, bias=False,
                                              module_path=f"{module_prefix}.out_proj", **tpkw, **kw)
        else:
            self.kv_b_proj = Linear(config.kv_lora_rank, kv_out, bias=False, module_path=f"{module_prefix}.kv_b_proj",
                                    **kw)
            self.out_proj = Linear(self.num_heads * self.v_head_dim, self.hidden_size, bias=False,
                                   module_path=f"{module_prefix}.out_proj", **kw)
        self.dropout = Dropout(config.attention_dropout)

    def _qkv(self, x: torch.Tensor):
        """q [B, S, h, Dn + R], kv [B, S, h, Dn + Dv] (nope keys | values per head), k_rope [B, S, R]."""
        B, S, _ = x.shape
        h = self.local_num_heads
        q = self.q_proj(x) if self.q_proj is not None else self.q_b_proj(self.q_a_norm(self.q_a_proj(x)))
        q = q.view(B, S, h, self.qk_head_dim)
        kv_a = self.kv_a_proj(x)
        kv_latent, k_rope = torch.split(kv_a, [self.kv_a_norm.weight.shape[0], self.qk_rope_head_dim], dim=-1)
        kv = self.kv_b_proj(self.kv_a_norm(kv_latent)).view(B, S, h, self.qk_nope_head_dim + self.v_head_dim)
        return q, kv, k_rope

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, _ = x.shape
        h = self.local_num_heads
        q, kv, k_rope = self._qkv(x)
        k_nope, v = torch.split(kv, [self.qk_nope_head_dim, self.v_head_dim], dim=-1)
        if x.is_cuda and attention_mask is None:
            qf = q if q.is_contiguous() else q.contiguous()
            qf = _RopeColumnsInPlace.apply(qf, self.qk_nope_head_dim, self.qk_rope_head_dim, float(self.rope_theta),
                                           "deepseek")
            if _mla_fused_ok(qf, kv, k_rope, self.qk_nope_head_dim):
                o = _MlaAttention.apply(qf, kv, k_rope, self.qk_nope_head_dim, self.scale, float(self.rope_theta))
                return self.out_proj(self.dropout(o).reshape(B, S, h * self.v_head_dim))
            k_rope = ops.apply_rope(k_rope.unsqueeze(2), self.rope_theta, "deepseek")
            kf = torch.cat([k_nope, k_rope.expand(B, S, h, self.qk_rope_head_dim)], dim=-1)
            o = flash_attention(qf, kf, v, causal=True, softmax_scale=self.scale)
            o = self.dropout(o)
            return self.out_proj(o.reshape(B, S, h * self.v_head_dim))
        # Reference math path (CPU / explicit masks): materialised scores, fp32 softmax.
        pos = torch.arange(S, device=x.device)
        q_nope, q_rope = torch.split(q, [self.qk_nope_head_dim, self.qk_rope_head_dim], dim=-1)
        q_rope = rope_reference(q_rope, pos, self.rope_theta, "deepseek")
        k_rope = rope_reference(k_rope.unsqueeze(2), pos, self.rope_theta, "deepseek")
        qf = torch.cat([q_nope, q_rope], dim=-1).permute(0, 2, 1, 3)
        kf = torch.cat([k_nope, k_rope.expand(B, S, h, self.qk_rope_head_dim)], dim=-1).permute(0, 2, 1, 3)
        vf = v.permute(0, 2, 1, 3)
        scores = torch.matmul(qf, kf.transpose(-2, -1)) * self.scale
        if attention_mask is None:
            attention_mask = torch.full((S, S), float("-inf"), device=x.device).triu(1)
        scores = scores + attention_mask
        probs = torch.softmax(scores.float(), dim=-1).to(vf.dtype)
        probs = self.dropout(probs)
        out = torch.matmul(probs, vf).permute(0, 2, 1, 3).reshape(B, S, h * self.v_head_dim)
        return self.out_proj(out)


class RoutedMoE(nn.Module):
    def __init__(self, config: DeepSeekModelConfig, parallel_context: Optional[DeepSeekParallelContext] = None, *,
                 module_prefix: str):
        super().__init__()
        self.parallel_context = parallel_context or DeepSeekParallelContext()
        pc = self.parallel_context
        (self.expert_model_parallel_rank, self.expert_model_parallel_size,
         self.expert_model_parallel_group) = pc.resolve_expert_model_parallel()
        self.use_moe_sequence_parallel = pc.sequence_parallel and pc.tensor_model_parallel_size > 1
        shared = dict(hidden_size=config.hidden_size, expert_intermediate_size=config.moe_intermediate_size,
                      num_experts=config.n_routed_experts, top_k=config.num_experts_per_tok,
                      param_dtype=config.param_dtype, param_device=config.param_device,
                      precision_resolver=config.precision_resolver, module_prefix=module_prefix,
                      dropout=config.dropout, n_shared_experts=config.n_shared_experts,
                      scoring_func=config.scoring_func, n_group=config.n_group, topk_group=config.topk_group,
                      norm_topk_prob=config.norm_topk_prob, routed_scaling_factor=config.routed_scaling_factor,
                      capacity_factor=pc.capacity_factor)
        if self.expert_model_parallel_size > 1:
            recipe = None
            fn = getattr(config.precision_resolver, "deepseek_v3_recipe", None)
            if callable(fn):
                recipe = fn()
            cq = recipe.comm_quant_granularity if (recipe is not None and recipe.comm_quant_enabled) else None
            rnd = recipe.rounding_mode if recipe is not None else "nearest"
            self.moe = ExpertParallelMoE(**shared, ep_rank=self.expert_model_parallel_rank,
                                         ep_size=self.expert_model_parallel_size,
                                         ep_group=self.expert_model_parallel_group,
                                         expert_tp_size=pc.expert_tensor_parallel_size, comm_quant_granularity=cq,
                                         comm_quant_rounding=rnd, comm_quant_backend=config.comm_quant_backend)
        else:
            self.moe = LocalRoutedMoE(**shared)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.use_moe_sequence_parallel:
            return self.moe(x)
        pc = self.parallel_context
        local = scatter_to_sequence_parallel_region(x, pc.tensor_model_parallel_rank, pc.tensor_model_parallel_size,
                                                    pc.tensor_model_parallel_group, seq_dim=1)
        out = self.moe(local)
        return gather_from_sequence_parallel_region(out, pc.tensor_model_parallel_rank,
                                                    pc.tensor_model_parallel_size, pc.tensor_model_parallel_group,
                                                    seq_dim=1)


class DeepSeekDecoderBlock(nn.Module):
    def __init__(self, config: DeepSeekModelConfig, layer_idx: int,
                 parallel_context: Optional[DeepSeekParallelContext] = None, *, module_prefix: str):
        super().__init__()
        self.parallel_context = parallel_context or DeepSeekParallelContext()
        kw = dict(param_dtype=config.param_dtype, param_device=config.param_device,
                  precision_resolver=config.precision_resolver)
        self.attn_norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps, module_path=f"{module_prefix}.attn_norm",
                                 **kw)
        self.attn = MultiHeadLatentAttention(config, parallel_context=self.parallel_context,
                                             module_prefix=f"{module_prefix}.attn")
        self.ffn_norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps, module_path=f"{module_prefix}.ffn_norm",
                                **kw)
        use_dense = layer_idx < config.first_k_dense_replace
        use_moe = (not use_dense and (layer_idx - config.first_k_dense_replace) % max(1, config.moe_layer_freq) == 0)
        if use_moe:
            self.ffn = RoutedMoE(config, parallel_context=self.parallel_context, module_prefix=f"{module_prefix}.ffn")
            self.ffn_type = "moe"
        else:
            self.ffn = GatedMLP(config.hidden_size, config.intermediate_size, config.dropout, config.param_dtype,
                                config.param_device, config.precision_resolver, f"{module_prefix}.ffn",
                                parallel_context=self.parallel_context)
            self.ffn_type = "dense"

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        x = x + self.attn(self.attn_norm(x), attention_mask)
        return x + self.ffn(self.ffn_norm(x))


class DeepSeekModel(nn.Module):
    def __init__(self, config: DeepSeekModelConfig, parallel_context: Optional[DeepSeekParallelContext] = None):
        super().__init__()
        if config.precision_resolver is None:
            config.precision_resolver = _default_precision_resolver()
        if config.module_compute_dtype_overrides:
            config.precision_resolver = _DeepSeekConfigPrecisionResolver(config.precision_resolver,
                                                                         config.module_compute_dtype_overrides)
        self.config = config
        self.parallel_context = parallel_context or DeepSeekParallelContext()
        pc = self.parallel_context
        self.pipeline_model_parallel_rank = pc.pipeline_model_parallel_rank
        self.pipeline_model_parallel_size = pc.pipeline_model_parallel_size
        self.pipeline_model_parallel_group = pc.pipeline_model_parallel_group
        self.pipeline_layer_start, self.pipeline_layer_end = pc.resolve_pp_layer_range(config.num_hidden_layers)
        self.pipeline_layer_boundaries = pc.resolve_pp_layer_boundaries(config.num_hidden_layers)
        if pc.tensor_model_parallel_size > 1 and config.intermediate_size % pc.tensor_model_parallel_size != 0:
            raise ValueError("intermediate_size must be divisible by tensor_model_parallel_size for TP dense FFN")
        if pc.tensor_model_parallel_size > 1 and config.num_attention_heads % pc.tensor_model_parallel_size != 0:
            raise ValueError("num_attention_heads must be divisible by attention TP size")
        if pc.expert_model_parallel_size > 1 and config.n_routed_experts % pc.expert_model_parallel_size != 0:
            raise ValueError("n_routed_experts must be divisible by expert_model_parallel_size for EP MoE")
        if self.pipeline_layer_end <= self.pipeline_layer_start:
            raise ValueError("Each PP stage must own at least one decoder layer")
        if config.tie_word_embeddings and self.pipeline_model_parallel_size > 1:
            raise ValueError("tie_word_embeddings is not supported when pipeline_model_parallel_size > 1")
        kw = dict(param_dtype=config.param_dtype, param_device=config.param_device,
                  precision_resolver=config.precision_resolver)
        if self.is_first_pp_stage:
            self.token_embeddings = Embedding(config.vocab_size, config.hidden_size, module_path="token_embeddings", **kw)
            self.dropout = Dropout(config.dropout)
        else:
            self.token_embeddings = None
            self.dropout = None
        self.blocks = nn.ModuleList([DeepSeekDecoderBlock(config, i, parallel_context=pc, module_prefix=f"blocks.{i}")
                                     for i in range(self.pipeline_layer_start, self.pipeline_layer_end)])
        if self.is_last_pp_stage:
            self.final_norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps, module_path="final_norm", **kw)
            self.lm_head = Linear(config.hidden_size, config.vocab_size, bias=False, module_path="lm_head", **kw)
        else:
            self.final_norm = None
            self.lm_head = None
        self.apply(self._init_weights)
        if config.tie_word_embeddings and self.token_embeddings is not None and self.lm_head is not None:
            self.lm_head.weight = self.token_embeddings.weight

    def _init_weights(self, module: nn.Module) -> None:
        if isinstance(module, (Linear, ColumnParallelLinear, RowParallelLinear)):
            if module.weight.device.type != "meta":
                nn.init.normal_(module.weight, mean=0.0, std=0.02)
                if module.bias is not None:
                    nn.init.zeros_(module.bias)
        elif isinstance(module, Embedding):
            if module.weight.device.type != "meta":
                nn.init.normal_(module.weight, mean=0.0, std=0.02)
        elif isinstance(module, RMSNorm):
            if module.weight.device.type != "meta":
                nn.init.ones_(module.weight)

    def _create_causal_mask(self, batch_size: int, seq_len: int, device) -> torch.Tensor:
        m = torch.full((seq_len, seq_len), float("-inf"), device=device).triu(1)
        return m.view(1, 1, seq_len, seq_len).expand(batch_size, -1, -1, -1)

    @property
    def is_first_pp_stage(self) -> bool:
        return self.pipeline_model_parallel_rank == 0

    @property
    def is_last_pp_stage(self) -> bool:
        return self.pipeline_model_parallel_rank == self.pipeline_model_parallel_size - 1

    def local_layer_range(self) -> tuple[int, int]:
        return self.pipeline_layer_start, self.pipeline_layer_end

    def forward_stage(self, input_ids: Optional[torch.Tensor], hidden_states: Optional[torch.Tensor],
                      attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """First stage: ids -> hidden (or logits when PP == 1); middle: hidden -> hidden; last: -> logits."""
        if self.is_first_pp_stage:
            if input_ids is None:
                raise ValueError("input_ids is required on the first PP stage")
            if self.token_embeddings is None or self.dropout is None:
                raise RuntimeError("First PP stage is missing embedding modules")
            x = self.dropout(self.token_embeddings(input_ids))
        else:
            if hidden_states is None:
                raise ValueError("hidden_states is required on non-first PP stages")
            x = hidden_states
        for block in self.blocks:
            x = block(x, attention_mask)
        if self.is_last_pp_stage:
            if self.final_norm is None or self.lm_head is None:
                raise RuntimeError("Last PP stage is missing output modules")
            return self.lm_head(self.final_norm(x))
        return x

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.pipeline_model_parallel_size > 1:
            raise RuntimeError("forward() is only valid for pipeline_model_parallel_size==1; use forward_stage() for PP")
        return self.forward_stage(input_ids=input_ids, hidden_states=None, attention_mask=attention_mask)

    @property
    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())


def gather_moe_metrics(model: nn.Module) -> tuple[torch.Tensor, float, int]:
    """(sum of MoE aux losses, sum of dropped fractions, number of MoE layers) of the last forward."""
    aux = None
    drops = []
    for m in model.modules():
        if isinstance(m, (LocalRoutedMoE, ExpertParallelMoE)):
            a = m.last_aux_loss
            aux = a if aux is None else aux + a
            drops.append(m.last_dropped_fraction_tensor.float().reshape(()))
    if aux is None:
        p = next(model.parameters())
        aux = torch.zeros((), device=p.device, dtype=torch.float32)
    # One host read for every layer's dropped fraction.
    drop = float(torch.stack([d.to(aux.device) for d in drops]).sum()) if drops else 0.0
    return aux, drop, len(drops)
