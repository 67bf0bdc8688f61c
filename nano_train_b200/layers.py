"""Layer primitives (L1): linear layers (plain / column / row tensor-parallel),
norms, embedding, dropout, GELU, gradient clipping and the tensor/sequence
parallel region functions.

Public names, constructor keywords (``param_dtype``, ``param_device``,
``module_path``, ``precision_resolver``) and forward semantics follow the
reference's src/layers.py (Linear 465-632, LayerNorm 639-781, Embedding
788-900, Dropout 907-1010, GELU 1017-1095, clip_grad_norm 1102-1189,
Column/RowParallelLinear 1235-1496, SP scatter/gather 1499-1597). The math
underneath runs on the sm_100a kernels of ``nano_train_b200.ops``;
low-bit compute and persistent low-bit weights come from
``nano_train_b200.precision`` through the mixins below.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from .config import _default_precision_resolver
from .parallel import comm
from .parallel.tp_linear import column_parallel_linear_sp, row_parallel_linear_sp
from .precision.lowbit_linear import LowBitLinearMixin, ModulePrecisionStateMixin

__all__ = [
    "Linear", "ColumnParallelLinear", "RowParallelLinear", "LayerNorm", "RMSNorm", "Embedding",
    "VocabParallelEmbedding", "Dropout", "GELU", "clip_grad_norm", "scatter_to_sequence_parallel_region",
    "gather_from_sequence_parallel_region", "copy_to_tensor_parallel_region", "reduce_from_tensor_parallel_region",
]

copy_to_tensor_parallel_region = comm.copy_to_tensor_parallel_region
reduce_from_tensor_parallel_region = comm.reduce_from_tensor_parallel_region
scatter_to_sequence_parallel_region = comm.scatter_to_sequence_parallel_region
gather_from_sequence_parallel_region = comm.gather_from_sequence_parallel_region


def _resolver(precision_resolver):
    return precision_resolver if precision_resolver is not None else _default_precision_resolver()


class Linear(LowBitLinearMixin, nn.Module):
    """y = x W^T + b with W [out, in] ~ N(0, 0.02), b = 0."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, *,
                 param_dtype: torch.dtype = torch.float32, param_device: Optional[torch.device] = None,
                 module_path: str = "linear", precision_resolver=None, init_std: float = 0.02):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=param_dtype, device=param_device))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, dtype=param_dtype, device=param_device))
        else:
            self.register_parameter("bias", None)
        if self.weight.device.type != "meta":
            nn.init.normal_(self.weight, std=init_std)
            if self.bias is not None:
                nn.init.zeros_(self.bias)
        self._init_lowbit_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver),
                                          lowbit_capable_type="linear", in_features=in_features,
                                          out_features=out_features, has_bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._linear(x, self.bias)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


class ColumnParallelLinear(LowBitLinearMixin, nn.Module):
    """Output-sharded linear: W shard [out/tp, in].

    Without sequence parallelism the input is replicated and its gradient is
    all-reduced (reference semantics). With ``sequence_parallel=True`` the
    input is the local sequence shard and the layer runs the fused
    all-gather -> GEMM path.
    """

    def __init__(self, in_features: int, out_features: int, tp_rank: int = 0, tp_size: int = 1, bias: bool = True,
                 tp_group=None, *, param_dtype: torch.dtype = torch.float32,
                 param_device: Optional[torch.device] = None, module_path: str = "column_parallel_linear",
                 precision_resolver=None, sequence_parallel: bool = False, gather_output: bool = False,
                 init_std: float = 0.02):
        super().__init__()
        if out_features % tp_size != 0:
            raise ValueError(f"out_features {out_features} must be divisible by tp_size {tp_size}")
        self.in_features = in_features
        self.out_features = out_features
        self.tp_rank = tp_rank
        self.tp_size = tp_size
        self.tp_group = tp_group if tp_group is not None else (
            dist.group.WORLD if dist.is_available() and dist.is_initialized() else None)
        self.shard_size = out_features // tp_size
        self.sequence_parallel = sequence_parallel
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(self.shard_size, in_features, dtype=param_dtype, device=param_device))
        if bias:
            self.bias = nn.Parameter(torch.empty(self.shard_size, dtype=param_dtype, device=param_device))
        else:
            self.register_parameter("bias", None)
        if self.weight.device.type != "meta":
            nn.init.normal_(self.weight, std=init_std)
            if self.bias is not None:
                nn.init.zeros_(self.bias)
        self.weight.tensor_model_parallel = True
        self.weight.partition_dim = 0
        if self.bias is not None:
            self.bias.tensor_model_parallel = True
            self.bias.partition_dim = 0
        self._init_lowbit_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver),
                                          lowbit_capable_type="column_parallel_linear", in_features=in_features,
                                          out_features=self.shard_size, has_bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sequence_parallel and self.tp_size > 1 and not self._lowbit_active():
            lead = x.shape[:-1]
            y = column_parallel_linear_sp(x.reshape(-1, x.shape[-1]), self._effective_weight(), self.bias,
                                          self.tp_group)
            return y.view(-1, *lead[1:], self.shard_size) if len(lead) > 1 else y
        if self.tp_size > 1:
            x = comm.copy_to_tensor_parallel_region(x, self.tp_group)
        y = self._linear(x, self.bias)
        if self.gather_output and self.tp_size > 1:
            y = comm.gather_along_seq(y.movedim(-1, 0).contiguous(), self.tp_group, 0).movedim(0, -1)
        return y


class RowParallelLinear(LowBitLinearMixin, nn.Module):
    """Input-sharded linear: W shard [out, in/tp]; partial outputs are summed across TP.

    With ``sequence_parallel=True`` the sum is a reduce-scatter along the
    token dimension fused with the GEMM, and the output is the local
    sequence shard.
    """

    def __init__(self, in_features: int, out_features: int, tp_rank: int = 0, tp_size: int = 1, bias: bool = True,
                 tp_group=None, *, param_dtype: torch.dtype = torch.float32,
                 param_device: Optional[torch.device] = None, module_path: str = "row_parallel_linear",
                 precision_resolver=None, sequence_parallel: bool = False, init_std: float = 0.02):
        super().__init__()
        if in_features % tp_size != 0:
            raise ValueError(f"in_features {in_features} must be divisible by tp_size {tp_size}")
        self.in_features = in_features
        self.out_features = out_features
        self.tp_rank = tp_rank
        self.tp_size = tp_size
        self.tp_group = tp_group if tp_group is not None else (
            dist.group.WORLD if dist.is_available() and dist.is_initialized() else None)
        self.shard_size = in_features // tp_size
        self.sequence_parallel = sequence_parallel
        self.weight = nn.Parameter(torch.empty(out_features, self.shard_size, dtype=param_dtype, device=param_device))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, dtype=param_dtype, device=param_device))
        else:
            self.register_parameter("bias", None)
        if self.weight.device.type != "meta":
            nn.init.normal_(self.weight, std=init_std)
            if self.bias is not None:
                nn.init.zeros_(self.bias)
        self.weight.tensor_model_parallel = True
        self.weight.partition_dim = 1
        self._init_lowbit_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver),
                                          lowbit_capable_type="row_parallel_linear", in_features=self.shard_size,
                                          out_features=out_features, has_bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sequence_parallel and self.tp_size > 1 and not self._lowbit_active():
            lead = x.shape[:-1]
            y = row_parallel_linear_sp(x.reshape(-1, x.shape[-1]), self._effective_weight(), self.bias,
                                       self.tp_group)
            return y.view(-1, *lead[1:], self.out_features) if len(lead) > 1 else y
        y = self._linear(x, None)
        if self.tp_size > 1:
            y = comm.reduce_from_tensor_parallel_region(y, self.tp_group)
        if self.bias is not None:
            y = y + self.bias
        return y


class LayerNorm(ModulePrecisionStateMixin, nn.Module):
    """(x - mean) / sqrt(var + eps) * w + b with biased variance."""

    def __init__(self, normalized_shape: int, eps: float = 1e-5, *, param_dtype: torch.dtype = torch.float32,
                 param_device: Optional[torch.device] = None, module_path: str = "layernorm",
                 precision_resolver=None, bias: bool = True):
        super().__init__()
        self.normalized_shape = normalized_shape
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(normalized_shape, dtype=param_dtype, device=param_device))
        if bias:
            self.bias = nn.Parameter(torch.zeros(normalized_shape, dtype=param_dtype, device=param_device))
        else:
            self.register_parameter("bias", None)
        self._init_module_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = self._module_compute_dtype_override()
        if dt is not None:  # the override is the compute and the output dtype
            return ops.layer_norm(x.to(dt), self.weight.to(dt), None if self.bias is None else self.bias.to(dt),
                                  self.eps)
        return ops.layer_norm(x, self.weight, self.bias, self.eps)


class RMSNorm(ModulePrecisionStateMixin, nn.Module):
    """x * rsqrt(mean(x^2) + eps) * w (reference: src/models/deepseek.py:386-438)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, *, param_dtype: torch.dtype = torch.float32,
                 param_device: Optional[torch.device] = None, module_path: str = "rmsnorm",
                 precision_resolver=None, compute_dtype: Optional[torch.dtype] = None):
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.compute_dtype = compute_dtype
        self.weight = nn.Parameter(torch.ones(hidden_size, dtype=param_dtype, device=param_device))
        self._init_module_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = self.compute_dtype or self._module_compute_dtype_override()
        if dt is not None:  # the override is the compute and the output dtype
            return ops.rms_norm(x.to(dt), self.weight.to(dt), self.eps)
        return ops.rms_norm(x, self.weight.to(x.dtype), self.eps)

    def forward_residual(self, x: torch.Tensor, residual: torch.Tensor):
        """Returns (norm(x + residual), x + residual) in one pass."""
        return ops.add_rms_norm(x, residual, self.weight.to(x.dtype), self.eps)


class Embedding(ModulePrecisionStateMixin, nn.Module):
    """Token lookup table [num_embeddings, dim] ~ N(0, 0.02)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, *, param_dtype: torch.dtype = torch.float32,
                 param_device: Optional[torch.device] = None, module_path: str = "embedding",
                 precision_resolver=None, init_std: float = 0.02):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim, dtype=param_dtype,
                                               device=param_device))
        if self.weight.device.type != "meta":
            nn.init.normal_(self.weight, std=init_std)
        self._init_module_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver))

    def forward(self, indices: torch.Tensor) -> torch.Tensor:
        return ops.embedding(indices, self.weight)


class VocabParallelEmbedding(ModulePrecisionStateMixin, nn.Module):
    """Vocab-sharded embedding: rank r holds rows [r V/tp, (r+1) V/tp).

    The partial lookups are summed across TP (all-reduce), or reduce-scattered
    along the token dimension under sequence parallelism.
    """

    def __init__(self, num_embeddings: int, embedding_dim: int, tp_rank: int = 0, tp_size: int = 1, tp_group=None,
                 *, param_dtype: torch.dtype = torch.float32, param_device: Optional[torch.device] = None,
                 module_path: str = "embedding", precision_resolver=None, sequence_parallel: bool = False,
                 init_std: float = 0.02):
        super().__init__()
        if num_embeddings % tp_size != 0:
            raise ValueError(f"vocab {num_embeddings} must be divisible by tp_size {tp_size}")
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.tp_group = tp_group
        self.sequence_parallel = sequence_parallel
        self.shard = num_embeddings // tp_size
        self.vocab_start = tp_rank * self.shard
        self.weight = nn.Parameter(torch.empty(self.shard, embedding_dim, dtype=param_dtype, device=param_device))
        if self.weight.device.type != "meta":
            nn.init.normal_(self.weight, std=init_std)
        self.weight.tensor_model_parallel = True
        self.weight.partition_dim = 0
        self._init_module_precision_state(module_path=module_path, module_type=type(self).__name__,
                                          precision_resolver=_resolver(precision_resolver))

    def forward(self, indices: torch.Tensor) -> torch.Tensor:
        out = ops.embedding(indices, self.weight, self.vocab_start)
        if self.tp_size == 1:
            return out
        if self.sequence_parallel:
            return comm.reduce_scatter_along_seq(out, self.tp_group, 0)
        return comm.reduce_from_tensor_parallel_region(out, self.tp_group)


class Dropout(nn.Module):
    """Inverted dropout; identity when p == 0 or in eval mode. On CUDA the mask comes from a
    counter-based generator inside one kernel and is regenerated in the backward pass
    (``ops/dropout.py``); on CPU it is a bernoulli draw."""

    def __init__(self, p: float = 0.5):
        super().__init__()
        if p < 0 or p > 1:
            raise ValueError(f"dropout probability has to be between 0 and 1, but got {p}")
        self.p = p

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.training or self.p == 0.0:
            return x
        if self.p == 1.0:
            return torch.zeros_like(x)
        if x.is_cuda:
            from .ops.dropout import dropout

            return dropout(x, self.p)
        mask = torch.empty_like(x).bernoulli_(1.0 - self.p)
        return x * mask / (1.0 - self.p)


class GELU(nn.Module):
    """Exact GELU x * Phi(x)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.gelu(x)


def clip_grad_norm(parameters, max_norm: float) -> float:
    """Scale gradients in place so that their global L2 norm is at most ``max_norm``.

    Returns the pre-clip norm. One fused sum-of-squares launch per gradient on
    CUDA and a single host read (the reference reads one scalar per parameter).
    """
    if isinstance(parameters, torch.Tensor):
        parameters = [parameters]
    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        return 0.0
    dev = grads[0].device
    acc = torch.zeros(2, dtype=torch.float32, device=dev)
    for g in grads:
        if g.is_cuda and g.is_contiguous():
            ops.grad_stats_(g, acc)
        else:
            acc[0] += g.float().pow(2).sum()
    total = math.sqrt(float(acc[0].item()))
    coef = max_norm / (total + 1e-6)
    if coef < 1.0:
        for g in grads:
            g.mul_(coef)
    return total
