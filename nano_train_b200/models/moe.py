"""Routed mixture-of-experts: SwiGLU experts, DeepSeek top-k router, local and
expert-parallel MoE.

Semantics follow the reference (src/models/moe.py):
* ``TopKRouter`` (196-350): linear router -> sigmoid or fp32 softmax ->
  group-limited mask (group score = max inside the group, keep the top
  ``topk_group`` groups) -> top-k -> renormalise (sigmoid + norm_topk_prob) or
  re-softmax the top-k (softmax) -> x routed_scaling_factor; auxiliary loss
  N * sum_i f_i P_i.
* capacity ``ceil(capacity_factor * T * K / E)`` per expert, dropping the
  lowest-weight assignments; shared experts are averaged (353-509).
* ``ExpertParallelMoE``: experts split over the EP group, tokens dispatched
  and combined with all-to-all (512-1146), optional fp8 payload quantisation.

Implementation (B200 build): routing, capacity selection and the permutation
run as device-side sorts (no per-expert Python loop over nonzero()), experts
run as one grouped pass over tokens sorted by expert, and the dispatch /
combine exchange their per-rank counts once per layer.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..layers import Dropout, Linear
from ..ops.grouped import _StackCache, grouped_kernel_ok, grouped_swiglu_experts
from ..precision.backends import fp8_quant_dequant, quantize_dequantize


@dataclass
class RouterOutput:
    topk_indices: torch.Tensor
    topk_weights: torch.Tensor
    aux_loss: torch.Tensor
    dropped_fraction: float = 0.0


class ExpertMLP(nn.Module):
    """down(silu(gate(x)) * up(x)), no biases."""

    def __init__(self, hidden_size: int, intermediate_size: int, dropout: float = 0.0, *, param_dtype=torch.float32,
                 param_device=None, precision_resolver=None, module_prefix: str = "expert"):
        super().__init__()
        kw = dict(param_dtype=param_dtype, param_device=param_device, precision_resolver=precision_resolver)
        self.gate_proj = Linear(hidden_size, intermediate_size, bias=False, module_path=f"{module_prefix}.gate_proj",
                                **kw)
        self.up_proj = Linear(hidden_size, intermediate_size, bias=False, module_path=f"{module_prefix}.up_proj",
                              **kw)
        self.down_proj = Linear(intermediate_size, hidden_size, bias=False, module_path=f"{module_prefix}.down_proj",
                                **kw)
        self.dropout = Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and not self.gate_proj._lowbit_active() and not self.up_proj._lowbit_active():
            # One GEMM over the stacked gate|up weights + the fused SwiGLU kernel.
            w = torch.cat([self.gate_proj._effective_weight(), self.up_proj._effective_weight()], 0)
            h = ops.swiglu(ops.linear(x, w.to(x.dtype)))
        else:
            h = F.silu(self.gate_proj(x)) * self.up_proj(x)
        return self.dropout(self.down_proj(h))


class _RouterFn(torch.autograd.Function):
    """Fused router kernel (csrc/router.cu): scores, group-limited top-k, weight normalisation,
    per-expert counts and aux-loss probability sums in one launch; one launch for the backward."""

    @staticmethod
    def forward(ctx, logits, cfg):
        idx, w, counts, psum = ops.ext().router_fwd(logits, *cfg)
        ctx.save_for_backward(logits, idx)
        ctx.cfg = cfg
        ctx.mark_non_differentiable(idx, counts)
        return w, idx, counts, psum

    @staticmethod
    def backward(ctx, dw, _didx, _dcounts, dpsum):
        logits, idx = ctx.saved_tensors
        if dw is None:
            dw = torch.zeros(idx.shape, dtype=logits.dtype, device=logits.device)
        if dpsum is None:
            dpsum = torch.zeros(logits.shape[1], dtype=torch.float32, device=logits.device)
        return ops.ext().router_bwd(logits, idx, dw.contiguous().to(logits.dtype), dpsum.contiguous().float(),
                                    *ctx.cfg), None


class TopKRouter(nn.Module):
    def __init__(self, hidden_size: int, num_experts: int, top_k: int, *, param_dtype=torch.float32,
                 param_device=None, precision_resolver=None, module_prefix: str = "router",
                 scoring_func: str = "sigmoid", n_group: int = 1, topk_group: int = 1, norm_topk_prob: bool = True,
                 routed_scaling_factor: float = 1.0):
        super().__init__()
        if num_experts <= 0:
            raise ValueError("num_experts must be positive")
        if top_k <= 0 or top_k > num_experts:
            raise ValueError("top_k must be in [1, num_experts]")
        if scoring_func not in {"sigmoid", "softmax"}:
            raise ValueError("scoring_func must be 'sigmoid' or 'softmax'")
        if n_group <= 0 or num_experts % n_group != 0:
            raise ValueError("n_group must divide num_experts")
        if topk_group <= 0 or topk_group > n_group:
            raise ValueError("topk_group must be in [1, n_group]")
        if topk_group * (num_experts // n_group) < top_k:
            raise ValueError("topk_group exposes fewer experts than top_k")
        self.num_experts, self.top_k = num_experts, top_k
        self.scoring_func, self.n_group, self.topk_group = scoring_func, n_group, topk_group
        self.norm_topk_prob = norm_topk_prob
        self.routed_scaling_factor = routed_scaling_factor
        self.router = Linear(hidden_size, num_experts, bias=False, param_dtype=param_dtype, param_device=param_device,
                             module_path=f"{module_prefix}.router", precision_resolver=precision_resolver)

    def _kernel_ok(self, logits: torch.Tensor) -> bool:
        import os

        return (logits.is_cuda and logits.dtype in (torch.bfloat16, torch.float32) and self.num_experts <= 512
                and self.top_k <= 8 and self.n_group <= 32 and os.environ.get("NTB_ROUTER_KERNEL", "1") != "0")

    def _forward_kernel(self, logits: torch.Tensor) -> RouterOutput:
        T = logits.shape[0]
        cfg = (self.top_k, self.scoring_func == "softmax", self.n_group, self.topk_group, self.norm_topk_prob,
               float(self.routed_scaling_factor))
        w, idx, counts, psum = _RouterFn.apply(logits.contiguous(), cfg)
        frac = counts.float() / float(T * self.top_k)
        aux = ((frac * (psum / float(T))).sum() * float(self.num_experts)).to(logits.dtype)
        return RouterOutput(idx, w, aux, 0.0)

    def _score_experts(self, logits: torch.Tensor) -> torch.Tensor:
        if self.scoring_func == "sigmoid":
            return torch.sigmoid(logits)
        return torch.softmax(logits.float(), dim=-1).to(logits.dtype)

    def _apply_group_routing(self, scores: torch.Tensor) -> torch.Tensor:
        if self.n_group <= 1 or self.topk_group >= self.n_group:
            return scores
        T = scores.size(0)
        epg = self.num_experts // self.n_group
        gscore = scores.view(T, self.n_group, epg).max(dim=-1).values
        keep = torch.zeros_like(gscore, dtype=torch.bool)
        keep.scatter_(1, torch.topk(gscore, k=self.topk_group, dim=-1).indices, True)
        mask = keep.unsqueeze(-1).expand(-1, -1, epg).reshape(T, self.num_experts)
        fill = torch.zeros_like(scores) if self.scoring_func == "sigmoid" else torch.full_like(scores, float("-inf"))
        return torch.where(mask, scores, fill)

    def _compute_aux_loss(self, scores: torch.Tensor, topk_indices: torch.Tensor) -> torch.Tensor:
        if scores.numel() == 0:
            return torch.zeros((), dtype=scores.dtype, device=scores.device)
        normed = scores / torch.clamp(scores.sum(-1, keepdim=True), min=1e-9) if self.scoring_func == "sigmoid" \
            else scores
        counts = torch.zeros(self.num_experts, dtype=torch.float32, device=scores.device)
        counts.scatter_add_(0, topk_indices.reshape(-1), torch.ones(topk_indices.numel(), device=scores.device))
        frac = counts / float(topk_indices.numel())
        prob = normed.float().mean(0)
        return ((frac * prob).sum() * float(self.num_experts)).to(scores.dtype)

    def forward(self, tokens: torch.Tensor) -> RouterOutput:
        if tokens.dim() != 2:
            raise ValueError("tokens must have shape [num_tokens, hidden_size]")
        if tokens.size(0) == 0:
            z = torch.zeros((0, self.top_k), device=tokens.device)
            return RouterOutput(z.long(), z.to(tokens.dtype), torch.zeros((), dtype=tokens.dtype,
                                                                           device=tokens.device), 0.0)
        logits = self.router(tokens)
        if self._kernel_ok(logits):
            return self._forward_kernel(logits)
        scores = self._score_experts(logits)
        routed = self._apply_group_routing(scores)
        w, idx = torch.topk(routed, k=self.top_k, dim=-1)
        if self.scoring_func == "sigmoid" and self.norm_topk_prob:
            w = w / torch.clamp(w.sum(-1, keepdim=True), min=1e-9)
        elif self.scoring_func == "softmax":
            w = torch.softmax(w.float(), dim=-1).to(w.dtype)
        w = w * self.routed_scaling_factor
        return RouterOutput(idx, w, self._compute_aux_loss(scores, idx), 0.0)


def capacity_select(topk_indices: torch.Tensor, topk_weights: torch.Tensor, num_experts: int, capacity: int):
    """Device-side capacity filter.

    Returns (token_idx, slot_idx, expert_idx) of the kept assignments sorted by
    expert (descending weight inside an expert) and the per-expert kept counts.
    Each expert keeps its ``capacity`` highest-weight assignments.
    """
    T, K = topk_indices.shape
    flat_e = topk_indices.reshape(-1)
    flat_w = topk_weights.detach().reshape(-1).float()
    order_w = torch.argsort(flat_w, descending=True, stable=True)
    order = order_w[torch.argsort(flat_e[order_w], stable=True)]
    e_sorted = flat_e[order]
    counts = torch.bincount(e_sorted, minlength=num_experts)
    starts = torch.cumsum(counts, 0) - counts
    rank = torch.arange(order.numel(), device=order.device) - starts[e_sorted]
    keep = rank < capacity if capacity > 0 else torch.ones_like(rank, dtype=torch.bool)
    kept = order[keep]
    kept_counts = torch.bincount(e_sorted[keep], minlength=num_experts)
    return kept // K, kept % K, e_sorted[keep], kept_counts


def run_experts_grouped(experts: nn.ModuleList, x_sorted: torch.Tensor, counts: list[int]) -> torch.Tensor:
    """Apply expert e to its contiguous block of ``x_sorted`` rows (rows grouped by expert)."""
    outs = []
    off = 0
    for e, n in enumerate(counts):
        if n:
            outs.append(experts[e](x_sorted[off: off + n]))
        off += n
    if not outs:
        return x_sorted.new_zeros((0, x_sorted.shape[-1]))
    return torch.cat(outs, 0)


class LocalRoutedMoE(nn.Module):
    def __init__(self, hidden_size: int, expert_intermediate_size: int, num_experts: int, top_k: int, *,
                 param_dtype=torch.float32, param_device=None, precision_resolver=None, module_prefix: str = "moe",
                 dropout: float = 0.0, n_shared_experts: int = 0, scoring_func: str = "sigmoid", n_group: int = 1,
                 topk_group: int = 1, norm_topk_prob: bool = True, routed_scaling_factor: float = 1.0,
                 capacity_factor: float = 1.0):
        super().__init__()
        if capacity_factor <= 0:
            raise ValueError("capacity_factor must be positive")
        self.hidden_size, self.num_experts, self.top_k = hidden_size, num_experts, top_k
        self.capacity_factor = capacity_factor
        kw = dict(param_dtype=param_dtype, param_device=param_device, precision_resolver=precision_resolver)
        self.router = TopKRouter(hidden_size, num_experts, top_k, module_prefix=f"{module_prefix}.router",
                                 scoring_func=scoring_func, n_group=n_group, topk_group=topk_group,
                                 norm_topk_prob=norm_topk_prob, routed_scaling_factor=routed_scaling_factor, **kw)
        self.experts = nn.ModuleList([ExpertMLP(hidden_size, expert_intermediate_size, dropout,
                                                module_prefix=f"{module_prefix}.experts.{i}", **kw)
                                      for i in range(num_experts)])
        self.shared_experts = nn.ModuleList([ExpertMLP(hidden_size, expert_intermediate_size, dropout,
                                                       module_prefix=f"{module_prefix}.shared_experts.{i}", **kw)
                                             for i in range(n_shared_experts)])
        self._last_aux_loss = torch.zeros(())
        self._last_dropped_fraction = 0.0
        self._last_token_counts = torch.zeros(num_experts, dtype=torch.long)
        self._stack_cache = _StackCache()

    def _compute_capacity(self, num_tokens: int) -> int:
        if num_tokens <= 0:
            return 0
        return max(int(math.ceil(self.capacity_factor * (num_tokens * self.top_k) / float(self.num_experts))), 1)

    @property
    def last_aux_loss(self) -> torch.Tensor:
        return self._last_aux_loss

    @property
    def last_dropped_fraction(self) -> float:
        """Dropped fraction of the last forward; read from the device (once) when asked for."""
        d = self._last_dropped_fraction
        if isinstance(d, torch.Tensor):
            d = float(d)
            self._last_dropped_fraction = d
        return d

    @property
    def last_dropped_fraction_tensor(self) -> torch.Tensor:
        """Dropped fraction of the last forward as a scalar tensor, with no host synchronisation."""
        d = self._last_dropped_fraction
        return d if isinstance(d, torch.Tensor) else torch.tensor(float(d))

    @property
    def last_token_counts(self) -> torch.Tensor:
        return self._last_token_counts

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 3:
            raise ValueError("x must have shape [batch, seq, hidden]")
        B, S, H = x.shape
        if H != self.hidden_size:
            raise ValueError("hidden dimension mismatch")
        tokens = x.reshape(-1, H)
        ro = self.router(tokens)
        cap = self._compute_capacity(tokens.size(0))
        tok, slot, _, counts = capacity_select(ro.topk_indices, ro.topk_weights, self.num_experts, cap)
        if grouped_kernel_ok(tokens, self.experts):
            # One grouped tcgen05 GEMM per matrix over all experts, no host sync on the counts.
            y = grouped_swiglu_experts(tokens[tok], counts, self.experts, self._stack_cache,
                                       max_rows=ro.topk_indices.numel() + self.num_experts * 127)
        else:
            y = run_experts_grouped(self.experts, tokens[tok], counts.tolist())
        w = ro.topk_weights[tok, slot].unsqueeze(-1)
        out = torch.zeros_like(tokens).index_add(0, tok, (y * w).to(tokens.dtype))
        if len(self.shared_experts):
            shared = sum(se(tokens) for se in self.shared_experts)
            out = out + shared / float(len(self.shared_experts))
        total = ro.topk_indices.numel()
        self._last_aux_loss = ro.aux_loss
        self._last_dropped_fraction = (total - counts.sum()).float() / float(max(total, 1))  # read lazily
        self._last_token_counts = counts
        return out.view(B, S, H)


# ------------------------------------------------------------------ expert parallel
def _comm_quant_dequant(x: torch.Tensor, granularity: Optional[str] = None, rounding_mode: str = "nearest",
                        backend: str = "emulated", *, bits: int = 8) -> torch.Tensor:
    """Payload quantisation for the dispatch/combine exchange (straight-through; shape and dtype kept).

    A payload row is one token, so the 128x128 block of the recipe is applied as 1x128 tiles: each
    row keeps its own scales and can be quantised where it is sent (the fused dispatch does exactly
    this in flight)."""
    if granularity in (None, "none") or x.numel() == 0:
        return x
    gran = {"block_128x128": "tile_1x128"}.get(granularity, granularity)
    if backend == "native" and bits == 8:
        dq = fp8_quant_dequant(x.detach(), granularity=gran, rounding_mode=rounding_mode, channel_axis=-1)
    else:
        dq = quantize_dequantize(x.detach(), bits=bits, granularity=gran, rounding_mode=rounding_mode,
                                 channel_axis=-1)
    return x + (dq.to(x.dtype) - x).detach()


_UNSET = object()


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_splits, recv_splits, group):
        ctx.group, ctx.send, ctx.recv = group, send_splits, recv_splits
        out = x.new_empty((sum(recv_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((sum(ctx.send),) + tuple(g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


class ExpertParallelMoE(nn.Module):
    """Experts [ep_rank * E/ep, (ep_rank+1) * E/ep) live on this rank; tokens travel by all-to-all."""

    def __init__(self, hidden_size: int, expert_intermediate_size: int, num_experts: int, top_k: int, *,
                 ep_rank: int, ep_size: int, ep_group=None, expert_tp_size: int = 1, param_dtype=torch.float32,
                 param_device=None, precision_resolver=None, module_prefix: str = "moe", dropout: float = 0.0,
                 n_shared_experts: int = 0, scoring_func: str = "sigmoid", n_group: int = 1, topk_group: int = 1,
                 norm_topk_prob: bool = True, routed_scaling_factor: float = 1.0, capacity_factor: float = 1.0,
                 comm_quant_granularity=_UNSET, comm_quant_rounding: Optional[str] = None,
                 comm_quant_backend: str = "emulated"):
        super().__init__()
        if expert_tp_size != 1:
            raise ValueError("expert_tp_size must be 1")
        if num_experts % ep_size != 0:
            raise ValueError("num_experts must be divisible by ep_size")
        self.hidden_size, self.num_experts, self.top_k = hidden_size, num_experts, top_k
        self.ep_rank, self.ep_size, self.ep_group = ep_rank, ep_size, ep_group
        self.experts_per_rank = num_experts // ep_size
        self.global_expert_start = ep_rank * self.experts_per_rank
        self.capacity_factor = capacity_factor
        # Payload quantisation: explicit arguments win; otherwise the DeepSeek-V3 recipe of the
        # precision resolver decides (on, block_128x128, its rounding mode), as in the reference.
        recipe_fn = getattr(precision_resolver, "deepseek_v3_recipe", None)
        recipe = recipe_fn() if callable(recipe_fn) else None
        if comm_quant_granularity is _UNSET:
            comm_quant_granularity = (str(recipe.comm_quant_granularity)
                                      if recipe is not None and recipe.comm_quant_enabled else None)
        if comm_quant_rounding is None:
            comm_quant_rounding = str(recipe.rounding_mode) if recipe is not None else "nearest"
        self.comm_quant_granularity = comm_quant_granularity
        self.comm_quant_rounding = comm_quant_rounding
        self.comm_quant_backend = comm_quant_backend
        kw = dict(param_dtype=param_dtype, param_device=param_device, precision_resolver=precision_resolver)
        self.router = TopKRouter(hidden_size, num_experts, top_k, module_prefix=f"{module_prefix}.router",
                                 scoring_func=scoring_func, n_group=n_group, topk_group=topk_group,
                                 norm_topk_prob=norm_topk_prob, routed_scaling_factor=routed_scaling_factor, **kw)
        first = ep_rank * self.experts_per_rank
        self.experts = nn.ModuleList([ExpertMLP(hidden_size, expert_intermediate_size, dropout,
                                                module_prefix=f"{module_prefix}.experts.{first + i}", **kw)
                                      for i in range(self.experts_per_rank)])
        for p in self.experts.parameters():
            p.expert_model_parallel = True
        self.shared_experts = nn.ModuleList([ExpertMLP(hidden_size, expert_intermediate_size, dropout,
                                                       module_prefix=f"{module_prefix}.shared_experts.{i}", **kw)
                                             for i in range(n_shared_experts)])
        self._last_aux_loss = torch.zeros(())
        self._last_dropped_fraction = 0.0
        self._last_token_counts = torch.zeros(self.experts_per_rank, dtype=torch.long)
        self._stack_cache = _StackCache()
        self.last_path = None  # "fused" (peer-memory kernels) or "all_to_all", set by forward
        self.fused_rel_err: Optional[float] = None  # first fused call's error against the all-to-all path

    last_aux_loss = property(lambda self: self._last_aux_loss)
    last_token_counts = property(lambda self: self._last_token_counts)
    last_local_expert_counts = property(lambda self: self._last_token_counts)
    _comm_quant_enabled = property(lambda self: self.comm_quant_granularity not in (None, "none"))
    _comm_quant_granularity = property(lambda self: self.comm_quant_granularity or "tensor")
    _comm_quant_rounding_mode = property(lambda self: self.comm_quant_rounding)

    @property
    def last_dropped_fraction(self) -> float:
        """Dropped fraction of the last forward over the EP group; the device statistics
        (dropped, routed) are read only when asked for."""
        d = self._last_dropped_fraction
        if isinstance(d, torch.Tensor):
            s = d.tolist()
            d = float(s[0] / max(s[1], 1.0))
            self._last_dropped_fraction = d
        return d

    @property
    def last_dropped_fraction_tensor(self) -> torch.Tensor:
        """Dropped fraction of the last forward as a scalar tensor, with no host synchronisation."""
        d = self._last_dropped_fraction
        if isinstance(d, torch.Tensor):
            return d[0] / d[1].clamp_min(1.0)
        return torch.tensor(float(d))

    def _fused_payload(self):
        """(use the fused kernels, e4m3 payload) for this layer's settings."""
        g = self.comm_quant_granularity
        if g in (None, "none"):
            return True, False
        if self.comm_quant_backend == "native" and g in ("tile_1x128", "block_128x128") \
                and self.hidden_size % 128 == 0:
            return True, True
        return False, False  # emulated payload numerics stay on the all-to-all path

    def _fused_ok(self, tokens: torch.Tensor) -> bool:
        if not (tokens.is_cuda and tokens.dtype == torch.bfloat16 and self.top_k <= 8 and tokens.shape[0] > 0
                and self.hidden_size % 8 == 0):
            return False
        from ..parallel.ep_fused import fused_ep_enabled

        return fused_ep_enabled(self.ep_group) and grouped_kernel_ok(tokens, self.experts) and self._fused_payload()[0]

    def _compute_capacity(self, global_tokens: int) -> int:
        if global_tokens <= 0:
            return 0
        return max(int(math.ceil(self.capacity_factor * global_tokens * self.top_k / float(self.num_experts))), 1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 3:
            raise ValueError("x must have shape [batch, seq, hidden]")
        B, S, H = x.shape
        tokens = x.reshape(-1, H)
        T = tokens.size(0)
        ro = self.router(tokens)
        if self._fused_ok(tokens):
            out = self._forward_fused(tokens, ro)
            if self.fused_rel_err is None:
                self._check_fused_against_all_to_all(tokens, ro, out)
            return out.view(B, S, H)
        return self._forward_all_to_all(tokens, ro).view(B, S, H)

    FUSED_REL_TOL = {False: 2e-2, True: 1e-1}  # by e4m3 payload (independent rounding of the two paths)

    @torch.no_grad()
    def _check_fused_against_all_to_all(self, tokens: torch.Tensor, ro: RouterOutput, out: torch.Tensor) -> None:
        """First fused call of this layer: the all-to-all path recomputes the same layer output from
        the same routing; the relative L2 error (max over the EP group) is kept in
        ``fused_rel_err`` and a disagreement beyond tolerance raises. Runs once per layer, inside
        every multi-GPU job that takes the fused path."""
        saved = (self._last_aux_loss, self._last_dropped_fraction, self._last_token_counts, self.last_path)
        ref = self._forward_all_to_all(tokens.detach(), ro).float()
        self._last_aux_loss, self._last_dropped_fraction, self._last_token_counts, self.last_path = saved
        err = ((out.detach().float() - ref).norm() / ref.norm().clamp_min(1e-30)).reshape(1)
        dist.all_reduce(err, op=dist.ReduceOp.MAX, group=self.ep_group)
        self.fused_rel_err = float(err)
        tol = self.FUSED_REL_TOL[self._fused_payload()[1]]
        if not self.fused_rel_err <= tol:
            raise RuntimeError(f"fused expert-parallel output differs from the all-to-all path: relative error "
                               f"{self.fused_rel_err:.3e} > {tol}")

    def _forward_all_to_all(self, tokens: torch.Tensor, ro: RouterOutput) -> torch.Tensor:
        """Dispatch / experts / combine with NCCL all-to-all (one host read of the split sizes)."""
        T, H = tokens.shape
        self.last_path = "all_to_all"
        E, epr, K = self.num_experts, self.experts_per_rank, self.top_k
        # Assignments sorted by destination expert (hence by destination rank).
        flat_e = ro.topk_indices.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        dest_e = flat_e[order]
        send_counts = torch.bincount(dest_e // epr, minlength=self.ep_size)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.ep_group)
        t_all = torch.full((self.ep_size,), T, dtype=send_counts.dtype, device=tokens.device)
        dist.all_reduce(t_all, group=self.ep_group)  # each entry becomes the global token count
        # One host read per layer: the splits NCCL needs and the global token count (capacity).
        cnt = torch.stack([send_counts, recv_counts, t_all]).tolist()
        send_splits, recv_splits = cnt[0], cnt[1]
        capacity = self._compute_capacity(int(cnt[2][0]))
        tok_idx = order // K
        slot_idx = order % K
        payload = _comm_quant_dequant(tokens[tok_idx], self.comm_quant_granularity, self.comm_quant_rounding,
                                      self.comm_quant_backend)
        meta = dest_e.unsqueeze(1).contiguous()
        recv_x = _AllToAll.apply(payload, send_splits, recv_splits, self.ep_group)
        recv_meta = torch.empty((sum(recv_splits), 1), dtype=meta.dtype, device=meta.device)
        w_sorted = ro.topk_weights.detach().reshape(-1)[order].float()
        dist.all_to_all_single(recv_meta, meta.contiguous(), recv_splits, send_splits, group=self.ep_group)
        recv_w = torch.empty(sum(recv_splits), dtype=torch.float32, device=tokens.device)
        dist.all_to_all_single(recv_w, w_sorted.contiguous(), recv_splits, send_splits, group=self.ep_group)
        local_e = recv_meta[:, 0] - self.ep_rank * epr
        # Capacity per local expert over every source rank: keep highest-weight assignments.
        o1 = torch.argsort(recv_w, descending=True, stable=True)
        o2 = o1[torch.argsort(local_e[o1], stable=True)]
        le_sorted = local_e[o2]
        counts = torch.bincount(le_sorted, minlength=epr)
        starts = torch.cumsum(counts, 0) - counts
        rank_in = torch.arange(o2.numel(), device=o2.device) - starts[le_sorted]
        keep = rank_in < capacity
        kept = o2[keep]
        kept_counts = torch.bincount(le_sorted[keep], minlength=epr)
        if grouped_kernel_ok(recv_x, self.experts):
            y_kept = grouped_swiglu_experts(recv_x[kept], kept_counts, self.experts, self._stack_cache,
                                            max_rows=recv_x.shape[0] + epr * 127)
        else:
            y_kept = run_experts_grouped(self.experts, recv_x[kept], kept_counts.tolist())
        y_back = torch.zeros_like(recv_x).index_copy(0, kept, y_kept.to(recv_x.dtype))
        y_back = _comm_quant_dequant(y_back, self.comm_quant_granularity, self.comm_quant_rounding,
                                     self.comm_quant_backend)
        y_src = _AllToAll.apply(y_back, recv_splits, send_splits, self.ep_group)
        w = ro.topk_weights.reshape(-1)[order].unsqueeze(-1)
        out = torch.zeros_like(tokens).index_add(0, tok_idx, (y_src * w).to(tokens.dtype))
        del slot_idx
        if len(self.shared_experts):
            out = out + sum(se(tokens) for se in self.shared_experts) / float(len(self.shared_experts))
        stats = torch.tensor([float(recv_w.numel() - kept.numel()), float(recv_w.numel())], device=tokens.device)
        dist.all_reduce(stats, group=self.ep_group)  # enqueued; read lazily by last_dropped_fraction
        self._last_aux_loss = ro.aux_loss
        self._last_dropped_fraction = stats
        self._last_token_counts = kept_counts
        return out

    def _forward_fused(self, tokens: torch.Tensor, ro: RouterOutput) -> torch.Tensor:
        """Dispatch / experts / combine through the peer-memory kernels, no host synchronisation.

        Every EP rank must route the same number of tokens per call (capacity is computed from
        T * ep_size on the host to size the buffers; the device value is clamped to it).
        """
        from ..parallel.ep_fused import fused_ep_moe

        _, fp8 = self._fused_payload()
        out, stats, kept_counts = fused_ep_moe(
            tokens, ro.topk_indices, ro.topk_weights, self.experts, self._stack_cache, group=self.ep_group,
            num_experts=self.num_experts, capacity_factor=self.capacity_factor, fp8_payload=fp8,
            stochastic=fp8 and self.comm_quant_rounding == "stochastic")
        if len(self.shared_experts):
            out = out + sum(se(tokens) for se in self.shared_experts) / float(len(self.shared_experts))
        dist.all_reduce(stats, group=self.ep_group)  # enqueued on the stream; read lazily
        self._last_aux_loss = ro.aux_loss
        self._last_dropped_fraction = stats
        self._last_token_counts = kept_counts
        self.last_path = "fused"
        return out
