"""Dense decoder-only transformer (L2).

``TransformerModel(config, tp_config)`` keeps the reference's constructor,
module names and ``forward(input_ids, attention_mask=None) -> logits``
(src/models/transformer.py:25-289: GPT-2 block with LayerNorm, learned
positions, fused-QKV MHA, GELU MLP, tied LM head, column-parallel LM head
under TP). ``ModelConfig`` switches turn the same block into the Llama-3
shape used by the TP benchmark: RMSNorm, RoPE, grouped-query attention,
SwiGLU, untied head, and Megatron sequence parallelism.

Internally activations are token-major 2-D tensors [T, H] with tokens in
(batch, position) order, so sequence-parallel shards are plain row ranges,
q/k/v are strided views of the fused projection output, and no layout copies
sit between the GEMMs and the attention kernel. ``forward_loss`` runs the
training path: fused (vocab-parallel) cross-entropy without materialising the
full-precision logits.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from .. import ops
from ..config import ModelConfig, TPConfig
from ..layers import (ColumnParallelLinear, Dropout, Embedding, LayerNorm, Linear, RMSNorm, RowParallelLinear,
                      VocabParallelEmbedding)
from ..ops.attention import qkv_attention
from ..parallel import comm


def _norm(config: ModelConfig, path: str):
    if config.norm == "rmsnorm":
        return RMSNorm(config.hidden_size, eps=config.norm_eps, param_dtype=config.param_dtype,
                       param_device=config.param_device, module_path=path,
                       precision_resolver=config.precision_resolver)
    return LayerNorm(config.hidden_size, eps=config.norm_eps, param_dtype=config.param_dtype,
                     param_device=config.param_device, module_path=path,
                     precision_resolver=config.precision_resolver, bias=config.bias)


class MultiHeadAttention(nn.Module):
    """Fused-QKV self-attention (MHA or GQA), column/row tensor-parallel.

    Two entry points:

    * ``forward(x, attention_mask=None)`` — the reference's module API (src/models/attention.py:
      134-220): x [B, S, H]; an additive mask [B, 1, S, S] or none (no mask means no masking);
    * ``forward_tokens(x2d, batch, seq)`` — the training path: token-major [B*S(/tp), H], implicit
      causal mask, RoPE and flash attention on the fused projection output.

    Masks, attention-probability dropout in training and monitoring (``set_monitoring``: max logit,
    entropy, normalised entropy, fraction of logits above tau) need the probabilities, so they run
    the materialised path: scores in the input dtype, fp32 softmax, probabilities cast to V's dtype
    (the reference's numerics).
    """

    def __init__(self, config: ModelConfig, tp_config: Optional[TPConfig] = None, module_prefix: str = "attention"):
        super().__init__()
        tp_config = tp_config or TPConfig()
        H = config.hidden_size
        self.hidden_size = H
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads or self.num_heads
        if H % self.num_heads != 0:
            raise ValueError("hidden_size must be divisible by num_attention_heads")
        self.head_dim = H // self.num_heads
        tp = tp_config.size if tp_config.enabled else 1
        if self.num_heads % tp or self.num_kv_heads % tp:
            raise ValueError("attention heads must be divisible by tp_size")
        self.tp_enabled = tp_config.enabled
        self.tp_size = tp
        self.nq = self.num_heads // tp
        self.nkv = self.num_kv_heads // tp
        self.tp_num_heads = self.nq
        self.scale = self.head_dim ** -0.5
        self.rope = config.position == "rope"
        self.rope_theta = config.rope_theta
        D = self.head_dim
        qkv_out = (self.num_heads + 2 * self.num_kv_heads) * D
        common = dict(param_dtype=config.param_dtype, param_device=config.param_device,
                      precision_resolver=config.precision_resolver, init_std=config.init_std)
        if tp_config.enabled:
            self.qkv_proj = ColumnParallelLinear(H, qkv_out, tp_config.rank, tp, bias=config.bias,
                                                 tp_group=tp_config.group, module_path=f"{module_prefix}.qkv_proj",
                                                 sequence_parallel=config.sequence_parallel, **common)
            self.out_proj = RowParallelLinear(H, H, tp_config.rank, tp, bias=config.bias, tp_group=tp_config.group,
                                              module_path=f"{module_prefix}.out_proj",
                                              sequence_parallel=config.sequence_parallel, **common)
        else:
            self.qkv_proj = Linear(H, qkv_out, bias=config.bias, module_path=f"{module_prefix}.qkv_proj", **common)
            self.out_proj = Linear(H, H, bias=config.bias, module_path=f"{module_prefix}.out_proj", **common)
        self.dropout = Dropout(config.dropout)
        self._monitor_enabled = False
        self._monitor_tau = 100.0
        self._monitor_stats: Optional[dict] = None

    def set_monitoring(self, enabled: bool, *, tau: float = 100.0) -> None:
        """Enable/disable the attention vitals (host reads; opt-in) and set tau."""
        self._monitor_enabled = bool(enabled)
        self._monitor_tau = float(tau)
        if not self._monitor_enabled:
            self._monitor_stats = None

    def _needs_probs(self, attention_mask) -> bool:
        return attention_mask is not None or self._monitor_enabled or (self.training and self.dropout.p > 0)

    def _materialized(self, qkv: torch.Tensor, batch: int, seq: int, attention_mask, causal: bool) -> torch.Tensor:
        from ..ops.rope import apply_rope

        nq, nkv, D = self.nq, self.nkv, self.head_dim
        q = qkv[:, : nq * D].view(batch, seq, nq, D)
        k = qkv[:, nq * D: (nq + nkv) * D].view(batch, seq, nkv, D)
        v = qkv[:, (nq + nkv) * D:].view(batch, seq, nkv, D)
        if self.rope:
            q, k = apply_rope(q, self.rope_theta, "half"), apply_rope(k, self.rope_theta, "half")
        q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))
        if nkv != nq:
            k = k.repeat_interleave(nq // nkv, dim=1)
            v = v.repeat_interleave(nq // nkv, dim=1)
        scores = torch.matmul(q, k.transpose(-2, -1)) * self.scale
        if attention_mask is not None:
            scores = scores + attention_mask
        elif causal:
            scores = scores.masked_fill(torch.ones(seq, seq, dtype=torch.bool, device=scores.device).triu(1),
                                        float("-inf"))
        sm = scores if scores.dtype in (torch.float32, torch.float64) else scores.float()
        probs = torch.softmax(sm, dim=-1).to(v.dtype)
        if self._monitor_enabled:
            with torch.no_grad():
                pf = probs.float().clamp_min(1e-12)
                ent = float((-(pf * pf.log()).sum(-1)).mean().item())
                self._monitor_stats = {
                    "max_attn_logit": float(scores.max().item()),
                    "attn_entropy": ent,
                    "attn_entropy_norm": float(ent / math.log(seq)) if seq > 1 else 0.0,
                    "frac_logits_gt_tau": float((scores > self._monitor_tau).float().mean().item()),
                }
        probs = self.dropout(probs)
        o = torch.matmul(probs, v).permute(0, 2, 1, 3)
        return o.reshape(batch * seq, nq * D)

    def forward_tokens(self, x: torch.Tensor, batch: int, seq: int) -> torch.Tensor:
        qkv = self.qkv_proj(x)  # [T, (nq + 2 nkv) D] (full T under sequence parallelism)
        D = self.head_dim
        if self._needs_probs(None):
            o = self._materialized(qkv, batch, seq, None, causal=True)
        else:
            o = qkv_attention(qkv, batch, seq, self.nq, self.nkv, D, D, rope_dim=D if self.rope else 0,
                              rope_theta=self.rope_theta, rope_mode="half")
        return self.out_proj(o)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dim() != 3:
            raise ValueError("x must have shape [batch_size, seq_len, hidden_size]")
        B, S, _ = x.shape
        qkv = self.qkv_proj(x.reshape(B * S, -1))
        D = self.head_dim
        if self._needs_probs(attention_mask):
            o = self._materialized(qkv, B, S, attention_mask, causal=False)
        else:
            o = qkv_attention(qkv, B, S, self.nq, self.nkv, D, D, rope_dim=D if self.rope else 0,
                              rope_theta=self.rope_theta, rope_mode="half", causal=False)
        return self.out_proj(o).view(B, S, -1)


class MLP(nn.Module):
    """GELU MLP (fc1 -> GELU -> fc2) or SwiGLU (fused gate|up -> silu*up -> down)."""

    def __init__(self, config: ModelConfig, tp_config: TPConfig, module_prefix: str):
        super().__init__()
        H, I = config.hidden_size, config.intermediate_size
        self.swiglu = config.mlp == "swiglu"
        tp = tp_config.size if tp_config.enabled else 1
        first_out = 2 * I if self.swiglu else I
        common = dict(param_dtype=config.param_dtype, param_device=config.param_device,
                      precision_resolver=config.precision_resolver, init_std=config.init_std)
        if tp_config.enabled:
            self.fc1 = ColumnParallelLinear(H, first_out, tp_config.rank, tp, bias=config.bias,
                                            tp_group=tp_config.group, module_path=f"{module_prefix}.fc1",
                                            sequence_parallel=config.sequence_parallel, **common)
            self.fc2 = RowParallelLinear(I, H, tp_config.rank, tp, bias=config.bias, tp_group=tp_config.group,
                                         module_path=f"{module_prefix}.fc2",
                                         sequence_parallel=config.sequence_parallel, **common)
        else:
            self.fc1 = Linear(H, first_out, bias=config.bias, module_path=f"{module_prefix}.fc1", **common)
            self.fc2 = Linear(I, H, bias=config.bias, module_path=f"{module_prefix}.fc2", **common)
        self.dropout = Dropout(config.dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.fc1(x)
        h = ops.swiglu(h) if self.swiglu else ops.gelu(h)
        h = self.dropout(h)
        return self.dropout(self.fc2(h))


class TransformerBlock(nn.Module):
    """Pre-norm block: x + attention(attn_norm(x)), then x + mlp(mlp_norm(x)) (the reference's
    submodule names, so state dicts carry over). RMSNorm models fuse the residual add into the
    second norm."""

    def __init__(self, config: ModelConfig, layer_idx: int = 0, tp_config: Optional[TPConfig] = None, *,
                 module_prefix: str = "blocks.0"):
        super().__init__()
        tp_config = tp_config or TPConfig()
        self.layer_idx = layer_idx
        self.attention = MultiHeadAttention(config, tp_config, f"{module_prefix}.attention")
        self.attn_norm = _norm(config, f"{module_prefix}.attn_norm")
        self.mlp = MLP(config, tp_config, f"{module_prefix}.mlp")
        self.mlp_norm = _norm(config, f"{module_prefix}.mlp_norm")
        self._fused_residual = isinstance(self.mlp_norm, RMSNorm)

    def forward_tokens(self, x: torch.Tensor, batch: int, seq: int) -> torch.Tensor:
        a = self.attention.forward_tokens(self.attn_norm(x), batch, seq)
        if self._fused_residual:
            h, x = self.mlp_norm.forward_residual(a, x)
        else:
            x = x + a
            h = self.mlp_norm(x)
        return x + self.mlp(h)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dim() != 3:
            raise ValueError("x must have shape [batch_size, seq_len, hidden_size]")
        x = x + self.attention(self.attn_norm(x), attention_mask)
        return x + self.mlp(self.mlp_norm(x))


class TransformerModel(nn.Module):
    """Decoder-only LM. ``forward`` returns logits [B, S, V] (vocab-sharded under TP)."""

    def __init__(self, config: ModelConfig, tp_config: Optional[TPConfig] = None) -> None:
        super().__init__()
        tp_config = tp_config or TPConfig()
        self.config = config
        self.tp_enabled = tp_config.enabled
        self.tp_rank = tp_config.rank
        self.tp_size = tp_config.size if tp_config.enabled else 1
        self.tp_group = tp_config.group
        self.sequence_parallel = bool(config.sequence_parallel and self.tp_enabled)
        common = dict(param_dtype=config.param_dtype, param_device=config.param_device,
                      precision_resolver=config.precision_resolver)
        if self.tp_enabled and not config.tie_word_embeddings:
            self.token_embeddings = VocabParallelEmbedding(config.vocab_size, config.hidden_size, self.tp_rank,
                                                           self.tp_size, self.tp_group, module_path="token_embeddings",
                                                           sequence_parallel=self.sequence_parallel,
                                                           init_std=config.init_std, **common)
        else:
            self.token_embeddings = Embedding(config.vocab_size, config.hidden_size, module_path="token_embeddings",
                                              init_std=config.init_std, **common)
        if config.position == "learned":
            self.position_embeddings = Embedding(config.max_position_embeddings, config.hidden_size,
                                                 module_path="position_embeddings", init_std=config.init_std,
                                                 **common)
        else:
            self.position_embeddings = None
        self.dropout = Dropout(config.dropout)
        self.blocks = nn.ModuleList([TransformerBlock(config, layer_idx=i, tp_config=tp_config,
                                                      module_prefix=f"blocks.{i}") for i in range(config.num_layers)])
        self.ln_f = _norm(config, "ln_f")
        if self.tp_enabled:
            if config.vocab_size % self.tp_size != 0:
                raise ValueError(f"vocab_size ({config.vocab_size}) must be divisible by tp_size ({self.tp_size})")
            self.lm_head = ColumnParallelLinear(config.hidden_size, config.vocab_size, tp_rank=self.tp_rank,
                                                tp_size=self.tp_size, tp_group=self.tp_group, bias=False,
                                                module_path="lm_head", sequence_parallel=self.sequence_parallel,
                                                init_std=config.init_std, **common)
        else:
            self.lm_head = Linear(config.hidden_size, config.vocab_size, bias=False, module_path="lm_head",
                                  init_std=config.init_std, **common)
            if config.tie_word_embeddings:
                self.lm_head.weight = self.token_embeddings.weight
        self.vocab_start = self.tp_rank * (config.vocab_size // self.tp_size) if self.tp_enabled else 0

    # ------------------------------------------------------------------ internals
    def _embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        B, S = input_ids.shape
        ids = input_ids.reshape(-1)
        x = self.token_embeddings(ids)  # [T(_local), H]
        if self.position_embeddings is not None:
            pos = torch.arange(S, device=input_ids.device).repeat(B)
            if self.sequence_parallel:
                pos = pos.chunk(self.tp_size)[self.tp_rank]
            x = x + self.position_embeddings(pos)
        if self.tp_enabled and not self.sequence_parallel and isinstance(self.token_embeddings, Embedding):
            pass
        elif self.sequence_parallel and isinstance(self.token_embeddings, Embedding):
            x = comm.scatter_to_sequence_parallel_region(x, self.tp_rank, self.tp_size, self.tp_group, seq_dim=0)
        return self.dropout(x)

    def hidden_states(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Final normed hidden states [T_local, H] (token-major; a sequence shard under SP)."""
        if input_ids.dim() != 2:
            raise ValueError("input_ids must have shape [batch_size, seq_len]")
        B, S = input_ids.shape
        if self.sequence_parallel and (B * S) % self.tp_size != 0:
            raise ValueError("batch*seq must be divisible by tp_size under sequence parallelism")
        x = self._embed(input_ids)
        observers = self.__dict__.get("_block_observers")
        for i, block in enumerate(self.blocks):
            y = block.forward_tokens(x, B, S)
            if observers:
                for fn in list(observers.values()):
                    fn(i, x, y)
            x = y
        return self.ln_f(x)

    def register_block_observer(self, fn):
        """Call ``fn(block_index, block_input, block_output)`` after every block of the token-major
        forward (the residual stream around each block); returns a handle with ``remove()``. The
        blocks run through ``forward_tokens``, which module forward hooks do not see."""
        obs = self.__dict__.setdefault("_block_observers", {})
        key = object()
        obs[key] = fn

        class _Handle:
            def remove(self_inner):
                obs.pop(key, None)

        return _Handle()

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Logits [B, S, V(/tp)]. Without a mask the blocks run the fused causal path; an explicit
        additive mask [B, 1, S, S] (as the reference builds with ``_create_causal_mask``) runs the
        materialised attention with that mask."""
        if input_ids.dim() != 2:
            raise ValueError("input_ids must have shape [batch_size, seq_len]")
        B, S = input_ids.shape
        if attention_mask is None:
            h = self.hidden_states(input_ids)
            return self.lm_head(h).view(B, S, -1)  # [T, V(/tp)] -> [B, S, V(/tp)]
        if self.sequence_parallel:
            raise ValueError("explicit attention masks are not supported under sequence parallelism")
        x = self._embed(input_ids).view(B, S, -1)
        for block in self.blocks:
            x = block(x, attention_mask)
        return self.lm_head(self.ln_f(x))

    @staticmethod
    def _create_causal_mask(batch_size: int, seq_len: int, device) -> torch.Tensor:
        """Additive causal mask [B, 1, S, S] (0 on and below the diagonal, -inf above)."""
        m = torch.full((seq_len, seq_len), float("-inf"), device=device).triu(1)
        return m.view(1, 1, seq_len, seq_len).expand(batch_size, -1, -1, -1)

    def forward_loss(self, input_ids: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
        """Mean next-token cross-entropy; ``labels`` are already aligned to positions.

        Under TP the LM head stays vocab-sharded and the loss is the
        vocab-parallel cross-entropy (three [T] all-reduces), and the
        gradient is written over the logits buffer in place.
        """
        h = self.hidden_states(input_ids)
        logits = self.lm_head(h)
        group = self.tp_group if self.tp_enabled else None
        return ops.cross_entropy(logits, labels.reshape(-1), ignore_index=ignore_index, vocab_start=self.vocab_start,
                                 group=group, inplace_grad=True)

    # ------------------------------------------------------------------ full <-> TP-shard state
    def shard_full_state_dict(self, full: dict) -> dict:
        """Slice an unsharded (TP=1) state dict into this rank's TP shards.

        Column-parallel weights split their output rows: the fused QKV rows go
        to each rank as [q heads | k heads | v heads] of that rank, the fused
        SwiGLU gate|up rows as [gate rows | up rows]; row-parallel weights
        split their input columns; the vocab-parallel embedding and LM head
        split the vocabulary. Replicated tensors are copied.
        """
        if not self.tp_enabled:
            return dict(full)
        r, tp = self.tp_rank, self.tp_size
        out = {}
        for name, t in full.items():
            if name.endswith("attention.qkv_proj.weight") or name.endswith("attention.qkv_proj.bias"):
                attn = self.blocks[0].attention
                D = attn.head_dim
                nq, nkv = attn.num_heads * D, attn.num_kv_heads * D
                q, k, v = t[:nq], t[nq:nq + nkv], t[nq + nkv:]
                out[name] = torch.cat([q.chunk(tp)[r], k.chunk(tp)[r], v.chunk(tp)[r]], 0).contiguous()
            elif self.config.mlp == "swiglu" and (name.endswith("mlp.fc1.weight") or name.endswith("mlp.fc1.bias")):
                g, u = t.chunk(2, 0)
                out[name] = torch.cat([g.chunk(tp)[r], u.chunk(tp)[r]], 0).contiguous()
            elif name.endswith("mlp.fc1.weight") or name.endswith("mlp.fc1.bias"):
                out[name] = t.chunk(tp, 0)[r].contiguous()
            elif name.endswith(("attention.out_proj.weight", "mlp.fc2.weight")):
                out[name] = t.chunk(tp, 1)[r].contiguous()
            elif name in ("lm_head.weight",) or (name == "token_embeddings.weight"
                                                 and not isinstance(self.token_embeddings, Embedding)):
                out[name] = t.chunk(tp, 0)[r].contiguous()
            else:
                out[name] = t
        return out

    def load_full_state_dict(self, full: dict, strict: bool = True):
        """Load an unsharded state dict (e.g. from a TP=1 run) into this (possibly TP-sharded) model."""
        return self.load_state_dict(self.shard_full_state_dict(full), strict=strict)

    @property
    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    @property
    def num_parameters_global(self) -> int:
        return self.num_parameters * self.tp_size if self.tp_enabled else self.num_parameters


def llama3_8b_config(*, num_layers: int = 32, param_dtype=torch.bfloat16, param_device=None,
                     sequence_parallel: bool = True, vocab_size: int = 128256, **overrides) -> ModelConfig:
    """Llama-3-8B shape: H 4096, 32 q / 8 kv heads, SwiGLU 14336, vocab 128256, RMSNorm 1e-5, RoPE 5e5."""
    from ..config import _default_precision_resolver

    cfg = dict(param_dtype=param_dtype, param_device=param_device, precision_resolver=_default_precision_resolver(),
               hidden_size=4096, num_layers=num_layers, num_attention_heads=32, num_key_value_heads=8,
               intermediate_size=14336, max_position_embeddings=8192, vocab_size=vocab_size, dropout=0.0,
               norm="rmsnorm", norm_eps=1e-5, position="rope", rope_theta=500000.0, mlp="swiglu", bias=False,
               tie_word_embeddings=False, sequence_parallel=sequence_parallel, init_std=0.02)
    cfg.update(overrides)
    return ModelConfig(**cfg)


def gpt_1p3b_config(*, num_layers: int = 24, param_dtype=torch.bfloat16, param_device=None, precision_resolver=None,
                    **overrides) -> ModelConfig:
    """GPT-1.3B shape: H 2048, 24 layers, 16 heads, GELU FFN 8192, vocab 50304, LayerNorm, learned
    positions (2048), tied embeddings. ``precision_resolver`` selects the low-bit compute of the
    linears (e.g. the NVFP4 backend under ``--fp4 --fp4-backend native``)."""
    from ..config import _default_precision_resolver

    cfg = dict(param_dtype=param_dtype, param_device=param_device,
               precision_resolver=precision_resolver or _default_precision_resolver(), hidden_size=2048,
               num_layers=num_layers, num_attention_heads=16, intermediate_size=8192, max_position_embeddings=2048,
               vocab_size=50304, dropout=0.0, norm="layernorm", norm_eps=1e-5, position="learned", mlp="gelu",
               bias=True, tie_word_embeddings=True, sequence_parallel=False, init_std=0.02)
    cfg.update(overrides)
    return ModelConfig(**cfg)
