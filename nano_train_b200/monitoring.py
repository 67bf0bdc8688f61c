"""Torch-free monitoring math used by the Trainer (reference: src/monitoring.py:14-174).

Function names and formulas match the reference so dashboards and alerts
built on them carry over:

* ``resolve_sentinel_blocks(num_layers, requested)``: default (0, L//2, L-1),
  de-duplicated, out-of-range dropped, never empty.
* ``clip_coef(g, max_norm) = min(1, max_norm / (g + eps))`` (1 when clipping is off).
* ``global_update_ratio = lr * clip_coef * g_pre / (|w| + eps)``,
  ``update_ratio = lr * |g| / (|w| + eps)``.
* ``achieved_tflops = tokens/s * multiplier * N / 1e12``, ``mfu = achieved / peak``.
* ``eval_artifact_hash``: SHA-256 over the probe batch's dtypes, shapes,
  vocabulary, sequence length, seed and raw bytes.
"""
from __future__ import annotations

from hashlib import sha256
from typing import Iterable, Optional


def resolve_sentinel_blocks(num_layers: int, requested: Optional[Iterable[int]] = None) -> tuple[int, ...]:
    n = int(num_layers)
    if n <= 0:
        return ()
    cand = (0, n // 2, n - 1) if requested is None else requested
    out: list[int] = []
    for i in cand:
        i = int(i)
        if 0 <= i < n and i not in out:
            out.append(i)
    return tuple(out) or (0,)


def block_main_weight_names(block_idx: int) -> list[str]:
    """The four main matrices of a TransformerModel block (this framework's parameter names)."""
    b = int(block_idx)
    return [f"blocks.{b}.attention.qkv_proj.weight", f"blocks.{b}.attention.out_proj.weight",
            f"blocks.{b}.mlp.fc1.weight", f"blocks.{b}.mlp.fc2.weight"]


def candidate_sentinel_param_names(*, sentinel_blocks: Iterable[int]) -> set[str]:
    names = {"token_embeddings.weight", "position_embeddings.weight", "ln_f.weight", "ln_f.bias", "lm_head.weight"}
    for b in sentinel_blocks:
        names.update(block_main_weight_names(b))
    return names


def clip_coef(grad_norm: float, max_norm: float, *, eps: float = 1e-6) -> float:
    m = float(max_norm)
    if m <= 0:
        return 1.0
    return min(1.0, m / (float(grad_norm) + eps))


def global_update_ratio(lr: float, *, grad_norm_pre_clip: float, clip_coef_value: float, param_norm: float,
                        eps: float = 1e-12) -> float:
    w = float(param_norm)
    if w <= 0:
        return 0.0
    return float(lr) * float(clip_coef_value) * float(grad_norm_pre_clip) / (w + eps)


def update_ratio(lr: float, *, grad_norm: float, weight_norm: float, eps: float = 1e-12) -> float:
    w = float(weight_norm)
    if w <= 0:
        return 0.0
    return float(lr) * float(grad_norm) / (w + eps)


def achieved_tflops(effective_tokens_per_second: float, num_params: int, *, flops_multiplier: float = 6.0) -> float:
    t, n, k = float(effective_tokens_per_second), int(num_params), float(flops_multiplier)
    if t <= 0 or n <= 0 or k <= 0:
        return 0.0
    return t * k * n / 1e12


def mfu(achieved_tflops_value: float, peak_tflops: float) -> float:
    p = float(peak_tflops)
    return float(achieved_tflops_value) / p if p > 0 else 0.0


def eval_artifact_hash(*, input_ids_bytes: bytes, labels_bytes: bytes, input_dtype: str, labels_dtype: str,
                       input_shape: tuple[int, ...], labels_shape: tuple[int, ...], vocab_size: int,
                       max_seq_length: int, seed: int) -> str:
    h = sha256()
    for item in (str(input_dtype), str(labels_dtype), str(tuple(input_shape)), str(tuple(labels_shape)),
                 str(int(vocab_size)), str(int(max_seq_length)), str(int(seed))):
        h.update(item.encode("utf-8"))
    h.update(bytes(input_ids_bytes))
    h.update(bytes(labels_bytes))
    return h.hexdigest()
