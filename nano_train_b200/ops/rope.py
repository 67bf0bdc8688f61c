"""Rotary position embedding kernels.

Two layouts:
  * ``half``: Llama/NeoX rotate-half on (i, i + R/2) pairs.
  * ``deepseek``: the reference's layout (src/models/deepseek.py:517-543):
    rotate_half pairs interleaved elements (2i, 2i+1) while the cos/sin cache
    is cat(freqs, freqs), so element j uses freq[j mod R/2]. Kept bit-for-bit
    so losses match the reference.
"""
from __future__ import annotations

import torch

from ._ext import ext

MODES = {"half": 0, "deepseek": 1}


def _inv_freq(R: int, theta: float, device) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, R, 2, device=device, dtype=torch.float32) / R))


_TABLES: dict = {}


def rope_table(seq_len: int, R: int, theta: float, device) -> torch.Tensor:
    """(cos, sin) of pos * theta^(-2k/R) for pos < seq_len, k < R/2, as fp32 [seq_len, R/2, 2]: the
    same fp32 angles as ``rope_reference``. Built once per (seq_len, R, theta, device) and kept."""
    key = (int(seq_len), int(R), float(theta), str(device))
    t = _TABLES.get(key)
    if t is None:
        ang = torch.arange(seq_len, device=device, dtype=torch.float32)[:, None] * _inv_freq(R, theta, device)[None]
        t = torch.stack([ang.cos(), ang.sin()], dim=-1).contiguous()
        _TABLES[key] = t
    return t


def rope_rows_(x: torch.Tensor, off: int, R: int, seq_len: int, theta: float, mode: str, inverse: bool) -> None:
    """In-place RoPE of columns [off, off + R) of every head of x [T, heads, D] (positions t % seq_len).
    One vectorised launch from the cached table when the layout allows 16-byte access, else the
    per-element kernel."""
    C = ext()
    ok = (R % 16 == 0 and off % 8 == 0 and x.dim() == 3 and x.stride(-1) == 1 and x.stride(0) % 8 == 0
          and x.stride(1) % 8 == 0 and x.data_ptr() % 16 == 0)
    if ok:
        C.rope_table_(x, rope_table(seq_len, R, theta, x.device), off, R, seq_len, MODES[mode], inverse)
    else:
        C.rope_(x, None, off, R, seq_len, float(theta), MODES[mode], inverse)


def rope_reference(x: torch.Tensor, positions: torch.Tensor, theta: float, mode: str, inverse=False) -> torch.Tensor:
    """PyTorch math of both layouts on x[..., S, heads, R] (positions [S] or broadcastable)."""
    R = x.shape[-1]
    inv = _inv_freq(R, theta, x.device)
    freqs = positions.to(torch.float32)[..., None] * inv  # [S, R/2]
    emb = torch.cat([freqs, freqs], dim=-1)  # [S, R]
    cos = emb.cos()[..., None, :]
    sin = emb.sin()[..., None, :]
    xf = x.float()
    if mode == "half":
        x1, x2 = xf[..., : R // 2], xf[..., R // 2:]
        rot = torch.cat([-x2, x1], dim=-1)
        if inverse:
            # transpose of [[c, -s], [s, c]] on each pair
            y1 = x1 * cos[..., : R // 2] + x2 * sin[..., R // 2:]
            y2 = x2 * cos[..., R // 2:] - x1 * sin[..., : R // 2]
            return torch.cat([y1, y2], -1).to(x.dtype)
        return (xf * cos + rot * sin).to(x.dtype)
    xe, xo = xf[..., 0::2], xf[..., 1::2]
    ce, co = cos[..., 0::2], cos[..., 1::2]
    se, so = sin[..., 0::2], sin[..., 1::2]
    if not inverse:
        ye = xe * ce - xo * se
        yo = xo * co + xe * so
    else:
        ye = xe * ce + xo * so
        yo = xo * co - xe * se
    return torch.stack([ye, yo], dim=-1).flatten(-2).to(x.dtype)


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, positions, seq_len, theta, mode):
        y = x.contiguous().clone()
        ext().rope_(y, positions, 0, y.shape[-1], seq_len, theta, MODES[mode], False)
        ctx.meta = (positions, seq_len, theta, mode)
        return y

    @staticmethod
    def backward(ctx, dy):
        positions, seq_len, theta, mode = ctx.meta
        dx = dy.contiguous().clone()
        ext().rope_(dx, positions, 0, dx.shape[-1], seq_len, theta, MODES[mode], True)
        return dx, None, None, None, None


def apply_rope(x: torch.Tensor, theta: float, mode: str = "half", positions: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE over x[B, S, heads, R] (positions default to arange(S) per sequence)."""
    S = x.shape[-3]
    if x.is_cuda and x.dtype in (torch.bfloat16, torch.float32):
        pos = positions.reshape(-1).to(torch.int64).contiguous() if positions is not None else None
        if pos is not None and pos.numel() != x.numel() // (x.shape[-1] * x.shape[-2]):
            pos = pos.expand(*x.shape[:-2]).reshape(-1).contiguous()
        return _RopeFn.apply(x, pos, S, float(theta), mode)
    if positions is None:
        positions = torch.arange(S, device=x.device)
    return rope_reference(x, positions, theta, mode)
