"""Inverted dropout whose mask is regenerated, not stored.

The mask of element i is a function of (seed, i) only: Philox-4x32-10 (Salmon et al.,
SC 2011) with counter (i // 4, 0, 0) and key = seed, word i % 4, kept when
``(word >> 8) * 2**-24 >= p``. The backward pass runs the same kernel with the saved
seed, so a dropout layer keeps 8 bytes per call instead of a mask tensor.
``philox_keep_reference`` restates the generator with numpy (the CPU path and the
GPU tests' oracle).

Reference parity: src/layers.py:989-1010.
"""
from __future__ import annotations

import numpy as np
import torch

from ._ext import ext

_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int):
    """Vectorised Philox-4x32-10 on uint64 arrays holding 32-bit values."""
    k0, k1 = np.uint64(k0), np.uint64(k1)
    for r in range(10):
        if r:
            k0 = (k0 + _W0) & _MASK32
            k1 = (k1 + _W1) & _MASK32
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return c0, c1, c2, c3


def philox_keep_reference(n: int, p: float, seed: int) -> torch.Tensor:
    g = np.arange((n + 3) // 4, dtype=np.uint64)
    z = np.zeros_like(g)
    words = np.stack(philox4x32_10(g & _MASK32, g >> np.uint64(32), z, z, seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF),
                     axis=1).reshape(-1)[:n]
    u = (words >> np.uint64(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    return torch.from_numpy(u >= np.float32(p))


def _apply_reference(x: torch.Tensor, p: float, seed: int) -> torch.Tensor:
    keep = philox_keep_reference(x.numel(), p, seed).to(x.device).view(x.shape)
    return torch.where(keep, x * (1.0 / (1.0 - p)), torch.zeros_like(x))


def _apply(x: torch.Tensor, p: float, seed: int) -> torch.Tensor:
    if x.is_cuda and x.dtype in (torch.bfloat16, torch.float32):
        return ext().dropout_apply(x.contiguous(), float(p), int(seed))
    return _apply_reference(x, p, seed)


class _DropoutFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, p, seed):
        ctx.p, ctx.seed = p, seed
        return _apply(x, p, seed)

    @staticmethod
    def backward(ctx, g):
        return _apply(g, ctx.p, ctx.seed), None, None


def dropout(x: torch.Tensor, p: float, seed: int | None = None) -> torch.Tensor:
    """Training-mode inverted dropout (0 <= p < 1); ``seed`` defaults to a draw from torch's
    CPU generator, so runs are reproducible under ``torch.manual_seed``."""
    if p == 0.0:
        return x
    if seed is None:
        seed = int(torch.randint(0, 2 ** 62, (1,)).item())
    return _DropoutFn.apply(x, p, seed)
