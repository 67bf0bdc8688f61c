"""Persistent low-bit weight copies (fp8 e4m3 with per-channel/per-tensor
scales, or NF4 codes packed two per byte) kept as module buffers and used
through a straight-through estimator in the forward pass.

On CUDA the refresh (scales + codes, once per optimizer step) and the
dequantisation of the straight-through forward run in the kernels of
``csrc/persistent.cu`` (same fp32 arithmetic, same bits); the PyTorch
statements below are the CPU path and the tests' oracle.

Reference parity: src/layers.py:60-184 (NF4 codebook, pack/unpack,
quantizers) and 216-436 (buffers, refresh, STE forward).
"""
from __future__ import annotations

import torch

# The 16 NF4 levels (quantiles of a standard normal, normalised to [-1, 1]).
NF4_LEVELS = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453, -0.28444138169288635,
    -0.18477343022823334, -0.09105003625154495, 0.0, 0.07958029955625534, 0.16093020141124725,
    0.24611230194568634, 0.33791524171829224, 0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)
FP8_E4M3_MAX = 448.0


def nf4_codebook(device) -> torch.Tensor:
    return torch.tensor(NF4_LEVELS, dtype=torch.float32, device=device)


def _safe_scale(amax: torch.Tensor, qmax: float) -> torch.Tensor:
    s = amax / qmax
    return torch.where(s > 0, s, torch.ones_like(s))


def _amax(w: torch.Tensor, granularity: str) -> torch.Tensor:
    wf = w.detach().float()
    if granularity == "per_tensor":
        return wf.abs().amax().reshape(1)
    return wf.abs().amax(dim=1)


def _native(w: torch.Tensor) -> bool:
    return w.is_cuda and w.dim() == 2 and w.dtype in (torch.bfloat16, torch.float32)


def quantize_fp8_persistent(w: torch.Tensor, granularity: str):
    if _native(w):
        from ..ops._ext import ext

        q, scale = ext().persistent_quantize(w.detach().contiguous(), False, granularity == "per_tensor")
        return q.view(torch.float8_e4m3fn), scale
    scale = _safe_scale(_amax(w, granularity), FP8_E4M3_MAX)
    s = scale if granularity == "per_tensor" else scale[:, None]
    q = (w.detach().float() / s).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
    return q, scale


def dequantize_fp8_persistent(q: torch.Tensor, scale: torch.Tensor, granularity: str, dtype) -> torch.Tensor:
    if q.is_cuda and q.dim() == 2 and dtype in (torch.bfloat16, torch.float32):
        from ..ops._ext import ext

        return ext().persistent_dequantize(q.view(torch.uint8), scale, q.shape[0], q.shape[1], False, dtype)
    s = scale if granularity == "per_tensor" else scale[:, None]
    return (q.float() * s).to(dtype)


def pack_nibbles(idx: torch.Tensor) -> torch.Tensor:
    """Two 4-bit codes per byte, low nibble first."""
    flat = idx.reshape(-1).to(torch.uint8)
    if flat.numel() % 2:
        flat = torch.cat([flat, flat.new_zeros(1)])
    return (flat[0::2] & 0xF) | ((flat[1::2] & 0xF) << 4)


def unpack_nibbles(packed: torch.Tensor, numel: int) -> torch.Tensor:
    lo = packed & 0xF
    hi = (packed >> 4) & 0xF
    return torch.stack([lo, hi], dim=1).reshape(-1)[:numel].to(torch.int64)


def quantize_nf4_persistent(w: torch.Tensor, granularity: str):
    if _native(w):
        from ..ops._ext import ext

        codes, scale = ext().persistent_quantize(w.detach().contiguous(), True, granularity == "per_tensor")
        return codes, scale
    scale = _safe_scale(_amax(w, granularity), 1.0)
    s = scale if granularity == "per_tensor" else scale[:, None]
    normed = (w.detach().float() / s).reshape(-1, 1)
    cb = nf4_codebook(w.device).reshape(1, -1)
    idx = (normed - cb).abs().argmin(dim=1)
    return pack_nibbles(idx), scale


def dequantize_nf4_persistent(codes: torch.Tensor, scale: torch.Tensor, shape, granularity: str, dtype):
    if codes.is_cuda and len(shape) == 2 and dtype in (torch.bfloat16, torch.float32):
        from ..ops._ext import ext

        return ext().persistent_dequantize(codes, scale, shape[0], shape[1], True, dtype)
    numel = 1
    for d in shape:
        numel *= d
    idx = unpack_nibbles(codes, numel)
    vals = nf4_codebook(codes.device)[idx].reshape(shape)
    s = scale if granularity == "per_tensor" else scale[:, None]
    return (vals * s).to(dtype)


def _empty_buffers(module) -> None:
    dev = module.weight.device
    module._persistent_fp8_weight = torch.empty(0, device=dev)
    module._persistent_fp4_codes = torch.empty(0, dtype=torch.uint8, device=dev)
    module._persistent_scale = torch.empty(0, device=dev)
    module._persistent_numel = torch.zeros((), dtype=torch.int64, device=dev)


def init_persistent_buffers(module) -> None:
    """Register the four buffers (empty when the mode is off, as in the reference, so state dicts
    always carry the same keys) and fill them for an active persistent mode."""
    dev = module.weight.device
    module.register_buffer("_persistent_fp8_weight", torch.empty(0, device=dev), persistent=True)
    module.register_buffer("_persistent_fp4_codes", torch.empty(0, dtype=torch.uint8, device=dev), persistent=True)
    module.register_buffer("_persistent_scale", torch.empty(0, device=dev), persistent=True)
    module.register_buffer("_persistent_numel", torch.zeros((), dtype=torch.int64, device=dev), persistent=True)
    if module._persistent_mode() != "off" and dev.type != "meta":
        refresh_persistent(module)


def refresh_persistent(module) -> None:
    mode = module._persistent_mode()
    if mode == "off" or module.weight.device.type == "meta":
        _empty_buffers(module)
        return
    gran = module._persistent_granularity()
    dev = module.weight.device
    with torch.no_grad():
        if mode == "fp8":
            q, s = quantize_fp8_persistent(module.weight, gran)
            module._persistent_fp8_weight = q
            module._persistent_fp4_codes = torch.empty(0, dtype=torch.uint8, device=dev)
        elif mode == "fp4":
            codes, s = quantize_nf4_persistent(module.weight, gran)
            module._persistent_fp4_codes = codes
            module._persistent_fp8_weight = torch.empty(0, device=dev)
        else:
            raise ValueError(f"unknown persistent low-bit mode {mode}")
        module._persistent_scale = s
        module._persistent_numel = torch.tensor(module.weight.numel(), dtype=torch.int64, device=s.device)


def persistent_weight_ste(module) -> torch.Tensor:
    """w + (dequant(persistent) - w).detach(): forward sees the low-bit copy, gradient flows to w."""
    w = module.weight
    mode = module._persistent_mode()
    gran = module._persistent_granularity()
    if mode == "fp8" and module._persistent_fp8_weight.numel() > 0:
        dq = dequantize_fp8_persistent(module._persistent_fp8_weight, module._persistent_scale, gran, w.dtype)
    elif mode == "fp4" and module._persistent_fp4_codes.numel() > 0:
        dq = dequantize_nf4_persistent(module._persistent_fp4_codes, module._persistent_scale, tuple(w.shape), gran,
                                       w.dtype)
    else:
        return w
    return w + (dq - w).detach()
