"""Low-bit compute backends for linear layers.

* ``EmulatedLowBitBackend`` - the reference's software emulation
  (src/runtime/te_backend.py:40-260): symmetric fake quantisation on an
  integer grid (qmax = 2^(bits-1) - 1, i.e. 127 for "fp8", 7 for "fp4") at
  tensor / channel / 1x128-tile / 128x128-block granularity, nearest or
  stochastic rounding (floor(x + U)), straight-through gradients, fp32 GEMM.
  Kept as the CPU oracle and for bit-level parity runs.
* ``NativeFP8Backend`` - real e4m3 quantisation with fp32 scales per 1x128
  activation tile and per 128x128 weight block (the DeepSeek-V3 recipe) and
  stochastic or nearest rounding, run through the sm_100a quantiser kernels;
  the product of the dequantised operands is computed on the tcgen05 GEMM.
* ``NativeFP4Backend`` - NVFP4: e2m1 values in 1x16 blocks with an e4m3
  scale per block and an fp32 per-tensor scale; the forward GEMM runs on the
  e2m1 block-scaled tensor cores (``ops/fp4.py``, ``csrc/gemm_fp4.cu``).
* ``TransformerEngineBackend`` - wraps ``transformer_engine`` when it is
  installed (it is not on this image; selecting it raises at resolution time,
  like the reference).
"""
from __future__ import annotations

import weakref
from contextlib import nullcontext
from typing import Optional, Protocol

import torch
import torch.nn.functional as F

from .. import ops


class LowBitBackend(Protocol):
    name: str
    mode: str

    def linear(self, input_tensor: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
               module=None) -> torch.Tensor:
        ...


# ------------------------------------------------------------------ emulated (integer grid)
def stochastic_round(values: torch.Tensor, generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """floor(x + U) for x >= 0, ceil(x - U) for x < 0 with U ~ Uniform[0, 1)."""
    noise = torch.rand(values.shape, generator=generator, device=values.device, dtype=values.dtype)
    return torch.where(values >= 0, torch.floor(values + noise), torch.ceil(values - noise))


def round_values(values: torch.Tensor, rounding_mode: str) -> torch.Tensor:
    return stochastic_round(values) if rounding_mode == "stochastic" else torch.round(values)


def safe_scale(scale: torch.Tensor) -> torch.Tensor:
    return torch.where(torch.isfinite(scale) & (scale > 0), scale, torch.ones_like(scale))


def _grid_qdq(x: torch.Tensor, scale: torch.Tensor, qmax: int, rounding: str) -> torch.Tensor:
    return torch.clamp(round_values(x / scale, rounding), -qmax, qmax) * scale


def tile_quant_dequant(x_f: torch.Tensor, *, bits: int, tile_size: int, rounding_mode: str) -> torch.Tensor:
    shape = x_f.shape
    x2 = x_f.reshape(-1, shape[-1])
    rows, width = x2.shape
    nt = -(-width // tile_size)
    pad = nt * tile_size - width
    if pad:
        x2 = F.pad(x2, (0, pad))
    t = x2.reshape(rows, nt, tile_size)
    qmax = (1 << (bits - 1)) - 1
    s = safe_scale(t.detach().abs().amax(-1, keepdim=True) / qmax)
    dq = _grid_qdq(t, s, qmax, rounding_mode).reshape(rows, nt * tile_size)
    return dq[:, :width].reshape(shape)


def block_quant_dequant(x_f: torch.Tensor, *, bits: int, block_h: int, block_w: int,
                        rounding_mode: str) -> torch.Tensor:
    if x_f.dim() != 2:
        return tile_quant_dequant(x_f, bits=bits, tile_size=block_w, rounding_mode=rounding_mode)
    rows, cols = x_f.shape
    rb, cb = -(-rows // block_h), -(-cols // block_w)
    pr, pc = rb * block_h - rows, cb * block_w - cols
    if pr or pc:
        x_f = F.pad(x_f, (0, pc, 0, pr))
    blocks = x_f.reshape(rb, block_h, cb, block_w).permute(0, 2, 1, 3)
    qmax = (1 << (bits - 1)) - 1
    s = safe_scale(blocks.detach().abs().amax(dim=(-1, -2), keepdim=True) / qmax)
    dq = _grid_qdq(blocks, s, qmax, rounding_mode).permute(0, 2, 1, 3).reshape(rb * block_h, cb * block_w)
    return dq[:rows, :cols]


def quantize_dequantize(x: torch.Tensor, *, bits: int, granularity: str, rounding_mode: str,
                        channel_axis: int) -> torch.Tensor:
    """Integer-grid fake quantisation (the reference's "fp8"/"fp4" emulation)."""
    if x.numel() == 0:
        return x
    xf = x.float()
    qmax = (1 << (bits - 1)) - 1
    if granularity == "tensor":
        s = safe_scale(xf.detach().abs().amax() / qmax)
        return _grid_qdq(xf, s, qmax, rounding_mode).to(x.dtype)
    if granularity == "channel":
        axis = channel_axis % xf.dim()
        dims = [d for d in range(xf.dim()) if d != axis]
        s = safe_scale(xf.detach().abs().amax(dim=dims, keepdim=True) / qmax)
        return _grid_qdq(xf, s, qmax, rounding_mode).to(x.dtype)
    if granularity == "tile_1x128":
        return tile_quant_dequant(xf, bits=bits, tile_size=128, rounding_mode=rounding_mode).to(x.dtype)
    if granularity == "block_128x128":
        return block_quant_dequant(xf, bits=bits, block_h=128, block_w=128, rounding_mode=rounding_mode).to(x.dtype)
    s = safe_scale(xf.detach().abs().amax() / qmax)
    return (torch.clamp(torch.round(xf / s), -qmax, qmax) * s).to(x.dtype)


class EmulatedLowBitBackend:
    name = "emulated"

    def __init__(self, *, mode: str, kernel_spec=None) -> None:
        if mode not in ("fp8", "fp4"):
            raise ValueError("EmulatedLowBitBackend supports only fp8/fp4")
        self.mode = mode
        self._activation_granularity = "tensor"
        self._weight_granularity = "tensor"
        self._rounding_mode = "nearest"
        if kernel_spec is not None:
            self._activation_granularity = str(kernel_spec.activation_quant_granularity)
            self._weight_granularity = str(kernel_spec.weight_quant_granularity)
            self._rounding_mode = str(kernel_spec.rounding_mode)

    def linear(self, input_tensor, weight, bias, module=None):
        bits = 8 if self.mode == "fp8" else 4
        xdq = quantize_dequantize(input_tensor, bits=bits, granularity=self._activation_granularity,
                                  rounding_mode=self._rounding_mode, channel_axis=-1)
        wdq = quantize_dequantize(weight, bits=bits, granularity=self._weight_granularity,
                                  rounding_mode=self._rounding_mode, channel_axis=0)
        xq = input_tensor + (xdq - input_tensor).detach()
        wq = weight + (wdq - weight).detach()
        out = F.linear(xq.float(), wq.float(), None if bias is None else bias.float())
        return out.to(input_tensor.dtype)


# ------------------------------------------------------------------ native fp8 (e4m3)
E4M3_MAX = 448.0


def fp8_quant_dequant(x: torch.Tensor, *, granularity: str, rounding_mode: str, channel_axis: int = -1,
                      generator=None) -> torch.Tensor:
    """Real e4m3 round trip with fp32 scales at the given granularity.

    Uses the sm_100a quantiser kernel for 1x128 tiles / 128x128 blocks on
    CUDA; the PyTorch math below is the CPU oracle of the same numerics.
    """
    if x.numel() == 0:
        return x
    if x.is_cuda and granularity in ("tile_1x128", "block_128x128") and x.shape[-1] % 128 == 0 \
            and ops.available() and hasattr(ops.ext(), "fp8_quant_dequant"):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        seed = int(torch.randint(0, 2 ** 62, (1,), generator=generator).item()) if rounding_mode == "stochastic" else 0
        out = ops.ext().fp8_quant_dequant(x2, 1 if granularity == "tile_1x128" else 128, rounding_mode == "stochastic",
                                          seed)
        return out.view_as(x)
    xf = x.float()
    if granularity == "tensor":
        s = safe_scale(xf.detach().abs().amax() / E4M3_MAX)
        return _e4m3_qdq(xf, s, rounding_mode, generator).to(x.dtype)
    if granularity == "channel":
        axis = channel_axis % xf.dim()
        dims = [d for d in range(xf.dim()) if d != axis]
        s = safe_scale(xf.detach().abs().amax(dim=dims, keepdim=True) / E4M3_MAX)
        return _e4m3_qdq(xf, s, rounding_mode, generator).to(x.dtype)
    if granularity == "tile_1x128" or (granularity == "block_128x128" and xf.dim() != 2):
        shape = xf.shape
        x2 = xf.reshape(-1, shape[-1])
        rows, width = x2.shape
        nt = -(-width // 128)
        pad = nt * 128 - width
        if pad:
            x2 = F.pad(x2, (0, pad))
        t = x2.reshape(rows, nt, 128)
        s = safe_scale(t.detach().abs().amax(-1, keepdim=True) / E4M3_MAX)
        dq = _e4m3_qdq(t, s, rounding_mode, generator).reshape(rows, nt * 128)[:, :width]
        return dq.reshape(shape).to(x.dtype)
    rows, cols = xf.shape
    rb, cb = -(-rows // 128), -(-cols // 128)
    pr, pc = rb * 128 - rows, cb * 128 - cols
    xp = F.pad(xf, (0, pc, 0, pr)) if (pr or pc) else xf
    blocks = xp.reshape(rb, 128, cb, 128).permute(0, 2, 1, 3)
    s = safe_scale(blocks.detach().abs().amax(dim=(-1, -2), keepdim=True) / E4M3_MAX)
    dq = _e4m3_qdq(blocks, s, rounding_mode, generator).permute(0, 2, 1, 3).reshape(rb * 128, cb * 128)
    return dq[:rows, :cols].to(x.dtype)


def _e4m3_qdq(x: torch.Tensor, scale: torch.Tensor, rounding_mode: str, generator=None) -> torch.Tensor:
    y = (x / scale).clamp(-E4M3_MAX, E4M3_MAX)
    if rounding_mode == "stochastic":
        y = e4m3_stochastic_round(y, generator)
    q = y.to(torch.float8_e4m3fn).float()
    return q * scale


def e4m3_stochastic_round(y: torch.Tensor, generator=None) -> torch.Tensor:
    """Stochastic rounding onto the e4m3 grid: pick one of the two neighbouring
    representable values with probability proportional to proximity."""
    # e4m3 spacing: 2^(e-3) for normal numbers, 2^-9 for subnormals
    a = y.abs().clamp_min(2.0 ** -9)
    e = torch.floor(torch.log2(a)).clamp_min(-6)
    ulp = torch.pow(2.0, e - 3)
    down = torch.floor(y / ulp) * ulp
    frac = (y - down) / ulp
    u = torch.rand(y.shape, generator=generator, device=y.device)
    r = torch.where(u < frac, down + ulp, down)
    return r.clamp(-E4M3_MAX, E4M3_MAX)


_WQ_CACHE: dict = {}


def _remember(cache: dict, w: torch.Tensor, entry) -> None:
    """Store ``entry`` for weight ``w`` (keyed by ``id(w)``); the entry goes away with the weight,
    so quantised copies of dead weights are not kept alive and a reused id never hits a stale one."""
    key = id(w)
    if key not in cache:
        weakref.finalize(w, cache.pop, key, None)
    cache[key] = entry


def _quantized_weight(w: torch.Tensor):
    """e4m3 copy of a weight in 128 x 128 blocks, re-quantised only when the weight changed."""
    key = id(w)
    ent = _WQ_CACHE.get(key)
    if ent is not None and ent[0] == (w.data_ptr(), w._version):
        return ent[1], ent[2]
    wq, sw = ops.ext().fp8_quantize(w.detach().contiguous(), 128, False, 0)
    _remember(_WQ_CACHE, w, ((w.data_ptr(), w._version), wq, sw))
    return wq, sw


_WQT_CACHE: dict = {}


def _quantized_weight_t(w: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor):
    """Codes and block scales of W^T (the B operand of the input-gradient GEMM), from W's e4m3 copy:
    a 128 x 128 block of W^T is a transposed block of W, so its scale is the same number."""
    key = id(w)
    ent = _WQT_CACHE.get(key)
    if ent is not None and ent[0] == (w.data_ptr(), w._version):
        return ent[1], ent[2]
    wtq, swt = wq.t().contiguous(), sw.t().contiguous()
    _remember(_WQT_CACHE, w, ((w.data_ptr(), w._version), wtq, swt))
    return wtq, swt


class _FP8LinearFn(torch.autograd.Function):
    """Forward on the block-scaled e4m3 tensor cores. Backward: the input gradient also on the e4m3
    tensor cores when the output width is a multiple of 128 (dY quantised in 1 x 128 tiles, against
    the weight's transposed codes; ``NTB_FP8_DGRAD_NATIVE=0`` keeps bf16), the weight gradient as a
    bf16 GEMM on the dequantised activations accumulated in fp32 (straight-through); the fp8 copies
    are saved instead of bf16 activations."""

    @staticmethod
    def forward(ctx, x2, weight, bias, stochastic, seed):
        C = ops.ext()
        xq, sx = C.fp8_quantize(x2.contiguous(), 1, bool(stochastic), int(seed))
        wq, sw = _quantized_weight(weight)
        y = torch.empty(x2.shape[0], weight.shape[0], device=x2.device, dtype=torch.bfloat16)
        C.gemm_fp8_blockscaled(xq, sx, wq, sw, y, None if bias is None else bias.to(torch.bfloat16))
        ctx.save_for_backward(xq, sx, wq, sw)
        ctx.weight = weight
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops.linear import accumulate_weight_grad, gemm

        import os

        C = ops.ext()
        xq, sx, wq, sw = ctx.saved_tensors
        dy = dy.contiguous()
        N, K = wq.shape
        if N % 128 == 0 and K % 8 == 0 and os.environ.get("NTB_FP8_DGRAD_NATIVE", "1") != "0":
            wtq, swt = _quantized_weight_t(ctx.weight, wq, sw)
            dyq, sdy = C.fp8_quantize(dy, 1, False, 0)
            dx = torch.empty(dy.shape[0], K, device=dy.device, dtype=torch.bfloat16)
            C.gemm_fp8_blockscaled(dyq, sdy, wtq, swt, dx, None)
        else:
            dx = gemm(dy, C.fp8_dequantize(wq, sw, 128, torch.bfloat16), b_mn=True)
        xdq = C.fp8_dequantize(xq, sx, 1, torch.bfloat16)
        dw = accumulate_weight_grad(ctx.weight, dy, xdq)
        db = dy.float().sum(0).to(torch.bfloat16) if ctx.has_bias else None
        return dx, dw, db, None, None


class NativeFP8Backend:
    """e4m3 operands with fp32 tile/block scales; STE gradients in bf16/fp32.

    On CUDA with the recipe's tile_1x128 activations and block_128x128 weights the
    forward GEMM runs natively on the e4m3 tensor cores (``gemm_fp8_blockscaled``);
    other granularities and CPU tensors use quantise-dequantise + bf16/fp32 GEMM.
    """

    name = "native"

    def __init__(self, *, mode: str = "fp8", kernel_spec=None, fp8_format: str = "e4m3") -> None:
        if mode != "fp8":
            raise ValueError("NativeFP8Backend supports only fp8")
        self.mode = mode
        self.fp8_format = fp8_format
        self._activation_granularity = "tile_1x128"
        self._weight_granularity = "block_128x128"
        self._rounding_mode = "nearest"
        if kernel_spec is not None:
            self._activation_granularity = str(kernel_spec.activation_quant_granularity)
            self._weight_granularity = str(kernel_spec.weight_quant_granularity)
            self._rounding_mode = str(kernel_spec.rounding_mode)

    def _native_ok(self, x, weight) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and ops.available()
                and hasattr(ops.ext(), "gemm_fp8_blockscaled") and self._activation_granularity == "tile_1x128"
                and self._weight_granularity == "block_128x128" and x.shape[-1] % 128 == 0
                and weight.shape[0] % 8 == 0)

    def linear(self, input_tensor, weight, bias, module=None):
        if self._native_ok(input_tensor, weight):
            lead = input_tensor.shape[:-1]
            x2 = input_tensor.reshape(-1, input_tensor.shape[-1])
            self._seed = getattr(self, "_seed", 0) + 1
            y = _FP8LinearFn.apply(x2, weight, bias, self._rounding_mode == "stochastic", self._seed)
            # a 2-D input gets the Function's own output (not a view of it), so consumers that
            # modify it in place under autograd (the fused QKV attention) can
            return y if len(lead) == 1 else y.view(*lead, weight.shape[0])
        xdq = fp8_quant_dequant(input_tensor.detach(), granularity=self._activation_granularity,
                                rounding_mode=self._rounding_mode, channel_axis=-1)
        wdq = fp8_quant_dequant(weight.detach(), granularity=self._weight_granularity,
                                rounding_mode="nearest", channel_axis=0)
        xq = input_tensor + (xdq.to(input_tensor.dtype) - input_tensor).detach()
        wq = weight + (wdq.to(weight.dtype) - weight).detach()
        if input_tensor.is_cuda and input_tensor.dtype == torch.bfloat16:
            return ops.linear(xq, wq.to(torch.bfloat16), None if bias is None else bias.to(torch.bfloat16))
        out = F.linear(xq.float(), wq.float(), None if bias is None else bias.float())
        return out.to(input_tensor.dtype)


# ------------------------------------------------------------------ NVFP4 (e2m1 + e4m3 block scales)
E2M1_LEVELS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def nvfp4_quant_dequant(x: torch.Tensor, block: int = 16) -> torch.Tensor:
    """e2m1 values in 1 x block groups, e4m3 block scale, fp32 tensor scale (nearest rounding)."""
    if x.numel() == 0:
        return x
    shape = x.shape
    xf = x.float().reshape(-1, shape[-1])
    rows, width = xf.shape
    nb = -(-width // block)
    pad = nb * block - width
    if pad:
        xf = F.pad(xf, (0, pad))
    g = xf.reshape(rows, nb, block)
    tensor_amax = g.abs().amax()
    tscale = safe_scale(tensor_amax / (6.0 * 448.0))
    bamax = g.abs().amax(-1, keepdim=True)
    bscale = (bamax / 6.0 / tscale).clamp(max=448.0).to(torch.float8_e4m3fn).float() * tscale
    bscale = safe_scale(bscale)
    levels = torch.tensor(E2M1_LEVELS, device=x.device)
    mag = (g.abs() / bscale).clamp(max=6.0)
    idx = (mag[..., None] - levels).abs().argmin(-1)
    q = levels[idx] * torch.sign(g)
    dq = (q * bscale).reshape(rows, nb * block)[:, :width]
    return dq.reshape(shape).to(x.dtype)


_W4_CACHE: dict = {}


def _nvfp4_weight(w: torch.Tensor):
    """NVFP4 copy of a weight, re-quantised only when the weight changed."""
    from ..ops import fp4

    key = id(w)
    ent = _W4_CACHE.get(key)
    if ent is not None and ent[0] == (w.data_ptr(), w._version):
        return ent[1]
    packed = fp4.quantize(w.detach().to(torch.bfloat16))
    _remember(_W4_CACHE, w, ((w.data_ptr(), w._version), packed))
    return packed


class _FP4LinearFn(torch.autograd.Function):
    """Forward on the e2m1 block-scaled tensor cores (``gemm_nvfp4``); straight-through
    backward on the dequantised operands (bf16 GEMMs), saving the 4.5-bit copies instead of
    bf16 activations."""

    @staticmethod
    def forward(ctx, x2, weight, bias):
        from ..ops import fp4

        xq = fp4.quantize(x2.contiguous())
        wq = _nvfp4_weight(weight)
        y = fp4.gemm(xq, wq, bias=None if bias is None else bias.to(torch.bfloat16))
        ctx.save_for_backward(*xq, *wq)
        ctx.weight = weight
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops import fp4
        from ..ops.linear import accumulate_weight_grad, gemm

        xq, sx, gx, wq, sw, gw = ctx.saved_tensors
        dy = dy.contiguous()
        wdq = fp4.dequantize(wq, sw, gw, torch.bfloat16)
        dx = gemm(dy, wdq, b_mn=True)
        xdq = fp4.dequantize(xq, sx, gx, torch.bfloat16)
        dw = accumulate_weight_grad(ctx.weight, dy, xdq)
        db = dy.float().sum(0).to(torch.bfloat16) if ctx.has_bias else None
        return dx, dw, db


class NativeFP4Backend:
    """NVFP4: e2m1 values in 1x16 blocks, e4m3 block scales, fp32 per-tensor scale.

    On CUDA with bf16 activations and GEMM-compatible shapes (K % 256 == 0, N % 8 == 0)
    the forward GEMM runs on the e2m1 tensor cores (``tcgen05.mma kind::mxf4nvf4``, the
    block scales applied by the hardware); other shapes and CPU tensors use the same
    quantisation through quantise-dequantise + bf16/fp32 GEMM.
    """

    name = "native"

    def __init__(self, *, mode: str = "fp4", kernel_spec=None) -> None:
        if mode != "fp4":
            raise ValueError("NativeFP4Backend supports only fp4")
        self.mode = mode

    def linear(self, input_tensor, weight, bias, module=None):
        from ..ops import fp4

        K = input_tensor.shape[-1]
        if (input_tensor.is_cuda and input_tensor.dtype == torch.bfloat16 and weight.dim() == 2
                and fp4.gemm_supported(K, weight.shape[0])):
            lead = input_tensor.shape[:-1]
            x2 = input_tensor.reshape(-1, K)
            y = _FP4LinearFn.apply(x2, weight, bias)
            # a 2-D input gets the Function's own output (not a view of it), so consumers that
            # modify it in place under autograd (the fused QKV attention) can
            return y if len(lead) == 1 else y.view(*lead, weight.shape[0])
        if K % 64 == 0:
            xdq = fp4.quant_dequant_reference(input_tensor.detach())
            wdq = fp4.quant_dequant_reference(weight.detach())
        else:
            xdq = nvfp4_quant_dequant(input_tensor.detach())
            wdq = nvfp4_quant_dequant(weight.detach())
        xq = input_tensor + (xdq - input_tensor).detach()
        wq = weight + (wdq.to(weight.dtype) - weight).detach()
        if input_tensor.is_cuda and input_tensor.dtype == torch.bfloat16:
            return ops.linear(xq, wq.to(torch.bfloat16), None if bias is None else bias.to(torch.bfloat16))
        out = F.linear(xq.float(), wq.float(), None if bias is None else bias.float())
        return out.to(input_tensor.dtype)


# ------------------------------------------------------------------ Transformer Engine (optional)
class TransformerEngineBackend:
    """Routes fp8 linears through Transformer Engine's ``te.Linear`` (optional dependency, not
    installed on this image). One TE module per layer, built from the layer's kernel spec and
    bound to the layer's own trainable parameters (``bind_parameters``, called at layer init);
    tensors that are not the bound parameters (e.g. straight-through weights) take ``F.linear``.
    Reference parity: src/runtime/te_backend.py:263-385."""

    name = "transformer_engine"

    def __init__(self, *, mode: str, fp8_format: str, amax_history_len: int, amax_compute_algo: str,
                 kernel_spec=None) -> None:
        if mode != "fp8":
            raise ValueError("TransformerEngineBackend only supports fp8 mode")
        if kernel_spec is None:
            raise RuntimeError("Transformer Engine backend requires a per-module LowBitKernelSpec")
        try:
            import transformer_engine.pytorch as te  # type: ignore
        except Exception as exc:  # pragma: no cover - TE absent on this image
            raise RuntimeError("Transformer Engine backend requested but transformer_engine is unavailable") from exc
        self.mode = mode
        self._te = te
        self._fp8_format = fp8_format
        self._amax_history_len = int(amax_history_len)
        self._amax_compute_algo = str(amax_compute_algo)
        self._kernel_spec = kernel_spec
        self._te_linear = te.Linear(in_features=int(kernel_spec.in_features),
                                    out_features=int(kernel_spec.out_features), bias=bool(kernel_spec.has_bias))
        self._bound_weight = None
        self._bound_bias = None

    def bind_parameters(self, weight: torch.nn.Parameter, bias: Optional[torch.nn.Parameter]) -> None:
        spec = self._kernel_spec
        if not isinstance(weight, torch.nn.Parameter):
            raise TypeError("TransformerEngineBackend expects nn.Parameter weight binding")
        if tuple(weight.shape) != (int(spec.out_features), int(spec.in_features)):
            raise ValueError(f"TE backend weight shape mismatch: expected={(spec.out_features, spec.in_features)} "
                             f"got={tuple(weight.shape)}")
        if spec.has_bias:
            if not isinstance(bias, torch.nn.Parameter) or tuple(bias.shape) != (int(spec.out_features),):
                raise ValueError("TE backend expected a bias parameter of shape (out_features,)")
            self._te_linear.bias = bias
            self._bound_bias = bias
        else:
            self._bound_bias = None
        self._te_linear.weight = weight
        self._bound_weight = weight

    def _autocast(self):
        ac = getattr(self._te, "autocast", None) or getattr(self._te, "fp8_autocast", None)
        if ac is None:
            return nullcontext()
        try:  # the recipe object exists only in full TE installs
            from transformer_engine.common import recipe as te_recipe  # type: ignore

            fmt = te_recipe.Format.E4M3 if self._fp8_format == "e4m3" else te_recipe.Format.HYBRID
            rec = te_recipe.DelayedScaling(fp8_format=fmt, amax_history_len=self._amax_history_len,
                                           amax_compute_algo=self._amax_compute_algo)
        except Exception:
            return ac(enabled=True)
        return ac(enabled=True, fp8_recipe=rec)

    def linear(self, input_tensor, weight, bias, module=None):
        if self._bound_weight is None:
            raise RuntimeError("Transformer Engine backend used before parameter binding. "
                               "Layer init must bind module-owned trainable parameters.")
        te_linear = self._te_linear.to(device=input_tensor.device)
        with self._autocast():
            if weight is self._bound_weight and (bias is self._bound_bias or
                                                 (bias is None and self._bound_bias is None)):
                return te_linear(input_tensor)
            return F.linear(input_tensor, weight, bias)


def build_lowbit_backend_for_mode(config, *, mode: str, kernel_spec=None):
    """Backend for ``mode`` ('fp8' / 'fp4') under a resolved PrecisionConfig."""
    if mode == "fp8":
        name = str(getattr(config, "fp8_backend", "emulated"))
        if name == "emulated":
            return EmulatedLowBitBackend(mode="fp8", kernel_spec=kernel_spec)
        if name == "native":
            return NativeFP8Backend(mode="fp8", kernel_spec=kernel_spec, fp8_format=str(config.fp8_format))
        if name == "transformer_engine":
            return TransformerEngineBackend(mode="fp8", fp8_format=str(config.fp8_format),
                                            amax_history_len=int(config.fp8_amax_history_len),
                                            amax_compute_algo=str(config.fp8_amax_compute_algo),
                                            kernel_spec=kernel_spec)
        raise ValueError(f"unknown fp8 backend {name}")
    if mode == "fp4":
        name = str(getattr(config, "fp4_backend", "emulated"))
        if name == "emulated":
            return EmulatedLowBitBackend(mode="fp4", kernel_spec=kernel_spec)
        if name == "native":
            return NativeFP4Backend(mode="fp4", kernel_spec=kernel_spec)
        raise ValueError(f"unknown fp4 backend {name}")
    return None
