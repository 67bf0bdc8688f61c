"""Grouped (mixture-of-experts) SwiGLU expert MLP on the tcgen05 grouped GEMM.

Tokens routed to experts are laid out expert by expert, each expert's segment
padded with zero rows to a multiple of 128 (``pad_segments``), so one
persistent kernel runs every expert's GEMM (``gemm_grouped_bf16`` mode 1) and
the weight gradients are one more launch per matrix (mode 2, K = the
expert's rows). The per-expert ``nn.Linear`` parameters stay separate
parameters (checkpoint keys unchanged); their stacked copies are rebuilt only
when a parameter changed (once per optimizer step, not per micro-batch), and
their gradients are written into ``main_grad`` when the optimizer provides
one, otherwise returned as ordinary ``.grad``.

Reference parity: src/models/moe.py:146-193 (ExpertMLP) and the per-expert
loops of LocalRoutedMoE / ExpertParallelMoE (moe.py:456-509, 888-962).
"""
from __future__ import annotations

import torch

from ._ext import ext

SEG = 128


def pad_segments(counts: torch.Tensor, max_rows: int | None = None):
    """Padded row offsets (int32 [E + 1], multiples of 128) and an upper bound on the rows.

    ``max_rows`` (host int) avoids a device->host sync: T*K + E*127 rounded up works for any routing.
    """
    padded = (counts + (SEG - 1)) // SEG * SEG
    offsets = torch.zeros(counts.numel() + 1, dtype=torch.int32, device=counts.device)
    offsets[1:] = torch.cumsum(padded, 0).to(torch.int32)
    if max_rows is None:
        max_rows = int(offsets[-1])
    return offsets, (max_rows + SEG - 1) // SEG * SEG


def scatter_rows_to_segments(x_sorted: torch.Tensor, counts: torch.Tensor, offsets: torch.Tensor, rows: int):
    """x_sorted [n, H] grouped by expert (counts per expert) -> zero-padded [rows, H] and the destination index."""
    n = x_sorted.shape[0]
    starts = torch.cumsum(counts, 0) - counts
    expert_of = torch.repeat_interleave(torch.arange(counts.numel(), device=counts.device), counts, output_size=n)
    dest = offsets[:-1].long()[expert_of] + (torch.arange(n, device=counts.device) - starts[expert_of])
    out = x_sorted.new_zeros(rows, x_sorted.shape[1])
    out.index_copy_(0, dest, x_sorted)
    return out, dest


class Fp8Stacks:
    """e4m3 codes + 128x128 block scales of the stacked expert weights: w1 [E * 2I, H] (gate|up),
    w2 [E * H, I], and the per-expert transposes w1t [E * H, 2I], w2t [E * I, H]."""

    def __init__(self, w1q, s1, w2q, s2, w1tq, s1t, w2tq, s2t):
        self.w1q, self.s1, self.w2q, self.s2 = w1q, s1, w2q, s2
        self.w1tq, self.s1t, self.w2tq, self.s2t = w1tq, s1t, w2tq, s2t


class _StackCache:
    """Stacked expert weights, rebuilt only when a source parameter changed."""

    def __init__(self):
        self.key = None
        self.w1 = None
        self.w2 = None
        self._params = None
        self.codes_key = None
        self._codes = None

    def params(self, experts):
        """[gate_0, up_0, down_0, gate_1, ...] weights (list built once per module)."""
        if self._params is None or len(self._params) != 3 * len(experts):
            self._params = [p for e in experts for p in (e.gate_proj.weight, e.up_proj.weight, e.down_proj.weight)]
        return self._params

    @staticmethod
    def _expert_stride(params) -> int:
        """Element stride between consecutive experts when every expert's (gate, up, down) sit back to
        back in one storage at a constant stride (the flat optimizer's parameter layout), else 0."""
        g0, u0, d0 = params[0], params[1], params[2]
        if not (g0.is_cuda and g0.dtype == torch.bfloat16 and g0.is_contiguous()):
            return 0
        es = g0.element_size()
        st = g0.untyped_storage().data_ptr()
        stride = (params[3].data_ptr() - g0.data_ptr()) // es if len(params) > 3 else 0
        for e in range(len(params) // 3):
            g, u, d = params[3 * e: 3 * e + 3]
            if (g.untyped_storage().data_ptr() != st or not (g.is_contiguous() and u.is_contiguous()
                                                            and d.is_contiguous())
                    or g.data_ptr() != g0.data_ptr() + e * stride * es
                    or u.data_ptr() != g.data_ptr() + g.numel() * es
                    or d.data_ptr() != d0.data_ptr() + e * stride * es):
                return 0
        return stride if len(params) > 3 else g0.numel() + u0.numel() + d0.numel()

    def codes(self, experts) -> "Fp8Stacks | None":
        """e4m3 codes and 128 x 128 block scales of the expert stacks, and of their per-expert
        transposes (the B operands of the two input-gradient GEMMs), rebuilt when a weight changed;
        None when the experts do not sit at a constant stride in one buffer or a dimension is not a
        multiple of 128."""
        params = self.params(experts)
        key = ("codes",) + tuple((p.data_ptr(), p._version) for p in params)
        if key == self.codes_key:
            return self._codes
        stride = self._expert_stride(params)
        g, d = params[0], params[2]
        I, H = g.shape
        if not stride or I % 128 or H % 128:
            self.codes_key, self._codes = key, None
            return None
        E = len(experts)
        C = ext()
        with torch.no_grad():
            w1q, s1 = C.fp8_quantize_strided(g, E, 2 * I, H, stride)
            w2q, s2 = C.fp8_quantize_strided(d, E, H, I, stride)
            tr = lambda t, a, b: t.view(E, a, b).transpose(1, 2).contiguous().view(E * b, a)  # noqa: E731
            self._codes = Fp8Stacks(w1q, s1, w2q, s2, tr(w1q, 2 * I, H), tr(s1, 2 * I // 128, H // 128),
                                    tr(w2q, H, I), tr(s2, H // 128, I // 128))
        self.codes_key = key
        return self._codes

    def get(self, experts, fp8: bool = False):
        """(w1, w2); with ``fp8`` every expert matrix is rounded through e4m3 in 128 x 128 blocks
        first (the recipe's weight quantisation), so the bf16 GEMMs see the fp8 values. When the
        experts' weights lie at a constant stride in one buffer, the rounded stacks are written in
        one pass from the parameters in place (no concatenation first)."""
        params = self.params(experts)
        key = (bool(fp8),) + tuple((p.data_ptr(), p._version) for p in params)
        if key != self.key:
            with torch.no_grad():
                E = len(experts)
                stride = self._expert_stride(params) if fp8 else 0
                g, d = params[0], params[2]
                if stride and g.shape[0] % 128 == 0 and g.shape[1] % 128 == 0 and d.shape[1] % 128 == 0:
                    C = ext()
                    self.w1 = C.fp8_quant_dequant_strided(g, E, 2 * g.shape[0], g.shape[1], stride)
                    self.w2 = C.fp8_quant_dequant_strided(d, E, d.shape[0], d.shape[1], stride)
                else:
                    self.w1 = torch.cat([torch.cat([e.gate_proj.weight, e.up_proj.weight], 0) for e in experts], 0)
                    self.w2 = torch.cat([e.down_proj.weight for e in experts], 0)
                    if fp8:
                        # Every expert matrix has a multiple of 128 rows (the fp8 grouped path requires
                        # H % 128 == 0 and I % 128 == 0), so no 128 x 128 block spans two matrices and
                        # rounding the stack equals rounding each matrix on its own.
                        self.w1 = ext().fp8_quant_dequant(self.w1, 128, False, 0)
                        self.w2 = ext().fp8_quant_dequant(self.w2, 128, False, 0)
            self.key = key
        return self.w1, self.w2


_FLAT_CACHE: dict = {}


def _flat_main_grads(params, E: int, I: int, H: int):
    """Cached form of _flat_main_grads_uncached (keyed by the first and last gradient addresses)."""
    m0, m1 = getattr(params[0], "main_grad", None), getattr(params[-1], "main_grad", None)
    if m0 is None or m1 is None:
        return None
    key = (m0.data_ptr(), m1.data_ptr(), len(params), E, I, H)
    hit = _FLAT_CACHE.get(key, 0)
    if hit == 0:
        if len(_FLAT_CACHE) > 256:
            _FLAT_CACHE.clear()
        hit = _FLAT_CACHE[key] = _flat_main_grads_uncached(params, E, I, H)
    return hit


def _flat_main_grads_uncached(params, E: int, I: int, H: int):
    """Views for accumulating every expert's weight gradient in one launch per matrix.

    When the fp32 ``main_grad`` of the experts lie in one flat buffer as
    (gate [I, H], up [I, H], down [H, I]) per expert at a constant stride (the
    flat optimizer's layout for consecutive ExpertMLPs), returns
    (rows of pitch H starting at expert 0's gate gradient, rows of pitch I
    starting at expert 0's down gradient); otherwise None.
    """
    mgs = [getattr(p, "main_grad", None) for p in params]
    if len(mgs) != 3 * E or any(m is None or m.dtype != torch.float32 or not m.is_contiguous() for m in mgs):
        return None
    base, step, es = mgs[0].data_ptr(), 3 * I * H, 4
    st = mgs[0].untyped_storage().data_ptr()
    for e in range(E):
        g, u, d = mgs[3 * e:3 * e + 3]
        if (g.data_ptr() != base + e * step * es or u.data_ptr() != base + (e * step + I * H) * es
                or d.data_ptr() != base + (e * step + 2 * I * H) * es or g.untyped_storage().data_ptr() != st
                or u.untyped_storage().data_ptr() != st or d.untyped_storage().data_ptr() != st):
            return None
    out1 = mgs[0].as_strided(((E - 1) * 3 * I + 2 * I, H), (H, 1))
    out2 = mgs[2].as_strided(((E - 1) * 3 * H + H, I), (I, 1))
    return out1, out2


class GroupedBuffers:
    """Optional caller-owned outputs: ``y_out`` receives the expert outputs, ``dx_out``
    the input gradient (the expert-parallel path points both at peer-visible memory)."""

    def __init__(self, y_out: torch.Tensor | None = None, dx_out: torch.Tensor | None = None):
        self.y_out = y_out
        self.dx_out = dx_out


_FP8_SEED = [0]


class _GroupedSwiGLUFn(torch.autograd.Function):
    """``fp8``: None, or the rounding of the e4m3 activation quantisation ("nearest" /
    "stochastic").

    With ``codes`` (an ``Fp8Stacks``) the expert GEMMs run on e4m3 operands on the tensor cores:
    the forward quantises X and SwiGLU(H) in 1 x 128 tiles and multiplies them with the weight
    stacks' codes (128 x 128 block scales) in the grouped block-scaled GEMM; the backward quantises
    dY and dH the same way for the two input-gradient GEMMs (against the per-expert transposed
    weight codes). The weight gradients are bf16 grouped GEMMs on the rounded activations
    (straight-through), accumulated in fp32.

    Without ``codes`` both GEMM inputs are rounded through e4m3 (the weights arrive rounded in
    128 x 128 blocks) and every GEMM is bf16: the same numerics, emulated."""

    @staticmethod
    def forward(ctx, x_pad, offsets, w1, w2, n_experts, bufs, fp8, codes, *params):
        C = ext()
        R = x_pad.shape[0]
        if codes is not None:
            sr = fp8 == "stochastic"
            _FP8_SEED[0] += 1
            I2 = codes.w1q.shape[0] // n_experts
            H = codes.w2q.shape[0] // n_experts
            xq, sx, x_r = C.fp8_quantize_with_dq(x_pad.contiguous(), sr, _FP8_SEED[0])
            h = torch.empty(R, I2, device=x_pad.device, dtype=x_pad.dtype)
            C.gemm_fp8_grouped(xq, sx, codes.w1q, codes.s1, h, offsets)
            aq, sa, a_r = C.fp8_quantize_with_dq(C.swiglu_fwd(h), sr, _FP8_SEED[0] + (1 << 40))
            y = bufs.y_out if bufs is not None and bufs.y_out is not None else \
                torch.empty(R, H, device=x_pad.device, dtype=x_pad.dtype)
            C.gemm_fp8_grouped(aq, sa, codes.w2q, codes.s2, y, offsets)
            ctx.save_for_backward(x_r, offsets, h, a_r)
            ctx.codes = codes
            ctx.n_experts = n_experts
            ctx.params = params
            ctx.bufs = bufs
            return y
        ctx.codes = None
        I2 = w1.shape[0] // n_experts
        H = w2.shape[0] // n_experts
        if fp8 is not None:
            _FP8_SEED[0] += 1
            x_pad = C.fp8_quant_dequant(x_pad.contiguous(), 1, fp8 == "stochastic", _FP8_SEED[0])
        h = torch.empty(R, I2, device=x_pad.device, dtype=x_pad.dtype)
        C.gemm_grouped_bf16(x_pad, w1, h, offsets, 1)
        a = C.swiglu_fwd(h)
        if fp8 is not None:
            a = C.fp8_quant_dequant(a, 1, fp8 == "stochastic", _FP8_SEED[0] + (1 << 40))
        y = bufs.y_out if bufs is not None and bufs.y_out is not None else \
            torch.empty(R, H, device=x_pad.device, dtype=x_pad.dtype)
        C.gemm_grouped_bf16(a, w2, y, offsets, 1)
        ctx.save_for_backward(x_pad, offsets, w1, w2, h, a)
        ctx.n_experts = n_experts
        ctx.params = params
        ctx.bufs = bufs
        return y

    @staticmethod
    def backward(ctx, dy):
        C = ext()
        E = ctx.n_experts
        dy = dy.contiguous()
        codes = ctx.codes
        if codes is not None:
            x_pad, offsets, h, a = ctx.saved_tensors
            I2, H = h.shape[1], x_pad.shape[1]
            I = I2 // 2
            da = torch.empty_like(a)
            dyq, sdy = C.fp8_quantize(dy, 1, False, 0)
            C.gemm_fp8_grouped(dyq, sdy, codes.w2tq, codes.s2t, da, offsets)   # dA = dY . W2_e (e4m3)
        else:
            x_pad, offsets, w1, w2, h, a = ctx.saved_tensors
            I2 = w1.shape[0] // E
            H = w2.shape[0] // E
            I = I2 // 2
            da = torch.empty_like(a)
            C.gemm_grouped_bf16(dy, w2, da, offsets, 1, b_mn=True)          # dA = dY . W2_e
        flat = _flat_main_grads(ctx.params, E, I, H)
        dw2 = None
        if flat is not None:                                              # dW2_e += dY_e^T A_e into main_grad
            C.gemm_grouped_bf16(dy, a, flat[1], offsets, 2, b_mn=True, accumulate=True, c_group_stride=3 * H)
        else:
            dw2 = torch.zeros(E * H, I, device=dy.device, dtype=torch.float32)
            C.gemm_grouped_bf16(dy, a, dw2, offsets, 2, b_mn=True)      # dW2_e = dY_e^T A_e
        dh = C.swiglu_bwd(da, h)
        bufs = ctx.bufs
        dx = bufs.dx_out if bufs is not None and bufs.dx_out is not None else torch.empty_like(x_pad)
        if codes is not None:
            dhq, sdh = C.fp8_quantize(dh, 1, False, 0)
            C.gemm_fp8_grouped(dhq, sdh, codes.w1tq, codes.s1t, dx, offsets)  # dX = dH . W1_e (e4m3)
        else:
            C.gemm_grouped_bf16(dh, w1, dx, offsets, 1, b_mn=True)          # dX = dH . W1_e
        nones = (None,) * 8
        if flat is not None:                                              # dW1_e += dH_e^T X_e into main_grad
            C.gemm_grouped_bf16(dh, x_pad, flat[0], offsets, 2, b_mn=True, accumulate=True, c_group_stride=3 * I)
            return (dx, *nones[1:], *([None] * len(ctx.params)))
        dw1 = torch.zeros(E * I2, x_pad.shape[1], device=dy.device, dtype=torch.float32)
        C.gemm_grouped_bf16(dh, x_pad, dw1, offsets, 2, b_mn=True)      # dW1_e = dH_e^T X_e
        slices = []
        for e in range(E):
            slices += [dw1[e * I2:e * I2 + I], dw1[e * I2 + I:(e + 1) * I2], dw2[e * H:(e + 1) * H]]
        mgs = [getattr(p, "main_grad", None) for p in ctx.params]
        if all(m is not None for m in mgs):
            torch._foreach_add_(mgs, slices)
            grads = [None] * len(ctx.params)
        else:
            # one cast per stacked gradient; each parameter receives a view of it
            dt = ctx.params[0].dtype
            dw1c, dw2c = dw1.to(dt), dw2.to(dt)
            grads = []
            for e in range(E):
                grads += [dw1c[e * I2:e * I2 + I], dw1c[e * I2 + I:(e + 1) * I2], dw2c[e * H:(e + 1) * H]]
        return (dx, *nones[1:], *grads)


def grouped_swiglu_experts(x_sorted: torch.Tensor, counts: torch.Tensor, experts, cache: _StackCache,
                           max_rows: int | None = None) -> torch.Tensor:
    """Apply expert e to its rows of ``x_sorted`` (rows grouped by expert, ``counts`` per expert)."""
    offsets, rows = pad_segments(counts, max_rows)
    x_pad, dest = scatter_rows_to_segments(x_sorted, counts, offsets, rows)
    fp8 = grouped_fp8_rounding(experts)
    w1, w2, codes = expert_operands(experts, cache, fp8, x_pad.dtype)
    params = [p for e in experts for p in (e.gate_proj.weight, e.up_proj.weight, e.down_proj.weight)]
    y_pad = _GroupedSwiGLUFn.apply(x_pad, offsets, w1, w2, len(experts), None, fp8, codes, *params)
    return y_pad.index_select(0, dest)


def expert_operands(experts, cache: _StackCache, fp8, dtype):
    """(w1, w2, codes) for ``_GroupedSwiGLUFn``: under the fp8 recipe the e4m3 codes of the stacks
    (``NTB_FP8_GROUPED_NATIVE=0`` keeps the bf16 emulation), otherwise the bf16 stacks."""
    import os

    if fp8 is not None and os.environ.get("NTB_FP8_GROUPED_NATIVE", "1") != "0":
        codes = cache.codes(experts)
        if codes is not None:
            empty = torch.empty(0, device=codes.w1q.device, dtype=dtype)
            return empty, empty, codes
    w1, w2 = cache.get(experts, fp8=fp8 is not None)
    return w1.to(dtype), w2.to(dtype), None


def grouped_fp8_rounding(experts):
    """The activation rounding mode when the experts' linears run the native fp8 backend with the
    DeepSeek-V3 granularities (the grouped path then reproduces their numerics); else None."""
    from ..precision.backends import NativeFP8Backend

    e0 = experts[0]
    lins = (e0.gate_proj, e0.up_proj, e0.down_proj)
    if not any(lin._lowbit_active() for lin in lins):
        return None
    bes = [lin._lowbit_backend for lin in lins]
    if all(isinstance(b, NativeFP8Backend) and b._activation_granularity == "tile_1x128"
           and b._weight_granularity == "block_128x128" for b in bes):
        return bes[0]._rounding_mode
    return None


def grouped_kernel_ok(x: torch.Tensor, experts) -> bool:
    if not (x.is_cuda and x.dtype == torch.bfloat16 and len(experts) > 0):
        return False
    e0 = experts[0]
    H, I = e0.gate_proj.weight.shape[1], e0.gate_proj.weight.shape[0]
    if any(lin._lowbit_active() for lin in (e0.gate_proj, e0.up_proj, e0.down_proj)):
        # low-bit experts take the grouped path only where it reproduces their numerics
        return grouped_fp8_rounding(experts) is not None and H % 128 == 0 and I % 128 == 0
    return H % 8 == 0 and I % 8 == 0
