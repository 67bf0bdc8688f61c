"""NVFP4 tensors and the native e2m1 GEMM.

Format of one ``[R, K]`` matrix (K a multiple of 64), the layout the sm_100a
block-scaled tensor cores read directly:

* ``q``  uint8 ``[R, K/2]``: e2m1 codes, element k of a row in byte k/2, low
  nibble for even k (round to nearest even, saturating at 6);
* ``sf`` uint8 e4m3 scales, one per 1 x 16 group, in 512-byte blocks of 128 rows
  x 4 groups: block ``(r // 128, j // 4)`` at byte ``(r // 128 * K/64 + j // 4) * 512``
  and, inside it, row r / group j at ``(r % 32) * 16 + (r % 128) // 32 * 4 + j % 4``;
  rows past R in the last block hold 0;
* ``gs`` fp32 ``[1]``: per-tensor scale ``amax / (6 * 448)`` (1 for an all-zero
  tensor), so ``x ~= e2m1 * e4m3 * gs``.

``quantize_reference`` / ``dequantize_reference`` restate the kernels' numerics in
PyTorch with the same fp32 operation order (the CPU oracle of the GPU tests);
``quantize`` / ``dequantize`` / ``gemm`` run the kernels of ``csrc/gemm_fp4.cu``.

Reference parity: the reference only emulates fp4 GEMMs (integer-grid fake
quantisation and an fp32 GEMM, src/runtime/te_backend.py:229-260); this is the
GPT-1.3B fp4 configuration's NVFP4 recipe on real e2m1 tensor cores.
"""
from __future__ import annotations

import torch

from ._ext import ext

E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_MIDPOINTS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
E2M1_MAX = 6.0
E4M3_MAX = 448.0


def sf_bytes(rows: int, cols: int) -> int:
    return (rows + 127) // 128 * (cols // 64) * 512


def sf_index(rows: int, cols: int, device=None) -> torch.Tensor:
    """Byte offset of the scale of (row r, group j) for every r < rows, j < cols // 16."""
    r = torch.arange(rows, device=device).view(-1, 1)
    j = torch.arange(cols // 16, device=device).view(1, -1)
    return ((r // 128) * (cols // 64) + j // 4) * 512 + (r % 32) * 16 + (r % 128) // 32 * 4 + j % 4


def e2m1_encode(y: torch.Tensor) -> torch.Tensor:
    """fp32 -> e2m1 code (0..15), round to nearest even, saturating; -0 encodes as +0."""
    a = y.abs()
    code = torch.zeros_like(a, dtype=torch.int32)
    for i, m in enumerate(_MIDPOINTS):
        code += (a > m).to(torch.int32)
        if i % 2 == 1:  # a tie between code i and i + 1 goes to the even code i + 1
            code += (a == m).to(torch.int32)
    return torch.where((y < 0) & (code > 0), code + 8, code)


def e2m1_decode(code: torch.Tensor) -> torch.Tensor:
    table = torch.tensor(E2M1_VALUES + tuple(-v for v in E2M1_VALUES), dtype=torch.float32, device=code.device)
    return table[code.long()]


def tensor_scale(amax: torch.Tensor) -> torch.Tensor:
    g = amax.float() / (E2M1_MAX * E4M3_MAX)
    return torch.where(g > 0, g, torch.ones_like(g))


def quantize_reference(x: torch.Tensor):
    """PyTorch restatement of ``nvfp4_quantize``: returns ``(q, sf, gs)``."""
    R, K = x.shape
    if K % 64:
        raise ValueError("NVFP4 needs K % 64 == 0")
    xf = x.float()
    gs = tensor_scale(xf.abs().amax() if xf.numel() else torch.zeros((), device=x.device))
    g = xf.view(R, K // 16, 16)
    bmax = g.abs().amax(-1)
    s8 = torch.clamp(bmax / 6.0 / gs, max=E4M3_MAX).to(torch.float8_e4m3fn)
    eff = s8.float() * gs
    inv = torch.where(eff > 0, 1.0 / eff, torch.zeros_like(eff))
    codes = e2m1_encode(g * inv.unsqueeze(-1)).view(R, K)
    q = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    sf = torch.zeros(sf_bytes(R, K), dtype=torch.uint8, device=x.device)
    sf[sf_index(R, K, x.device).reshape(-1)] = s8.view(torch.uint8).reshape(-1)
    return q, sf, gs.reshape(1)


def dequantize_reference(q: torch.Tensor, sf: torch.Tensor, gs: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    R, K2 = q.shape
    K = 2 * K2
    codes = torch.stack([q & 0xF, q >> 4], dim=-1).reshape(R, K)
    vals = e2m1_decode(codes).view(R, K // 16, 16)
    s = sf[sf_index(R, K, q.device)].view(torch.float8_e4m3fn).float()
    out = vals * (s * gs.float()).unsqueeze(-1)
    return out.view(R, K).to(dtype)


def quant_dequant_reference(x: torch.Tensor) -> torch.Tensor:
    """Round trip through the format (any leading shape, last dim a multiple of 64)."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    q, sf, gs = quantize_reference(x2)
    return dequantize_reference(q, sf, gs).view(shape).to(x.dtype)


# ------------------------------------------------------------------ kernels
def quantize(x: torch.Tensor):
    """``(q, sf, gs)`` of a 2-D CUDA tensor (bf16 / fp32), two launches, no host sync."""
    return tuple(ext().nvfp4_quantize(x.contiguous()))


def dequantize(q: torch.Tensor, sf: torch.Tensor, gs: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    return ext().nvfp4_dequantize(q, sf, gs, dtype)


def gemm(a, b, out: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``dequant(a) @ dequant(b).T (+ bias)`` in bf16 on the e2m1 tensor cores; ``a`` and ``b``
    are ``(q, sf, gs)`` triples of ``[M, K]`` and ``[N, K]`` (K a multiple of 256)."""
    aq, sfa, gsa = a
    bq, sfb, gsb = b
    if out is None:
        out = torch.empty(aq.shape[0], bq.shape[0], device=aq.device, dtype=torch.bfloat16)
    ext().gemm_nvfp4(aq, sfa, gsa, bq, sfb, gsb, out, bias)
    return out


def gemm_supported(k: int, n: int) -> bool:
    return k % 256 == 0 and k > 0 and n % 8 == 0
