"""Causal flash attention (MHA, GQA and MLA head dims) for sm_100a.

``flash_attention(q, k, v)`` takes q [B, S, Hq, Dqk], k [B, S, Hkv, Dqk],
v [B, S, Hkv, Dv] as (possibly strided) views - e.g. column slices of a fused
QKV projection output - and returns o [B, S, Hq, Dv] contiguous. The
[B, H, S, S] score matrix of the reference (src/models/deepseek.py:681-738,
src/models/attention.py:134-220) is never materialised: scores live on chip
and only the per-row log-sum-exp is kept for the backward pass.
"""
from __future__ import annotations

import math

import torch

from ._ext import ext

_KERNEL_HEAD_DIMS = {(64, 64), (128, 128), (192, 128)}


def _fwd(q, k, v, scale: float, causal: bool):
    """Forward kernel: the tcgen05 kernel for every supported head-dim pair ((128, 128), MLA's (192, 128),
    (64, 64)); ``NTB_ATTN_FWD_LEGACY=1`` selects the mma.sync kernel (kept as a cross-check)."""
    import os

    C = ext()
    if os.environ.get("NTB_ATTN_FWD_LEGACY") != "1":
        return C.flash_attn_fwd_tc(q, k, v, float(scale), bool(causal))
    return C.flash_attn_fwd(q, k, v, float(scale), bool(causal))


def _kernel_ok(q, k, v) -> bool:
    return (q.is_cuda and q.dtype == torch.bfloat16 and (q.shape[-1], v.shape[-1]) in _KERNEL_HEAD_DIMS
            and hasattr(ext(), "flash_attn_fwd"))


def attention_reference(q, k, v, causal=True, scale=None, mask=None):
    """fp32 math of softmax(q k^T * scale + mask) v on [B, S, H, D] tensors (GQA by repeat)."""
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf = q.float().permute(0, 2, 1, 3)
    kf = k.float().permute(0, 2, 1, 3)
    vf = v.float().permute(0, 2, 1, 3)
    if Hkv != Hq:
        rep = Hq // Hkv
        kf = kf.repeat_interleave(rep, dim=1)
        vf = vf.repeat_interleave(rep, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if mask is not None:
        s = s + mask
    elif causal:
        Sk = k.shape[1]
        cm = torch.ones(S, Sk, dtype=torch.bool, device=q.device).tril(Sk - S)
        s = s.masked_fill(~cm, float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = p @ vf
    return o.permute(0, 2, 1, 3).to(q.dtype).contiguous()


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, causal):
        o, lse = _fwd(q, k, v, scale, causal)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale, ctx.causal = scale, causal
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ext().flash_attn_bwd(do.contiguous(), q, k, v, o, lse, float(ctx.scale), bool(ctx.causal))
        return dq, dk, dv, None, None


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
                    softmax_scale: float | None = None) -> torch.Tensor:
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if q.is_cuda:
        if _kernel_ok(q, k, v):
            return _FlashAttnFn.apply(q, k, v, scale, causal)
        # Head dims without a tuned kernel (tiny test configs) run the math path.
        return _math_attention(q, k, v, scale, causal)
    return _math_attention(q, k, v, scale, causal)


def _math_attention(q, k, v, scale, causal):
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    qf = q.permute(0, 2, 1, 3)
    kf = k.permute(0, 2, 1, 3)
    vf = v.permute(0, 2, 1, 3)
    if Hkv != Hq:
        rep = Hq // Hkv
        kf = kf.repeat_interleave(rep, dim=1)
        vf = vf.repeat_interleave(rep, dim=1)
    s = torch.matmul(qf.float(), kf.float().transpose(-1, -2)) * scale
    if causal:
        Sk = k.shape[1]
        cm = torch.ones(S, Sk, dtype=torch.bool, device=q.device).tril(Sk - S)
        s = s.masked_fill(~cm, float("-inf"))
    p = torch.softmax(s, dim=-1).to(vf.dtype)
    o = torch.matmul(p, vf)
    return o.permute(0, 2, 1, 3).contiguous()


class _QKVAttentionFn(torch.autograd.Function):
    """RoPE(q, k) in place on the fused projection output, then causal flash attention.

    The backward writes dQ, dK, dV straight into one dQKV buffer shaped like
    the projection output and undoes the rotation on it in place, so no
    gather/scatter copies sit between the QKV GEMM and the attention kernels.
    """

    @staticmethod
    def forward(ctx, qkv, B, S, nq, nkv, dqk, dv, scale, rope_dim, rope_theta, rope_mode, causal):
        from .rope import rope_rows_

        C = ext()
        T = B * S
        q2 = qkv.view(T, -1)
        qv = q2[:, : nq * dqk].view(T, nq, dqk)
        kv = q2[:, nq * dqk: (nq + nkv) * dqk].view(T, nkv, dqk)
        if rope_dim:  # q and k heads are adjacent in the row: one launch rotates both
            rope_rows_(q2[:, : (nq + nkv) * dqk].view(T, nq + nkv, dqk), dqk - rope_dim, rope_dim, S,
                       float(rope_theta), rope_mode, False)
        ctx.mark_dirty(qkv)
        q4, k4, v4 = _split4(q2, B, S, nq, nkv, dqk, dv)
        o, lse = _fwd(q4, k4, v4, scale, causal)
        ctx.save_for_backward(qkv, o, lse)
        ctx.meta = (B, S, nq, nkv, dqk, dv, scale, rope_dim, rope_theta, rope_mode, causal)
        return qkv, o.view(B, S, nq * dv)

    @staticmethod
    def backward(ctx, _g_qkv, do):
        from .rope import rope_rows_

        qkv, o, lse = ctx.saved_tensors
        B, S, nq, nkv, dqk, dv, scale, rope_dim, rope_theta, rope_mode, causal = ctx.meta
        C = ext()
        T = B * S
        q2 = qkv.view(T, -1)
        q4, k4, v4 = _split4(q2, B, S, nq, nkv, dqk, dv)
        dqkv = torch.empty_like(q2)
        dq4, dk4, dv4 = _split4(dqkv, B, S, nq, nkv, dqk, dv)
        C.flash_attn_bwd(do.reshape(B, S, nq, dv).contiguous(), q4, k4, v4, o, lse, float(scale), bool(causal),
                         dq4, dk4, dv4)
        if rope_dim:
            rope_rows_(dqkv[:, : (nq + nkv) * dqk].view(T, nq + nkv, dqk), dqk - rope_dim, rope_dim, S,
                       float(rope_theta), rope_mode, True)
        return (dqkv.view_as(qkv),) + (None,) * 11


def _split4(q2, B, S, nq, nkv, dqk, dv):
    q4 = q2[:, : nq * dqk].view(B, S, nq, dqk)
    k4 = q2[:, nq * dqk: (nq + nkv) * dqk].view(B, S, nkv, dqk)
    v4 = q2[:, (nq + nkv) * dqk:].view(B, S, nkv, dv)
    return q4, k4, v4


def qkv_attention(qkv: torch.Tensor, B: int, S: int, nq: int, nkv: int, dqk: int, dv: int, *,
                  rope_dim: int = 0, rope_theta: float = 10000.0, rope_mode: str = "half", causal: bool = True,
                  softmax_scale: float | None = None) -> torch.Tensor:
    """Attention over a fused projection output qkv [B*S, nq*dqk + nkv*dqk + nkv*dv].

    RoPE (if ``rope_dim``) rotates the last ``rope_dim`` columns of every q/k
    head. Returns [B*S, nq*dv].
    """
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(dqk)
    T = B * S
    if qkv.is_cuda and qkv.dtype == torch.bfloat16 and (dqk, dv) in _KERNEL_HEAD_DIMS:
        _, o = _QKVAttentionFn.apply(qkv, B, S, nq, nkv, dqk, dv, scale, rope_dim, rope_theta, rope_mode, causal)
        return o.view(T, nq * dv)
    from .rope import apply_rope

    q = qkv[:, : nq * dqk].view(B, S, nq, dqk)
    k = qkv[:, nq * dqk: (nq + nkv) * dqk].view(B, S, nkv, dqk)
    v = qkv[:, (nq + nkv) * dqk:].view(B, S, nkv, dv)
    if rope_dim:
        q = torch.cat([q[..., : dqk - rope_dim], apply_rope(q[..., dqk - rope_dim:], rope_theta, rope_mode)], -1)
        k = torch.cat([k[..., : dqk - rope_dim], apply_rope(k[..., dqk - rope_dim:], rope_theta, rope_mode)], -1)
    return _math_attention(q, k, v, scale, causal).view(T, nq * dv)
