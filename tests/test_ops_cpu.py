"""CPU paths of the op wrappers against independent PyTorch math.

On CPU tensors every op runs its PyTorch formulation; these tests pin those
formulations (the same oracles the GPU kernel tests compare against) to the
reference's math: RoPE layouts, cross-entropy with ignore_index, GQA causal
attention, RMSNorm / LayerNorm, SwiGLU / GELU, AdamW.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from nano_train_b200.ops.activation import gelu, swiglu
from nano_train_b200.ops.attention import attention_reference, flash_attention
from nano_train_b200.ops.linear import gemm, linear
from nano_train_b200.ops.loss import cross_entropy
from nano_train_b200.ops.norm import add_rms_norm, layer_norm, rms_norm
from nano_train_b200.ops.optim import adamw_flat_, grad_stats_
from nano_train_b200.ops.rope import apply_rope, rope_reference


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_majors(a_mn, b_mn):
    torch.manual_seed(0)
    M, N, K = 17, 9, 33
    A = torch.randn(M, K)
    B = torch.randn(N, K)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    bias = torch.randn(N)
    out = gemm(a, b, bias=bias, a_mn=a_mn, b_mn=b_mn, alpha=0.5)
    torch.testing.assert_close(out, 0.5 * A @ B.t() + bias)
    acc = torch.ones(M, N)
    gemm(a, b, acc, a_mn=a_mn, b_mn=b_mn, accumulate=True)
    torch.testing.assert_close(acc, 1 + A @ B.t())


def test_linear_autograd_cpu():
    torch.manual_seed(1)
    x = torch.randn(4, 6, 16, requires_grad=True)
    w = torch.randn(8, 16, requires_grad=True)
    b = torch.randn(8, requires_grad=True)
    y = linear(x, w, b)
    y.square().sum().backward()
    x2, w2, b2 = (t.detach().clone().requires_grad_(True) for t in (x, w, b))
    F.linear(x2, w2, b2).square().sum().backward()
    for t, r in ((x, x2), (w, w2), (b, b2)):
        torch.testing.assert_close(t.grad, r.grad)


def _rotate_half_interleaved(x):
    return torch.stack((-x[..., 1::2], x[..., ::2]), dim=-1).flatten(-2)


def test_rope_deepseek_layout_matches_reference_formula():
    """x * cos + rotate_half(x) * sin with interleaved rotate and cat(freqs, freqs) cache."""
    torch.manual_seed(2)
    B, S, H, R, theta = 2, 7, 3, 16, 10000.0
    x = torch.randn(B, S, H, R)
    inv = 1.0 / (theta ** (torch.arange(0, R, 2).float() / R))
    freqs = torch.outer(torch.arange(S).float(), inv)
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = emb.cos()[None, :, None, :], emb.sin()[None, :, None, :]
    expect = x * cos + _rotate_half_interleaved(x) * sin
    torch.testing.assert_close(apply_rope(x, theta, "deepseek"), expect, rtol=1e-5, atol=1e-5)


def test_rope_half_layout_and_inverse():
    torch.manual_seed(3)
    B, S, H, R, theta = 2, 5, 4, 8, 500000.0
    x = torch.randn(B, S, H, R)
    inv = 1.0 / (theta ** (torch.arange(0, R, 2).float() / R))
    ang = torch.outer(torch.arange(S).float(), inv)[None, :, None, :]
    x1, x2 = x[..., : R // 2], x[..., R // 2:]
    expect = torch.cat([x1 * ang.cos() - x2 * ang.sin(), x2 * ang.cos() + x1 * ang.sin()], -1)
    y = apply_rope(x, theta, "half")
    torch.testing.assert_close(y, expect, rtol=1e-5, atol=1e-5)
    pos = torch.arange(S).double()
    xd = x.double()
    # rotate-half is a rotation: the transposed map inverts it
    back = rope_reference(rope_reference(xd, pos, theta, "half"), pos, theta, "half", inverse=True)
    torch.testing.assert_close(back, xd)
    # both layouts: inverse=True is the adjoint (the backward map), <R x, g> == <x, R^T g>
    g = torch.randn_like(xd)
    for mode in ("half", "deepseek"):
        lhs = (rope_reference(xd, pos, theta, mode) * g).sum()
        rhs = (xd * rope_reference(g, pos, theta, mode, inverse=True)).sum()
        torch.testing.assert_close(lhs, rhs)


def test_cross_entropy_ignore_index():
    torch.manual_seed(4)
    logits = torch.randn(3, 5, 11)
    labels = torch.randint(0, 11, (3, 5))
    labels[0, 0] = -100
    labels[2, 3] = -100
    for red in ("mean", "sum", "none"):
        got = cross_entropy(logits, labels, reduction=red)
        ref = F.cross_entropy(logits.reshape(-1, 11), labels.reshape(-1), ignore_index=-100, reduction=red)
        torch.testing.assert_close(got, ref)


@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2)])
def test_attention_reference_gqa_causal(hq, hkv):
    torch.manual_seed(5)
    B, S, D = 2, 9, 16
    q, k, v = torch.randn(B, S, hq, D), torch.randn(B, S, hkv, D), torch.randn(B, S, hkv, D)
    out = attention_reference(q, k, v, causal=True)
    rep = hq // hkv
    for b in range(B):
        for h in range(hq):
            s = q[b, :, h] @ k[b, :, h // rep].t() / math.sqrt(D)
            s = s.masked_fill(torch.ones(S, S).triu(1).bool(), float("-inf"))
            o = torch.softmax(s, -1) @ v[b, :, h // rep]
            torch.testing.assert_close(out[b, :, h], o, rtol=1e-5, atol=1e-5)
    # the dispatching entry falls back to the same math on CPU, with autograd
    qq = q.clone().requires_grad_(True)
    flash_attention(qq, k, v, causal=True).sum().backward()
    assert qq.grad is not None and torch.isfinite(qq.grad).all()


def test_norms():
    torch.manual_seed(6)
    x = torch.randn(4, 32)
    r = torch.randn(4, 32)
    w = torch.randn(32)
    b = torch.randn(32)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    torch.testing.assert_close(rms_norm(x, w, 1e-6), ref)
    y, h = add_rms_norm(x, r, w, 1e-6)
    torch.testing.assert_close(h, x + r)
    torch.testing.assert_close(y, (x + r) * torch.rsqrt((x + r).pow(2).mean(-1, keepdim=True) + 1e-6) * w)
    torch.testing.assert_close(layer_norm(x, w, b, 1e-5), F.layer_norm(x, (32,), w, b, 1e-5))


def test_activations():
    torch.manual_seed(7)
    gu = torch.randn(5, 12)
    torch.testing.assert_close(swiglu(gu), F.silu(gu[:, :6]) * gu[:, 6:])
    x = torch.randn(5, 12)
    torch.testing.assert_close(gelu(x), 0.5 * x * (1 + torch.erf(x / math.sqrt(2))))


def test_adamw_flat_matches_torch():
    torch.manual_seed(8)
    p0 = torch.randn(50)
    grads = [torch.randn(50) for _ in range(4)]
    ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    p, m, v = p0.clone(), torch.zeros(50), torch.zeros(50)
    for step, g in enumerate(grads, 1):
        ref.grad = g.clone()
        opt.step()
        adamw_flat_(p, m, v, g, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=step)
    torch.testing.assert_close(p, ref.detach(), rtol=1e-6, atol=1e-6)
    # skip flag and grad scale
    before = p.clone()
    adamw_flat_(p, m, v, grads[0], lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=5,
                skip=torch.ones(1, dtype=torch.int32))
    torch.testing.assert_close(p, before)


def test_grad_stats():
    g = torch.tensor([3.0, 4.0])
    out = torch.zeros(2)
    grad_stats_(g, out, inv_scale=torch.tensor(0.5))
    torch.testing.assert_close(out, torch.tensor([6.25, 0.0]))
    grad_stats_(torch.tensor([float("inf")]), out)
    assert out[1] == 1.0
