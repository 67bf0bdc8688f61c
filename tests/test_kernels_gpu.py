"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.fixture(scope="module")
def C():
    from nano_train_b200.ops._ext import ext
    return ext()


SHAPES = [(128, 128, 64), (256, 512, 256), (304, 200, 136), (1000, 777 * 8, 520), (2048, 4096, 1024)]


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_bf16(C, a_mn, b_mn, shape):
    M, N, K = shape
    torch.manual_seed(0)
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm_bf16(a, b, out, None, a_mn, b_mn, False, 1.0)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    assert rel_err(out, ref) < 1e-2, rel_err(out, ref)
    from nano_train_b200.ops._ext import check_status
    check_status(0)


def test_gemm_fp32_accumulate_bias(C):
    M, N, K = 384, 640, 192
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    out = torch.randn(M, N, device="cuda", dtype=torch.float32)
    ref = out + 0.5 * (A.float() @ B.float().t()) + bias.float()
    C.gemm_bf16(A, B, out, bias, False, False, True, 0.5)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-5


# Weight-gradient shapes of a tensor-parallel rank (Llama-8B, TP = 8, 4096 tokens) and of one GPU: the
# tile picker splits K into slices for most of them (fp32 C accumulated with atomics) and picks the
# 128-wide tile for some; ragged shapes check the edges of a split unit.
@pytest.mark.parametrize("M,N,K", [(768, 4096, 4096), (4096, 512, 4096), (3584, 4096, 4096), (4096, 1792, 4096),
                                   (6144, 4096, 4096), (1000, 520, 2056), (200, 136, 8192)])
def test_gemm_weight_grad_split_k(C, M, N, K):
    torch.manual_seed(M + N + K)
    dy = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)  # [tokens, out] (M-major A)
    x = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)   # [tokens, in]  (N-major B)
    out = torch.randn(M, N, device="cuda", dtype=torch.float32)
    ref = out + dy.float().t() @ x.float()
    C.gemm_bf16(dy, x, out, None, True, True, True, 1.0)
    torch.cuda.synchronize()
    from nano_train_b200.ops._ext import check_status
    check_status(0)
    assert rel_err(out, ref) < 1e-5, rel_err(out, ref)


def test_linear_autograd_matches_reference():
    from nano_train_b200.ops.linear import linear
    torch.manual_seed(0)
    x = torch.randn(4, 64, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(384, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    b = torch.randn(384, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = linear(x, w, b)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr, wr, br = (t.detach().float().requires_grad_() for t in (x, w, b))
    yr = F.linear(xr, wr, br)
    yr.backward(gy.float())
    assert rel_err(y, yr) < 1e-2
    assert rel_err(x.grad, xr.grad) < 1e-2
    assert rel_err(w.grad, wr.grad) < 1e-2
    assert rel_err(b.grad, br.grad) < 1e-2


def test_linear_main_grad_accumulation():
    from nano_train_b200.ops.linear import linear
    x = torch.randn(512, 256, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(128, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w.main_grad = torch.ones(128, 256, device="cuda", dtype=torch.float32)
    gy = torch.randn(512, 128, device="cuda", dtype=torch.bfloat16)
    linear(x, w).backward(gy)
    ref = 1.0 + gy.float().t() @ x.float()
    assert w.grad is None
    assert rel_err(w.main_grad, ref) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H", [128, 4096, 100])
def test_rmsnorm(dtype, H):
    from nano_train_b200.ops.norm import add_rms_norm, rms_norm
    x = torch.randn(64, H, device="cuda", dtype=dtype, requires_grad=True)
    r = torch.randn(64, H, device="cuda", dtype=dtype, requires_grad=True)
    w = (1 + 0.1 * torch.randn(H, device="cuda", dtype=dtype)).requires_grad_()
    y, h = add_rms_norm(x, r, w, 1e-5)
    gy = torch.randn_like(y)
    gh = torch.randn_like(h)
    (y * gy).sum().backward(retain_graph=True)
    (h * gh).sum().backward()
    xr, rr, wr = (t.detach().float().requires_grad_() for t in (x, r, w))
    hr = xr + rr
    yr = hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    ((yr * gy.float()).sum() + (hr * gh.float()).sum()).backward()
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert rel_err(y, yr) < tol
    assert rel_err(x.grad, xr.grad) < tol
    assert rel_err(w.grad, wr.grad) < tol
    y2 = rms_norm(x.detach(), w.detach(), 1e-5)
    assert rel_err(y2, xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr) < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,H", [(5003, 4096), (4099, 2048), (3001, 1536), (2999, 512), (1201, 8192),
                                    (777, 7168), (9, 4096)])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm_bwd_many_rows(dtype, rows, H, with_res):
    """Each CTA streams many rows through its shared-memory ring (stage reuse, parity flips,
    a remainder of rows in the last CTA); checked against fp32 PyTorch autograd."""
    from nano_train_b200.ops._ext import check_status, ext
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + H)
    h = torch.randn(rows, H, device="cuda", dtype=dtype, generator=g)
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(dtype)
    dy = torch.randn(rows, H, device="cuda", dtype=dtype, generator=g)
    dres = torch.randn(rows, H, device="cuda", dtype=dtype, generator=g) if with_res else None
    rstd = torch.rsqrt(h.float().pow(2).mean(-1) + 1e-5).contiguous()
    dx, dw = ext().rmsnorm_bwd(dy, h, w, rstd, dres)
    check_status(0)
    hf = h.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * wf).backward(dy.float())
    ref_dx = hf.grad + (dres.float() if with_res else 0)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert rel_err(dx, ref_dx) < tol
    assert rel_err(dw, wf.grad) < tol


def test_rmsnorm_weight_grad_into_main_grad():
    """A weight with an fp32 main_grad bucket view gets dW added there (no .grad, no bf16 rounding)."""
    from nano_train_b200.ops.norm import add_rms_norm
    H, rows = 2048, 3000
    x = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    r = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.nn.Parameter((1 + 0.1 * torch.randn(H, device="cuda")).to(torch.bfloat16))
    w.main_grad = torch.full((H,), 0.5, device="cuda")
    ready = []
    w._ntb_grad_ready_hook = lambda p: ready.append(p)
    y, h = add_rms_norm(x, r, w, 1e-5)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()
    assert w.grad is None and len(ready) == 1
    hr = (x.detach().float() + r.detach().float())
    wr = w.detach().float().requires_grad_()
    (hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr * gy.float()).sum().backward()
    assert rel_err(w.main_grad - 0.5, wr.grad) < 1e-2


def test_layernorm():
    from nano_train_b200.ops.norm import layer_norm
    x = torch.randn(32, 192, device="cuda", requires_grad=True)
    w = torch.randn(192, device="cuda", requires_grad=True)
    b = torch.randn(192, device="cuda", requires_grad=True)
    y = layer_norm(x, w, b, 1e-5)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr, br = (t.detach().clone().requires_grad_() for t in (x, w, b))
    yr = F.layer_norm(xr, (192,), wr, br, 1e-5)
    yr.backward(g)
    assert rel_err(y, yr) < 1e-5
    assert rel_err(x.grad, xr.grad) < 1e-4
    assert rel_err(w.grad, wr.grad) < 1e-4
    assert rel_err(b.grad, br.grad) < 1e-4


@pytest.mark.parametrize("mode", ["half", "deepseek"])
def test_rope(mode):
    from nano_train_b200.ops.rope import apply_rope, rope_reference
    x = torch.randn(2, 48, 4, 64, device="cuda", requires_grad=True)
    y = apply_rope(x, 10000.0, mode)
    pos = torch.arange(48, device="cuda")
    xr = x.detach().clone().requires_grad_()
    yr = rope_reference(xr, pos, 10000.0, mode)
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g)
    assert rel_err(y, yr) < 1e-5
    assert rel_err(x.grad, xr.grad) < 1e-5


@pytest.mark.parametrize("mode", ["half", "deepseek"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dqk,R", [(128, 128), (192, 64)])
@pytest.mark.parametrize("inverse", [False, True])
def test_rope_table_rows(mode, dtype, dqk, R, inverse):
    """Vectorised table RoPE on q|k heads of a fused projection row (rotary part at the end of each
    head, as in MLA's [nope | rope]) against the fp32 PyTorch statement."""
    from nano_train_b200.ops.rope import rope_reference, rope_rows_
    B, S, nq, nkv = 2, 200, 4, 2
    width = (nq + nkv) * dqk + nkv * 128
    x = torch.randn(B * S, width, device="cuda", dtype=dtype)
    ref = x.clone()
    heads = x[:, : (nq + nkv) * dqk].view(B * S, nq + nkv, dqk)
    rope_rows_(heads, dqk - R, R, S, 5e5, mode, inverse)
    r = ref[:, : (nq + nkv) * dqk].view(B, S, nq + nkv, dqk)[..., dqk - R:]
    exp = rope_reference(r.float(), torch.arange(S, device="cuda"), 5e5, mode, inverse=inverse)
    got = x[:, : (nq + nkv) * dqk].view(B, S, nq + nkv, dqk)
    assert rel_err(got[..., dqk - R:], exp) < (1e-5 if dtype == torch.float32 else 8e-3)
    torch.testing.assert_close(got[..., : dqk - R], ref[:, : (nq + nkv) * dqk].view(B, S, nq + nkv, dqk)[..., : dqk - R])
    torch.testing.assert_close(x[:, (nq + nkv) * dqk:], ref[:, (nq + nkv) * dqk:])  # v untouched


@pytest.mark.parametrize("B,S,h,Dn,Dv,R,lat", [(2, 128, 16, 128, 128, 64, 512), (1, 100, 3, 128, 128, 64, 64),
                                                (3, 37, 5, 64, 64, 16, 48)])
def test_mla_k_assemble(C, B, S, h, Dn, Dv, R, lat):
    """MLA key assembly [k_nope | rope(k_rope) broadcast over heads] and its backward (nope part of dK
    copied into dkv, rope part summed over heads and rotated back) against the fp32 PyTorch statement."""
    from nano_train_b200.ops.rope import rope_reference, rope_table
    torch.manual_seed(0)
    theta = 1e4
    kv = torch.randn(B, S, h * (Dn + Dv), device="cuda", dtype=torch.bfloat16).view(B, S, h, Dn + Dv)
    kv_a = torch.randn(B, S, lat + R, device="cuda", dtype=torch.bfloat16)
    k_rope = kv_a[..., lat:]
    table = rope_table(S, R, theta, kv.device)
    kf = C.mla_k_assemble(kv.reshape(B * S, h, Dn + Dv), k_rope.reshape(B * S, R), table, Dn, S).view(B, S, h, Dn + R)
    pos = torch.arange(S, device="cuda")
    rot = rope_reference(k_rope.float().unsqueeze(2), pos, theta, "deepseek")
    assert torch.equal(kf[..., :Dn], kv[..., :Dn])
    assert rel_err(kf[..., Dn:], rot.expand(B, S, h, R)) < 8e-3
    dk = torch.randn(B, S, h, Dn + R, device="cuda", dtype=torch.bfloat16)
    dkv = torch.full((B, S, h, Dn + Dv), 7.0, device="cuda", dtype=torch.bfloat16)
    dkr = C.mla_k_assemble_bwd(dk.view(B * S, h, Dn + R), dkv.view(B * S, h, Dn + Dv), table, Dn, S)
    assert torch.equal(dkv[..., :Dn], dk[..., :Dn])
    assert bool((dkv[..., Dn:] == 7).all())
    exp = rope_reference(dk[..., Dn:].float().sum(2, keepdim=True), pos, theta, "deepseek", inverse=True)
    assert rel_err(dkr.view(B, S, R), exp[:, :, 0]) < 8e-3


def test_swiglu_gelu():
    from nano_train_b200.ops.activation import gelu, swiglu
    gu = torch.randn(40, 2 * 96, device="cuda", requires_grad=True)
    y = swiglu(gu)
    g = torch.randn_like(y)
    y.backward(g)
    gr = gu.detach().clone().requires_grad_()
    a, b = gr.chunk(2, -1)
    (F.silu(a) * b).backward(g)
    assert rel_err(y, F.silu(a) * b) < 1e-5
    assert rel_err(gu.grad, gr.grad) < 1e-5
    x = torch.randn(1000, device="cuda", requires_grad=True)
    y = gelu(x)
    y.backward(torch.ones_like(y))
    xr = x.detach().clone().requires_grad_()
    F.gelu(xr).backward(torch.ones_like(y))
    assert rel_err(y, F.gelu(xr)) < 1e-5
    assert rel_err(x.grad, xr.grad) < 1e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cross_entropy(dtype):
    from nano_train_b200.ops.loss import cross_entropy
    logits = torch.randn(37, 1000, device="cuda", dtype=dtype, requires_grad=True)
    labels = torch.randint(0, 1000, (37,), device="cuda")
    labels[3] = -100
    loss = cross_entropy(logits, labels)
    loss.backward()
    lr = logits.detach().float().requires_grad_()
    ref = F.cross_entropy(lr, labels)
    ref.backward()
    assert abs(loss.item() - ref.item()) < (1e-4 if dtype == torch.float32 else 1e-2)
    assert rel_err(logits.grad, lr.grad) < (1e-4 if dtype == torch.float32 else 2e-2)


def test_embedding():
    from nano_train_b200.ops.embedding import embedding
    W = torch.randn(100, 64, device="cuda", requires_grad=True)
    ids = torch.randint(0, 100, (4, 16), device="cuda")
    y = embedding(ids, W)
    g = torch.randn_like(y)
    y.backward(g)
    Wr = W.detach().clone().requires_grad_()
    F.embedding(ids, Wr).backward(g)
    assert torch.equal(y, F.embedding(ids, W.detach()))
    assert rel_err(W.grad, Wr.grad) < 1e-6


def test_adamw_flat_matches_torch():
    from nano_train_b200.ops.optim import adamw_flat_
    torch.manual_seed(0)
    n = 1001
    p = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    ref = torch.nn.Parameter(p.clone())
    opt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for step in range(1, 7):
        g = torch.randn(n, device="cuda")
        ref.grad = g.clone()
        opt.step()
        adamw_flat_(p, m, v, g, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=step, param_bf16=pb)
    torch.testing.assert_close(p, ref.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(pb.float(), ref.detach(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("n", [5000, 5003, 3, 1 << 22])
def test_grad_stats(n):
    """Sum of squares, optional in-place unscale and the non-finite flag: the fp32 vector kernel
    (n % 4 tails included) and the scalar one."""
    from nano_train_b200.ops.optim import grad_stats_
    gb = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    outb = torch.zeros(2, device="cuda")
    grad_stats_(gb, outb)
    refb = gb.float().pow(2).sum()
    assert abs(outb[0].item() - refb.item()) / refb.item() < 1e-4
    g = torch.randn(n, device="cuda")
    g_half = g * 0.5
    out = torch.zeros(2, device="cuda")
    inv = torch.tensor([0.5], device="cuda")
    ref = (g * 0.5).pow(2).sum()
    grad_stats_(g, out, inv)
    assert abs(out[0].item() - ref.item()) / ref.item() < 1e-4
    assert out[1].item() == 0
    torch.testing.assert_close(g, g_half, rtol=0, atol=0)  # unscaled in place
    g[n - 1] = float("inf")  # the last element: in the tail when n % 4 != 0
    grad_stats_(g, out)
    assert out[1].item() == 1


@pytest.mark.parametrize("dims", [(64, 64), (128, 128), (192, 128)])
@pytest.mark.parametrize("S", [128, 200, 512])
@pytest.mark.parametrize("heads", [(4, 4), (8, 2)])
def test_flash_attention(dims, S, heads):
    from nano_train_b200.ops.attention import attention_reference, flash_attention
    dqk, dv = dims
    hq, hkv = heads
    torch.manual_seed(0)
    B = 2
    # q/k/v as strided views of one fused projection output, like the model uses
    qkv = torch.randn(B, S, hq * dqk + hkv * dqk + hkv * dv, device="cuda", dtype=torch.bfloat16)
    q = qkv[..., : hq * dqk].view(B, S, hq, dqk)
    k = qkv[..., hq * dqk: hq * dqk + hkv * dqk].view(B, S, hkv, dqk)
    v = qkv[..., hq * dqk + hkv * dqk:].view(B, S, hkv, dv)
    q, k, v = (t.detach().requires_grad_() for t in (q, k, v))
    o = flash_attention(q, k, v, causal=True)
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = attention_reference(qr, kr, vr, causal=True)
    orf.backward(g.float())
    assert rel_err(o, orf) < 1e-2, rel_err(o, orf)
    assert rel_err(q.grad, qr.grad) < 2e-2, rel_err(q.grad, qr.grad)
    assert rel_err(k.grad, kr.grad) < 2e-2, rel_err(k.grad, kr.grad)
    assert rel_err(v.grad, vr.grad) < 2e-2, rel_err(v.grad, vr.grad)
