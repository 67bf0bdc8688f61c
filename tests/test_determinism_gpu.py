"""Determinism: kernels whose algorithm has a fixed reduction order must give bit-identical results when
run twice on the same inputs (GEMM and its fp32 accumulate form, tcgen05 attention forward, RMSNorm forward
and backward, SwiGLU, cross-entropy, fused AdamW, grouped expert GEMM, block-scaled fp8 GEMM, router
selection). Kernels that add partial sums with atomics (attention dQ, router probability sums) are left
out on purpose."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _twice(fn):
    torch.manual_seed(0)
    a = fn()
    torch.cuda.synchronize()
    torch.manual_seed(0)
    b = fn()
    torch.cuda.synchronize()
    return a, b


def _same(a, b):
    if isinstance(a, (tuple, list)):
        return all(_same(x, y) for x, y in zip(a, b))
    return torch.equal(a, b)


@pytest.fixture(scope="module")
def C():
    from nano_train_b200.ops._ext import ext
    return ext()


def test_gemm_deterministic(C):
    x = torch.randn(1024, 2048, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3072, 2048, device="cuda", dtype=torch.bfloat16)

    def run():
        y = torch.empty(1024, 3072, device="cuda", dtype=torch.bfloat16)
        C.gemm_bf16(x, w, y, None, False, False, False, 1.0)
        acc = torch.ones(3072, 2048, device="cuda", dtype=torch.float32)
        C.gemm_bf16(y, x, acc, None, True, True, True, 1.0)  # weight-gradient form, fp32 accumulate
        return y, acc

    assert _same(*_twice(run))


def test_attention_forward_deterministic(C):
    qkv = torch.randn(1, 1024, 12, 128, device="cuda", dtype=torch.bfloat16)
    q, k, v = qkv[:, :, :8], qkv[:, :, 8:10], qkv[:, :, 10:]
    assert _same(*_twice(lambda: C.flash_attn_fwd_tc(q, k, v, 128 ** -0.5, True)))


def test_norm_activation_loss_deterministic():
    from nano_train_b200 import ops

    x0 = torch.randn(512, 4096, device="cuda", dtype=torch.bfloat16)
    r0 = torch.randn(512, 4096, device="cuda", dtype=torch.bfloat16)
    w0 = torch.randn(4096, device="cuda", dtype=torch.bfloat16)
    gu = torch.randn(512, 2 * 1408, device="cuda", dtype=torch.bfloat16)
    logits = torch.randn(512, 32000, device="cuda", dtype=torch.bfloat16)
    labels = torch.randint(0, 32000, (512,), device="cuda")

    def run():
        x, r, w = (t.clone().requires_grad_() for t in (x0, r0, w0))
        y, h = ops.add_rms_norm(x, r, w, 1e-5)
        (y.float().square().sum() + h.float().sum()).backward()
        lg = logits.clone().requires_grad_()
        loss = ops.cross_entropy(lg, labels)
        loss.backward()
        return y, x.grad, w.grad, ops.swiglu(gu), loss.detach(), lg.grad

    assert _same(*_twice(run))


def test_adamw_grouped_fp8_router_deterministic(C):
    from nano_train_b200.ops.grouped import pad_segments

    n = 1 << 20
    g = torch.randn(n, device="cuda")
    p0, m0, v0 = torch.randn(n, device="cuda"), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    counts = torch.tensor([300, 0, 129, 77], device="cuda")
    off, rows = pad_segments(counts)
    xg = torch.randn(rows, 512, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(4 * 384, 512, device="cuda", dtype=torch.bfloat16)
    xa = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    wa = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    xq, sx = C.fp8_quantize(xa, 1, False, 0)
    wq, sw = C.fp8_quantize(wa, 128, False, 0)
    logits = torch.randn(4096, 64, device="cuda", dtype=torch.bfloat16)

    def run():
        p, m, v = p0.clone(), m0.clone(), v0.clone()
        C.adamw_flat_(p, m, v, g, None, 1e-3, 0.9, 0.95, 1e-8, 0.1, 3, None, None)
        yg = torch.empty(rows, 384, device="cuda", dtype=torch.bfloat16)
        C.gemm_grouped_bf16(xg, wg, yg, off, 1)
        yq = torch.empty(512, 512, device="cuda", dtype=torch.bfloat16)
        C.gemm_fp8_blockscaled(xq, sx, wq, sw, yq)
        idx, w, counts_out, _ = C.router_fwd(logits, 6, True, 1, 1, True, 1.0)
        return p, m, v, yg, yq, idx, w, counts_out

    assert _same(*_twice(run))
