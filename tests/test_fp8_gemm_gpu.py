"""Block-scaled e4m3 GEMM (DeepSeek-V3 recipe) vs fp32 math on the dequantised operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("M,N,K,bias", [(256, 384, 512, False), (300, 200, 256, True), (1024, 1024, 1024, False),
                                         (128, 8, 128, True)])
def test_gemm_fp8_blockscaled(M, N, K, bias):
    from nano_train_b200.ops._ext import check_status, ext

    C = ext()
    dev = torch.device("cuda", 0)
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16) * torch.linspace(0.1, 3.0, K, device=dev).to(torch.bfloat16)
    w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.05
    b = torch.randn(N, device=dev, dtype=torch.bfloat16) if bias else None
    xq, sx = C.fp8_quantize(x, 1, False, 0)
    wq, sw = C.fp8_quantize(w, 128, False, 0)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    C.gemm_fp8_blockscaled(xq, sx, wq, sw, y, b)
    torch.cuda.synchronize()
    check_status(0)
    xd = C.fp8_dequantize(xq, sx, 1, torch.float32)
    wd = C.fp8_dequantize(wq, sw, 128, torch.float32)
    ref = xd @ wd.t() + (b.float() if bias else 0)
    assert _rel(y, ref) < 5e-3
    # and close to the unquantised product (fp8 error only)
    assert _rel(y, x.float() @ w.float().t() + (b.float() if bias else 0)) < 6e-2


def test_native_fp8_linear_forward_backward():
    from nano_train_b200.precision.backends import NativeFP8Backend

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    be = NativeFP8Backend()
    x = torch.randn(4, 64, 256, device=dev, dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(512, 256, device=dev, dtype=torch.bfloat16) * 0.05).requires_grad_(True)
    y = be.linear(x, w, None)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = xr @ wr.t()
    yr.backward(g.float())
    assert _rel(y, yr) < 6e-2
    assert _rel(x.grad, xr.grad) < 6e-2
    assert _rel(w.grad, wr.grad) < 6e-2


def test_native_fp8_dgrad_matches_bf16_dgrad(monkeypatch):
    """The input gradient on e4m3 operands (dY in 1x128 tiles, W^T codes) against the bf16 GEMM on
    the dequantised weight, and the transposed weight codes against a transposed quantisation."""
    from nano_train_b200.ops._ext import ext
    from nano_train_b200.precision.backends import NativeFP8Backend, _quantized_weight, _quantized_weight_t

    torch.manual_seed(1)
    be = NativeFP8Backend()
    x = torch.randn(300, 384, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(640, 384, device="cuda", dtype=torch.bfloat16) * 0.05).requires_grad_(True)
    g = torch.randn(300, 640, device="cuda", dtype=torch.bfloat16)
    grads = {}
    for native in ("1", "0"):
        monkeypatch.setenv("NTB_FP8_DGRAD_NATIVE", native)
        xx = x.clone().requires_grad_(True)
        be.linear(xx, w, None).backward(g)
        grads[native] = xx.grad
    assert _rel(grads["1"], grads["0"]) < 5e-2
    wq, sw = _quantized_weight(w)
    wtq, swt = _quantized_weight_t(w, wq, sw)
    q2, s2 = ext().fp8_quantize(w.detach().t().contiguous(), 128, False, 0)
    assert torch.equal(wtq, q2) and torch.equal(swt, s2)
