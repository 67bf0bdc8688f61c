"""NVFP4 kernels on the B200: the quantiser and dequantiser against their PyTorch
restatement (bit for bit), and the e2m1 block-scaled tcgen05 GEMM against fp32 math on
the dequantised operands."""
import pytest
import torch

from nano_train_b200.ops import fp4

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


# Bound for the e2m1 GEMM against the fp32 product of its dequantised operands: the measured error
# is the bf16 rounding of the output alone (1.66e-3 for K from 256 to 16384). Quantisation oracles
# run on the CPU: the kernels divide exactly, while PyTorch on CUDA turns a division by a Python
# scalar into a multiplication by its reciprocal, which moves some e4m3 / e2m1 roundings.
GEMM_TOL = 5e-3


@pytest.mark.parametrize("R,K,dtype", [(300, 512, torch.bfloat16), (128, 64, torch.float32), (1000, 2048, torch.bfloat16)])
def test_quantize_matches_reference(R, K, dtype):
    from nano_train_b200.ops._ext import check_status

    dev = torch.device("cuda", 0)
    torch.manual_seed(R + K)
    x = (torch.randn(R, K, device=dev) * torch.linspace(0.01, 8.0, K, device=dev)).to(dtype)
    q, sf, gs = fp4.quantize(x)
    torch.cuda.synchronize()
    check_status(0)
    rq, rsf, rgs = fp4.quantize_reference(x)
    assert torch.equal(gs, rgs)
    assert torch.equal(sf, rsf)
    # codes agree up to the sign of zero (the hardware keeps -0, the restatement writes +0)
    assert torch.equal(fp4.dequantize_reference(q, sf, gs), fp4.dequantize_reference(rq, rsf, rgs))
    d = fp4.dequantize(q, sf, gs, torch.float32)
    assert torch.equal(d, fp4.dequantize_reference(q, sf, gs))


@pytest.mark.parametrize("M,N,K,bias", [(256, 256, 256, False), (300, 384, 512, True), (1024, 1024, 2048, False),
                                         (128, 8, 256, True), (2048, 1536, 1024, True)])
def test_gemm_nvfp4(M, N, K, bias):
    from nano_train_b200.ops._ext import check_status

    dev = torch.device("cuda", 0)
    torch.manual_seed(M * 7 + N + K)
    x = (torch.randn(M, K, device=dev) * torch.linspace(0.1, 3.0, K, device=dev)).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
    b = torch.randn(N, device=dev, dtype=torch.bfloat16) if bias else None
    a = fp4.quantize(x)
    bw = fp4.quantize(w)
    y = fp4.gemm(a, bw, bias=b)
    torch.cuda.synchronize()
    check_status(0)
    ref = fp4.dequantize_reference(*a) @ fp4.dequantize_reference(*bw).t() + (b.float() if bias else 0)
    assert torch.isfinite(y).all()
    assert _rel(y, ref) < GEMM_TOL
    # two calls in a row give the same bits (fixed accumulation order)
    y2 = fp4.gemm(a, bw, bias=b)
    assert torch.equal(y, y2)


def test_native_fp4_linear_forward_backward():
    from nano_train_b200.precision.backends import NativeFP4Backend

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    be = NativeFP4Backend()
    x = torch.randn(4, 64, 512, device=dev, dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(768, 512, device=dev, dtype=torch.bfloat16) * 0.05).requires_grad_(True)
    y = be.linear(x, w, None)
    g = torch.randn_like(y)
    y.backward(g)
    xq = fp4.quant_dequant_reference(x.detach().float().cpu().view(-1, 512)).to(dev)
    wq = fp4.quant_dequant_reference(w.detach().float().cpu()).to(dev)
    yr = (xq @ wq.t()).view_as(y)
    assert _rel(y, yr) < GEMM_TOL
    assert _rel(x.grad.view(-1, 512), g.float().view(-1, 768) @ wq) < 1e-2
    assert _rel(w.grad, g.float().view(-1, 768).t() @ xq) < 1e-2
    # and close to the unquantised product (fp4 error only)
    assert _rel(y, x.detach().float() @ w.detach().float().t()) < 0.2
