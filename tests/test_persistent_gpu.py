"""Persistent fp8 / NF4 weight refresh kernels against the PyTorch statement of the format
(same bits), per channel and per tensor. The oracle runs on the CPU: PyTorch's CUDA
tensor-by-scalar division multiplies by the reciprocal, while the kernels (like the CPU)
divide exactly."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gran", ["per_channel", "per_tensor"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(257, 384), (3, 5)])
def test_persistent_refresh_matches_reference(gran, dtype, shape):
    from nano_train_b200.ops._ext import check_status
    from nano_train_b200.precision import persistent as P

    dev = torch.device("cuda", 0)
    torch.manual_seed(shape[0])
    wc = (torch.randn(*shape) * torch.linspace(0.01, 2.0, shape[1])).to(dtype)
    wc[1].zero_()  # an all-zero channel takes the unit scale
    w = wc.to(dev)

    q, s = P.quantize_fp8_persistent(w, gran)
    q_ref, s_ref = P.quantize_fp8_persistent(wc, gran)
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.view(torch.uint8).cpu(), q_ref.view(torch.uint8))
    assert torch.equal(P.dequantize_fp8_persistent(q, s, gran, torch.float32).cpu(),
                       P.dequantize_fp8_persistent(q_ref, s_ref, gran, torch.float32))

    codes, s4 = P.quantize_nf4_persistent(w, gran)
    codes_ref, s4_ref = P.quantize_nf4_persistent(wc, gran)
    assert torch.equal(s4.cpu(), s4_ref)
    assert torch.equal(codes.cpu(), codes_ref)
    assert torch.equal(P.dequantize_nf4_persistent(codes, s4, shape, gran, dtype).cpu(),
                       P.dequantize_nf4_persistent(codes_ref, s4_ref, shape, gran, dtype))
    torch.cuda.synchronize()
    check_status(0)
