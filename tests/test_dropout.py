"""Counter-based dropout: Philox-4x32-10 known-answer vectors (Random123's published KAT),
keep statistics, regenerated-mask backward; the CUDA kernel against the numpy oracle."""
import numpy as np
import pytest
import torch

from nano_train_b200.ops.dropout import _DropoutFn, dropout, philox4x32_10, philox_keep_reference


@pytest.mark.parametrize("ctr,key,want", [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
])
def test_philox_known_answers(ctr, key, want):
    out = philox4x32_10(*(np.array([c], dtype=np.uint64) for c in ctr), *key)
    assert tuple(int(o[0]) for o in out) == want


def test_keep_fraction_and_scaling_cpu():
    keep = philox_keep_reference(200_000, 0.3, seed=1234)
    assert abs(keep.float().mean().item() - 0.7) < 0.01
    x = torch.ones(1000)
    y = _DropoutFn.apply(x, 0.25, 7)
    assert torch.allclose(y[y != 0], torch.full_like(y[y != 0], 1 / 0.75))


def test_backward_reuses_the_mask_cpu():
    x = torch.randn(3, 333, requires_grad=True)
    y = _DropoutFn.apply(x, 0.5, 99)
    y.sum().backward()
    assert torch.equal(x.grad != 0, y.detach() != 0) or torch.equal(x.grad != 0, philox_keep_reference(999, 0.5, 99).view(3, 333))
    assert dropout(x, 0.0) is x


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_dropout_kernel_matches_reference(dtype):
    from nano_train_b200.ops._ext import check_status

    dev = torch.device("cuda", 0)
    n = 3 * 1000 + 3
    x = torch.randn(n, device=dev).to(dtype).requires_grad_(True)
    seed = (1 << 40) + 17
    y = _DropoutFn.apply(x, 0.1, seed)
    keep = philox_keep_reference(n, 0.1, seed).to(dev)
    scale = float(np.float32(1.0 / (1.0 - 0.1)))  # the kernel multiplies by the fp32 reciprocal
    want = torch.where(keep, x.detach().float() * scale, torch.zeros_like(x.detach().float())).to(dtype)
    assert torch.equal(y.detach(), want)
    g = torch.randn_like(y)
    y.backward(g)
    assert torch.equal(x.grad, torch.where(keep, g.float() * scale, torch.zeros_like(g.float())).to(dtype))
    torch.cuda.synchronize()
    check_status(0)
