"""NVFP4 format (e2m1 in 1x16 groups, e4m3 group scales in tensor-core scale blocks,
fp32 tensor scale): the PyTorch restatement of the kernels, checked on CPU."""
import pytest
import torch

from nano_train_b200.ops import fp4


def test_e2m1_round_to_nearest_even_and_saturation():
    y = torch.tensor([0.0, 0.2, 0.25, 0.3, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 7.0, 100.0, -0.75, -5.0, -0.1])
    got = fp4.e2m1_decode(fp4.e2m1_encode(y))
    want = torch.tensor([0.0, 0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, 6.0, -1.0, -4.0, 0.0])
    assert torch.equal(got, want)


def test_scale_block_layout_is_a_bijection():
    R, K = 300, 192
    idx = fp4.sf_index(R, K).reshape(-1)
    assert idx.numel() == R * K // 16
    assert idx.unique().numel() == idx.numel()
    assert int(idx.max()) < fp4.sf_bytes(R, K)
    # a 128-row block holds 4 scales of each row in one 32-bit word, rows 32 apart in adjacent words
    assert int(fp4.sf_index(128, 64)[0, 1]) == 1
    assert int(fp4.sf_index(128, 64)[32, 0]) == 4
    assert int(fp4.sf_index(128, 64)[1, 0]) == 16
    assert int(fp4.sf_index(128, 128)[0, 4]) == 512


@pytest.mark.parametrize("R,K", [(1, 64), (130, 128), (64, 256)])
def test_quantize_round_trip_error_bound(R, K):
    torch.manual_seed(R + K)
    x = torch.randn(R, K) * torch.linspace(0.01, 10.0, K)
    q, sf, gs = fp4.quantize_reference(x)
    assert q.shape == (R, K // 2) and q.dtype == torch.uint8
    assert sf.numel() == fp4.sf_bytes(R, K)
    xd = fp4.dequantize_reference(q, sf, gs)
    g = x.view(R, K // 16, 16)
    err = (xd.view_as(g) - g).abs().amax(-1)
    bmax = g.abs().amax(-1)
    # e2m1 spacing near the top of a group is 2 (of 6), the e4m3 scale adds 1/16 relative
    assert bool((err <= bmax * (1.0 / 6.0 + 1.0 / 16.0) + 1e-6).all())
    # padded rows of the last scale block are zero
    valid = torch.zeros(fp4.sf_bytes(R, K), dtype=torch.bool)
    valid[fp4.sf_index(R, K).reshape(-1)] = True
    assert int(sf[~valid].abs().sum()) == 0


def test_all_zero_tensor_uses_unit_scale():
    q, sf, gs = fp4.quantize_reference(torch.zeros(4, 64))
    assert float(gs) == 1.0 and int(q.sum()) == 0 and int(sf.sum()) == 0


def test_native_fp4_backend_cpu_ste():
    from nano_train_b200.precision.backends import NativeFP4Backend

    torch.manual_seed(0)
    be = NativeFP4Backend()
    x = torch.randn(2, 8, 128, requires_grad=True)
    w = (torch.randn(64, 128) * 0.05).requires_grad_(True)
    y = be.linear(x, w, None)
    assert y.shape == (2, 8, 64)
    ref = fp4.quant_dequant_reference(x.detach()) @ fp4.quant_dequant_reference(w.detach()).t()
    torch.testing.assert_close(y.detach(), ref, rtol=1e-5, atol=1e-5)
    y.sum().backward()
    # straight-through: gradients are those of the unquantised linear on the quantised operands
    torch.testing.assert_close(w.grad, (torch.ones(16, 64).t() @ fp4.quant_dequant_reference(x.detach()).view(16, 128)),
                               rtol=1e-5, atol=1e-5)


def test_quantised_weight_cache_entries_die_with_the_weight():
    import gc

    from nano_train_b200.precision.backends import _remember

    cache = {}
    w = torch.nn.Parameter(torch.randn(4, 4))
    _remember(cache, w, "quantised copy")
    _remember(cache, w, "refreshed copy")  # same weight, new version: one entry
    assert list(cache.values()) == ["refreshed copy"]
    del w
    gc.collect()
    assert cache == {}
