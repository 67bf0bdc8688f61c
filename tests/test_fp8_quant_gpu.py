"""e4m3 quantisers of the DeepSeek-V3 recipe (1x128 tiles, 128x128 blocks) against a CPU statement of
the same math: scale = amax / 448 per tile / block, codes = e4m3(x / scale) with round-to-nearest-even
(PyTorch's float8_e4m3fn conversion on the CPU), and the stochastic-rounding contract (one of the two
grid neighbours, unbiased in expectation, deterministic per seed)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _oracle(x: torch.Tensor, block_rows: int):
    """CPU fp32 statement: per-tile / per-block scales and RNE e4m3 codes."""
    xf = x.float().cpu()
    R, C = xf.shape
    br = block_rows
    nb = (R + br - 1) // br
    pad = torch.zeros(nb * br, C)
    pad[:R] = xf
    blocks = pad.view(nb, br, C // 128, 128).abs().amax(dim=(1, 3))  # [nb, C/128]
    s = torch.where(blocks > 0, blocks / 448.0, torch.ones_like(blocks))
    sfull = s.repeat_interleave(br, 0)[:R].repeat_interleave(128, 1)
    y = (xf / sfull).clamp(-448, 448)
    codes = y.to(torch.float8_e4m3fn).view(torch.uint8)
    return codes, s


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("block_rows", [1, 128])
@pytest.mark.parametrize("R,C", [(300, 512), (128, 128), (1000, 2048), (7, 256)])
def test_nearest_codes_and_scales_match_cpu_statement(dtype, block_rows, R, C):
    from nano_train_b200.ops._ext import ext

    torch.manual_seed(R + C + block_rows)
    x = (torch.randn(R, C) * torch.logspace(-3, 2, C)[None]).to(dtype).cuda()
    x[0, :128] = 0  # an all-zero tile / block row gets scale 1
    q, s = ext().fp8_quantize(x, block_rows, False, 0)
    codes, s_ref = _oracle(x, block_rows)
    torch.testing.assert_close(s.cpu(), s_ref, rtol=0, atol=0)
    assert torch.equal(q.cpu(), codes)
    dq = ext().fp8_dequantize(q, s, block_rows, torch.float32)
    ref = codes.view(torch.float8_e4m3fn).float() * s_ref.repeat_interleave(block_rows, 0)[:R].repeat_interleave(128, 1)
    torch.testing.assert_close(dq.cpu(), ref, rtol=0, atol=0)
    qd = ext().fp8_quant_dequant(x, block_rows, False, 0)
    torch.testing.assert_close(qd.float().cpu(), ref.to(dtype).float(), rtol=0, atol=0)


def test_stochastic_rounding_contract():
    from nano_train_b200.ops._ext import ext

    torch.manual_seed(3)
    x = torch.randn(64, 256, device="cuda")
    q0, s0 = ext().fp8_quantize(x, 1, False, 0)
    grid = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    grid = torch.sort(grid[torch.isfinite(grid)]).values.cuda()
    y = (x / s0.repeat_interleave(128, 1)).clamp(-448, 448)
    lo = grid[torch.searchsorted(grid, y.contiguous(), right=True) - 1]
    hi = grid[torch.clamp(torch.searchsorted(grid, y.contiguous(), right=False), max=grid.numel() - 1)]
    acc = torch.zeros_like(x)
    n = 64
    for seed in range(n):
        q, s = ext().fp8_quantize(x, 1, True, seed)
        assert torch.equal(s, s0)  # scales do not depend on the rounding
        v = q.view(torch.float8_e4m3fn).float()
        assert bool(((v == lo) | (v == hi)).all())  # one of the two neighbours on the grid
        acc += v
        if seed == 0:
            q_again, _ = ext().fp8_quantize(x, 1, True, seed)
            assert torch.equal(q, q_again)  # deterministic per seed
    mean = acc / n
    gap = (hi - lo).clamp_min(1e-12)
    # unbiased: the mean of n draws is within a few standard errors of y (per-element, in units of the gap)
    err = ((mean - y) / gap).abs()
    assert float(err.mean()) < 0.05 and float(err.max()) < 0.6


@pytest.mark.parametrize("E,I,H", [(4, 256, 128), (3, 128, 384)])
def test_strided_expert_stack_equals_quantising_the_concatenation(E, I, H):
    """The rounded expert stacks read in place from a flat buffer (gate|up|down per expert at a
    fixed stride) equal rounding the concatenated stacks."""
    from nano_train_b200.ops._ext import ext

    torch.manual_seed(E * I + H)
    stride = 3 * I * H + 1024  # experts padded apart in the buffer
    flat = torch.randn(E * stride, device="cuda", dtype=torch.bfloat16)
    gate = [flat[e * stride: e * stride + I * H].view(I, H) for e in range(E)]
    up = [flat[e * stride + I * H: e * stride + 2 * I * H].view(I, H) for e in range(E)]
    down = [flat[e * stride + 2 * I * H: e * stride + 3 * I * H].view(H, I) for e in range(E)]
    w1 = ext().fp8_quant_dequant_strided(gate[0], E, 2 * I, H, stride)
    w2 = ext().fp8_quant_dequant_strided(down[0], E, H, I, stride)
    ref1 = ext().fp8_quant_dequant(torch.cat([torch.cat([g, u]) for g, u in zip(gate, up)]), 128, False, 0)
    ref2 = ext().fp8_quant_dequant(torch.cat(down), 128, False, 0)
    assert torch.equal(w1, ref1) and torch.equal(w2, ref2)
