"""Grouped expert GEMMs under the DeepSeek-V3 fp8 recipe (native backend): the grouped path
(e4m3-rounded operands, bf16 tensor-core GEMMs, straight-through backward) against the
per-expert loop of fp8 linears (block-scaled e4m3 GEMM forward, bf16 backward)."""
import argparse

import pytest
import torch

pytestmark = pytest.mark.gpu


def _moe(seed):
    from nano_train_b200.models.moe import LocalRoutedMoE
    from nano_train_b200.precision.mixed_precision import build_module_precision_resolver, resolve_precision_config

    args = argparse.Namespace(precision_recipe="deepseek_v3", fp8=True, fp8_backend="native", params_dtype="bf16",
                              fp8_rounding="nearest")
    res = build_module_precision_resolver(resolve_precision_config(args, torch.device("cuda")))
    torch.manual_seed(seed)
    return LocalRoutedMoE(256, 256, 8, 2, param_dtype=torch.bfloat16, param_device=torch.device("cuda"),
                          precision_resolver=res, scoring_func="softmax", n_shared_experts=1, capacity_factor=2.0)


def test_grouped_fp8_matches_expert_loop(monkeypatch):
    import nano_train_b200.models.moe as moe_mod
    from nano_train_b200.ops._ext import check_status
    from nano_train_b200.ops.grouped import grouped_fp8_rounding, grouped_kernel_ok

    a, b = _moe(0), _moe(0)
    b.load_state_dict(a.state_dict())
    x = torch.randn(2, 300, 256, device="cuda", dtype=torch.bfloat16)
    assert grouped_fp8_rounding(a.experts) == "nearest" and grouped_kernel_ok(x.view(-1, 256), a.experts)
    xa = x.clone().requires_grad_(True)
    ya = a(xa)
    ya.float().square().sum().backward()
    monkeypatch.setattr(moe_mod, "grouped_kernel_ok", lambda *args, **kw: False)
    xb = x.clone().requires_grad_(True)
    yb = b(xb)
    yb.float().square().sum().backward()
    torch.cuda.synchronize()
    check_status(0)
    rel = lambda p, q: ((p.float() - q.float()).norm() / q.float().norm()).item()  # noqa: E731
    assert rel(ya, yb) < 2e-2
    assert rel(xa.grad, xb.grad) < 3e-2
    ga, gb = a.experts[0].gate_proj.weight, b.experts[0].gate_proj.weight
    da = ga.main_grad if getattr(ga, "main_grad", None) is not None else ga.grad
    db = gb.main_grad if getattr(gb, "main_grad", None) is not None else gb.grad
    assert rel(da, db) < 3e-2


@pytest.mark.parametrize("E,N,K", [(4, 256, 256), (3, 384, 512), (5, 128, 128)])
def test_gemm_fp8_grouped_matches_fp32_on_dequantised_operands(E, N, K):
    """Grouped block-scaled e4m3 GEMM: segment g of the rows times expert g's [N, K] weights, against
    fp32 math on the dequantised operands; rows past the last segment are left untouched."""
    from nano_train_b200.ops._ext import check_status, ext
    from nano_train_b200.ops.grouped import pad_segments

    C = ext()
    torch.manual_seed(E * N + K)
    counts = torch.tensor([37, 0, 200, 129, 5][:E], device="cuda", dtype=torch.int32)
    offsets, rows = pad_segments(counts, int(counts.sum()) + 128 * E + 128)  # spare rows past the segments
    x = torch.randn(rows, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(E * N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    xq, sx = C.fp8_quantize(x, 1, False, 0)
    wq, sw = C.fp8_quantize(w, 128, False, 0)
    out = torch.full((rows, N), 7.0, device="cuda", dtype=torch.bfloat16)
    C.gemm_fp8_grouped(xq, sx, wq, sw, out, offsets)
    torch.cuda.synchronize()
    check_status(0)
    xd = C.fp8_dequantize(xq, sx, 1, torch.float32)
    wd = C.fp8_dequantize(wq, sw, 128, torch.float32)
    off = offsets.tolist()
    for g in range(E):
        a, b = off[g], off[g + 1]
        if b > a:
            ref = xd[a:b] @ wd[g * N:(g + 1) * N].t()
            rel = ((out[a:b].float() - ref).norm() / ref.norm().clamp_min(1e-12)).item()
            assert rel < 1e-2, (g, rel)
    assert bool((out[off[-1]:] == 7.0).all())  # rows past the last segment are not written


def test_moe_experts_run_native_fp8_gemms_from_a_flat_buffer(monkeypatch):
    """With the experts' weights in the flat optimizer buffer (gate | up | down per expert at a fixed
    stride) the grouped path multiplies e4m3 codes on the tensor cores (forward and input gradient),
    and agrees with the per-expert loop of fp8 linears."""
    import nano_train_b200.models.moe as moe_mod
    from nano_train_b200.ops._ext import check_status
    from nano_train_b200.optimizer import create_optimizer

    a, b = _moe(1), _moe(1)
    b.load_state_dict(a.state_dict())
    create_optimizer(a, 1e-3, 0.0)  # binds the parameters to flat buffers (and main_grad views)
    x = torch.randn(2, 300, 256, device="cuda", dtype=torch.bfloat16)
    xa = x.clone().requires_grad_(True)
    ya = a(xa)
    assert a._stack_cache._codes is not None  # the native e4m3 path ran
    ya.float().square().sum().backward()
    monkeypatch.setattr(moe_mod, "grouped_kernel_ok", lambda *args, **kw: False)
    xb = x.clone().requires_grad_(True)
    yb = b(xb)
    yb.float().square().sum().backward()
    torch.cuda.synchronize()
    check_status(0)
    rel = lambda p, q: ((p.float() - q.float()).norm() / q.float().norm()).item()  # noqa: E731
    assert rel(ya, yb) < 2e-2
    assert rel(xa.grad, xb.grad) < 6e-2  # dY and dH are e4m3 in the native input-gradient GEMMs
    ga, gb = a.experts[0].down_proj.weight, b.experts[0].down_proj.weight
    assert rel(ga.main_grad, gb.grad) < 4e-2
