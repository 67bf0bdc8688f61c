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
