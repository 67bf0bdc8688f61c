"""Fused router kernel vs the PyTorch router (same module, NTB_ROUTER_KERNEL=0), fp32 math reference."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(router, x, R, aux_w, kernel: bool):
    os.environ["NTB_ROUTER_KERNEL"] = "1" if kernel else "0"
    router.zero_grad(set_to_none=True)
    ro = router(x)
    # weight of (token, expert) times a per-(token, expert) coefficient: independent of the order in
    # which tied experts are returned
    loss = (ro.topk_weights.float() * R.gather(1, ro.topk_indices)).sum() + aux_w * ro.aux_loss.float()
    loss.backward()
    os.environ.pop("NTB_ROUTER_KERNEL")
    return ro, router.router.weight.grad.detach().clone()


@pytest.mark.parametrize("dtype,scoring,E,K,ng,tg,norm,scale", [
    (torch.float32, "softmax", 64, 6, 1, 1, True, 1.0),
    (torch.float32, "sigmoid", 64, 6, 8, 3, True, 2.5),
    (torch.float32, "sigmoid", 16, 2, 1, 1, False, 1.0),
    (torch.float32, "softmax", 160, 8, 8, 4, True, 16.0),
    (torch.bfloat16, "softmax", 64, 6, 1, 1, True, 1.0),
    (torch.bfloat16, "sigmoid", 256, 8, 8, 4, True, 2.5),
])
def test_router_kernel_matches_torch(dtype, scoring, E, K, ng, tg, norm, scale):
    from nano_train_b200.models.moe import TopKRouter
    from nano_train_b200.ops._ext import check_status

    torch.manual_seed(E + K)
    dev = torch.device("cuda", 0)
    H, T = 128, 1000
    router = TopKRouter(H, E, K, param_dtype=dtype, param_device=dev, scoring_func=scoring, n_group=ng,
                        topk_group=tg, norm_topk_prob=norm, routed_scaling_factor=scale)
    x = torch.randn(T, H, device=dev, dtype=dtype)
    R = torch.randn(T, E, device=dev)
    ro_t, g_t = _run(router, x, R, 0.7, kernel=False)
    ro_k, g_k = _run(router, x, R, 0.7, kernel=True)
    check_status(0)
    # weights come out sorted by score; compare per token as sets (ties may swap in bf16)
    wk, wt = ro_k.topk_weights.float(), ro_t.topk_weights.float()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(wk.sort(-1).values, wt.sort(-1).values, rtol=tol, atol=tol)
    if dtype == torch.float32:
        assert torch.equal(ro_k.topk_indices.sort(-1).values, ro_t.topk_indices.sort(-1).values)
    else:
        same = (ro_k.topk_indices.sort(-1).values == ro_t.topk_indices.sort(-1).values).all(-1).float().mean()
        assert same > 0.97
    assert abs(float(ro_k.aux_loss.detach()) - float(ro_t.aux_loss.detach())) <= 2e-2 * abs(float(ro_t.aux_loss.detach())) + 1e-6
    rel = ((g_k.float() - g_t.float()).norm() / g_t.float().norm()).item()
    assert rel < (1e-3 if dtype == torch.float32 else 5e-2), rel
