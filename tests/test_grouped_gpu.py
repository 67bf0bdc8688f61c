"""Grouped (mixture-of-experts) tcgen05 GEMM and the grouped SwiGLU expert MLP vs fp32 PyTorch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _segments(counts, dev):
    from nano_train_b200.ops.grouped import pad_segments

    c = torch.tensor(counts, device=dev)
    off, rows = pad_segments(c)
    return c, off, rows


@pytest.mark.parametrize("counts,H,N", [([130, 0, 256, 5], 256, 384), ([1, 2, 3], 512, 128), ([300], 128, 512)])
def test_grouped_gemm_three_forms(counts, H, N):
    from nano_train_b200.ops._ext import check_status, ext

    dev = torch.device("cuda", 0)
    torch.manual_seed(len(counts) * 10 + H)
    E = len(counts)
    c, off, rows = _segments(counts, dev)
    offs = off.tolist()
    x = torch.zeros(rows, H, device=dev, dtype=torch.bfloat16)
    for e in range(E):
        x[offs[e]:offs[e] + counts[e]] = torch.randn(counts[e], H, device=dev, dtype=torch.bfloat16)
    w = torch.randn(E * N, H, device=dev, dtype=torch.bfloat16) * 0.1
    # mode 1 forward: y = x_e W_e^T
    y = torch.empty(rows, N, device=dev, dtype=torch.bfloat16)
    ext().gemm_grouped_bf16(x, w, y, off, 1)
    # mode 1 dgrad form: dx = dy_e W_e (W_e stored [N, H] -> B is [K=N, N=H])
    dy = torch.zeros(rows, N, device=dev, dtype=torch.bfloat16)
    for e in range(E):
        dy[offs[e]:offs[e] + counts[e]] = torch.randn(counts[e], N, device=dev, dtype=torch.bfloat16)
    dx = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
    ext().gemm_grouped_bf16(dy, w, dx, off, 1, b_mn=True)
    # mode 2 weight gradient, accumulating: dW_e += dy_e^T x_e
    dw = torch.ones(E * N, H, device=dev, dtype=torch.float32)
    ext().gemm_grouped_bf16(dy, x, dw, off, 2, b_mn=True, accumulate=True)
    torch.cuda.synchronize()
    check_status(0)
    for e in range(E):
        s = slice(offs[e], offs[e] + counts[e])
        we = w[e * N:(e + 1) * N].float()
        if counts[e]:
            assert _rel(y[s], x[s].float() @ we.t()) < 1e-2, ("y", e)
            assert _rel(dx[s], dy[s].float() @ we) < 1e-2, ("dx", e)
        ref_dw = 1.0 + dy[s].float().t() @ x[s].float()
        assert _rel(dw[e * N:(e + 1) * N], ref_dw) < 1e-2, ("dw", e)
    # padded rows of the outputs are zero (zero input rows)
    for e in range(E):
        pad = slice(offs[e] + counts[e], offs[e + 1])
        assert float(y[pad].abs().sum()) == 0.0


@pytest.mark.parametrize("grad_mode", ["grad", "flat_main_grad", "separate_main_grad"])
def test_grouped_swiglu_experts_matches_loop(grad_mode):
    """.grad outputs; fp32 main_grad in a flat buffer (accumulated by the weight-gradient GEMM in place,
    one launch per matrix); fp32 main_grad tensors at unrelated addresses (one multi-tensor add)."""
    from nano_train_b200.models.moe import ExpertMLP
    from nano_train_b200.ops.grouped import _StackCache, _flat_main_grads, grouped_swiglu_experts
    from nano_train_b200.parallel.flat_optimizer import FlatParamBuffer

    dev = torch.device("cuda", 0)
    torch.manual_seed(3)
    E, H, I = 5, 256, 192
    experts = torch.nn.ModuleList([ExpertMLP(H, I, param_dtype=torch.bfloat16, param_device=dev) for _ in range(E)])
    plist = [p for e in experts for p in (e.gate_proj.weight, e.up_proj.weight, e.down_proj.weight)]
    if grad_mode == "flat_main_grad":
        buf = FlatParamBuffer(plist)
        assert _flat_main_grads(plist, E, I, H) is not None
        buf.grad_data.fill_(0.25)  # accumulation must add to what is there
    elif grad_mode == "separate_main_grad":
        for p in plist:
            p.main_grad = torch.full(p.shape, 0.25, device=dev, dtype=torch.float32)
        assert _flat_main_grads(plist, E, I, H) is None
    counts = torch.tensor([37, 0, 129, 64, 3], device=dev)
    x = torch.randn(int(counts.sum()), H, device=dev, dtype=torch.bfloat16, requires_grad=True)
    y = grouped_swiglu_experts(x, counts, experts, _StackCache())
    gy = torch.randn_like(y)
    y.backward(gy)
    # fp32 reference: per-expert loop
    xr = x.detach().float().requires_grad_(True)
    outs, off = [], 0
    ref_params = []
    for e, n in enumerate(counts.tolist()):
        g = experts[e].gate_proj.weight.detach().float().requires_grad_(True)
        u = experts[e].up_proj.weight.detach().float().requires_grad_(True)
        d = experts[e].down_proj.weight.detach().float().requires_grad_(True)
        ref_params.append((g, u, d))
        xs = xr[off:off + n]
        outs.append((torch.nn.functional.silu(xs @ g.t()) * (xs @ u.t())) @ d.t())
        off += n
    yr = torch.cat(outs)
    yr.backward(gy.float())
    assert _rel(y, yr) < 2e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    for e in range(E):
        for p, r in zip((experts[e].gate_proj.weight, experts[e].up_proj.weight, experts[e].down_proj.weight),
                        ref_params[e]):
            if grad_mode == "grad":
                if counts[e] == 0:
                    continue
                assert _rel(p.grad, r.grad) < 3e-2, e
            else:
                assert p.grad is None
                got = p.main_grad - 0.25
                if counts[e] == 0:
                    assert got.abs().max().item() == 0.0, e
                else:
                    assert _rel(got, r.grad) < 3e-2, e
