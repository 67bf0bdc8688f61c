"""Allocation-free C entry point of the RMSNorm backward (ntb_rmsnorm_bwd_bf16_noalloc).

Loads the exported C symbol from the built extension with ctypes and checks two
calls in a row against the PyTorch-bound rmsnorm_bwd of the same extension (and
an fp32 PyTorch reference). The file name sorts last so the test also runs after
every other test in the session.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from nano_train_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.ntb_rmsnorm_bwd_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    err = lib.ntb_noalloc_last_error
    err.restype = ctypes.c_char_p
    err.argtypes = []
    return fn, err


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("rows,H,with_res", [(1000, 4096, False), (257, 1024, True), (3, 4096, True)])
def test_noalloc_rmsnorm_bwd_matches_bound_entry(rows, H, with_res):
    from nano_train_b200.ops._ext import check_status, ext

    fn, err = _lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(rows + H)
    h = torch.randn(rows, H, device=dev, dtype=torch.bfloat16, generator=g)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).to(torch.bfloat16)
    dy = torch.randn(rows, H, device=dev, dtype=torch.bfloat16, generator=g)
    dres = torch.randn(rows, H, device=dev, dtype=torch.bfloat16, generator=g) if with_res else None
    rstd = torch.rsqrt(h.float().pow(2).mean(-1) + 1e-5).contiguous()

    dx_ref, dw_ref = ext().rmsnorm_bwd(dy, h, w, rstd, dres)
    # fp32 PyTorch reference of the same op
    hf = h.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    y = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * wf
    y.backward(dy.float())
    dx32 = hf.grad + (dres.float() if with_res else 0)

    stream = torch.cuda.current_stream(dev)
    for call in range(2):
        dx = torch.full((rows, H), float("nan"), device=dev, dtype=torch.bfloat16)
        dw = torch.full((H,), float("nan"), device=dev, dtype=torch.float32)
        rc = fn(_ptr(dy), _ptr(h), _ptr(w), _ptr(rstd), _ptr(dres), _ptr(dx), _ptr(dw), rows, H,
                ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, err().decode()
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(dx.float(), dx_ref.float(), rtol=2e-2, atol=2e-2, msg=f"dx call {call}")
        torch.testing.assert_close(dw, dw_ref.float(), rtol=2e-2, atol=2e-2 * max(1.0, rows ** 0.5),
                                   msg=f"dw call {call}")
        rel = ((dx.float() - dx32).norm() / dx32.norm()).item()
        assert rel < 1e-2, f"dx vs fp32 reference, call {call}: rel {rel}"
        relw = ((dw - wf.grad).norm() / wf.grad.norm()).item()
        assert relw < 1e-2, f"dw vs fp32 reference, call {call}: rel {relw}"
    check_status(0)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_noalloc_rmsnorm_bwd_rejects_oversized_hidden():
    fn, err = _lib()
    rc = fn(*([ctypes.c_void_p(0)] * 7), 16, 8192, ctypes.c_void_p(0))
    assert rc == 1
    assert b"outside" in err()
