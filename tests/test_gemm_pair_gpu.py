"""The CTA-pair (cta_group::2, 256 x 256 tiles on two SMs) bf16 GEMM against fp32 PyTorch.

The tile shape is chosen once per process, so the checks run in a child process with
NTB_GEMM_2SM=1 (pair tiles for every wide tile, short K included); every operand major, ragged
M / N / K, fp32 accumulation into C, K slices and a publishing launch are covered."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

_CHILD = textwrap.dedent(r"""
    import torch
    from nano_train_b200.ops._ext import check_status, ext

    C = ext()

    def rel(a, b):
        return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))

    errs = []
    torch.manual_seed(0)
    for (M, N, K) in [(256, 256, 64), (512, 768, 320), (1000, 520, 2056), (4096, 4096, 4096), (304, 136, 200)]:
        for a_mn in (False, True):
            for b_mn in (False, True):
                A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
                B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
                a = A.t().contiguous() if a_mn else A
                b = B.t().contiguous() if b_mn else B
                out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                C.gemm_bf16(a, b, out, None, a_mn, b_mn, False, 1.0)
                errs.append((f"bf16 {M}x{N}x{K} a_mn={a_mn} b_mn={b_mn}", rel(out, A.float() @ B.float().t()), 1e-2))
    # weight-gradient form: fp32 C accumulated (K slices where the picker splits)
    for (M, N, K) in [(768, 4096, 4096), (4096, 512, 4096), (1000, 520, 2056)]:
        dy = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
        out = torch.randn(M, N, device="cuda", dtype=torch.float32)
        ref = out + dy.float().t() @ x.float()
        C.gemm_bf16(dy, x, out, None, True, True, True, 1.0)
        errs.append((f"wgrad {M}x{N}x{K}", rel(out, ref), 1e-5))
    # bias + alpha
    A = torch.randn(384, 192, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(640, 192, device="cuda", dtype=torch.bfloat16)
    bias = torch.randn(640, device="cuda", dtype=torch.bfloat16)
    out = torch.randn(384, 640, device="cuda", dtype=torch.float32)
    ref = out + 0.5 * (A.float() @ B.float().t()) + bias.float()
    C.gemm_bf16(A, B, out, bias, False, False, True, 0.5)
    errs.append(("bias alpha accumulate", rel(out, ref), 1e-5))
    # publishing launch: the last CTA writes the epoch into the flag
    flag = torch.zeros(1, device="cuda", dtype=torch.int64)
    ctr = torch.zeros(1, device="cuda", dtype=torch.int32)
    A = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16)
    W = torch.randn(512, 2048, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(1024, 2048, device="cuda", dtype=torch.bfloat16)
    C.gemm_bf16_publish(A, W, out, True, [flag.data_ptr()], 7, ctr)
    torch.cuda.synchronize()
    errs.append(("publish", rel(out, A.float() @ W.float()), 1e-2))
    assert int(flag.item()) == 7 and int(ctr.item()) == 0, (flag.item(), ctr.item())
    check_status(0)
    bad = [(n, e, t) for n, e, t in errs if not e < t]
    for n, e, t in errs:
        print(n, e)
    assert not bad, bad
    print("PAIR_OK")
""")


def test_pair_gemm_matches_fp32():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NTB_GEMM_2SM="1", PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", _CHILD], env=env, cwd=root, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "PAIR_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
