"""Tensor-core efficiency model of the analytic report (the reference's eta_tc model,
src/utils/model_info.py:425-499): eta(M) = min(1, M / b_sat) on the eligible FLOPs, eta_scalar on the
rest, realizable = peak-equivalent cost, P_eff = peak x theory / realizable."""
import pytest
import torch

from nano_train_b200.models.transformer import TransformerModel, llama3_8b_config
from nano_train_b200.utils.model_info import FlopBreakdown, TensorCoreModel, estimate


def test_eta_and_breakdown_formulas():
    tc = TensorCoreModel(b_sat=64, eta_scalar=0.5, eligible={"linear": 0.9})
    assert tc.eta(16) == pytest.approx(0.25) and tc.eta(1000) == 1.0
    b = tc.breakdown(100.0, 16, "linear")
    assert b.tensorcore == pytest.approx(90.0) and b.eta_tc == pytest.approx(0.25)
    assert b.realizable == pytest.approx(90.0 / 0.25 + 10.0 / 0.5)
    assert b.p_effective_tflops(1000.0) == pytest.approx(1000.0 * 100.0 / b.realizable)
    c = b + tc.breakdown(100.0, 640, "linear")  # eta of a sum: weighted by eligible FLOPs
    assert c.theory == 200.0 and c.eta_tc == pytest.approx((90 * 0.25 + 90 * 1.0) / 180)
    off = TensorCoreModel(enabled=False).breakdown(50.0, 1, "linear")
    assert off.realizable == 50.0 and off.eta_tc == 1.0
    assert (FlopBreakdown(0, 0, 0) + off).theory == 50.0


def test_decode_is_tensor_core_starved_and_training_is_not():
    model = TransformerModel(llama3_8b_config(num_layers=2, param_device=torch.device("meta"), sequence_parallel=False))
    info = estimate(model, batch=1, seq_len=4096, decode_ctx=4096)
    by = {(k.mode, k.exec_model, k.target): k for k in info.kpis}
    dec = next(k for (m, _, _), k in by.items() if m == "decode")
    tr = next(k for (m, _, _), k in by.items() if m == "train")
    assert dec.eta_tc < 0.05 and dec.flops_realizable > 10 * dec.flops_theory
    assert tr.eta_tc == pytest.approx(1.0) and tr.p_effective_tflops > 0.5 * dec.p_effective_tflops
    assert all(k.flops_tensorcore <= k.flops_theory for k in info.kpis)


def test_sync_and_run_plans_commit_push_and_remote(tmp_path):
    """The development sync workflow on a throwaway repository (no network: planning and dry run)."""
    import subprocess

    from nano_train_b200.utils.sync_and_run import main, notebook_cell, plan

    repo = str(tmp_path)
    for cmd in (["git", "init", "-q"], ["git", "config", "user.email", "a@b"], ["git", "config", "user.name", "a"]):
        subprocess.run(cmd, cwd=repo, check=True)
    (tmp_path / "f.txt").write_text("x")
    steps = plan(cwd=repo, message="m", push=True, remote="me@box", remote_dir="d", command="run")
    assert steps == [["git", "add", "-A"], ["git", "commit", "-m", "m"], ["git", "push"],
                     ["ssh", "me@box", "cd d && git pull --ff-only && run"]]
    subprocess.run(["git", "add", "-A"], cwd=repo, check=True)
    subprocess.run(["git", "commit", "-qm", "init"], cwd=repo, check=True)
    assert plan(cwd=repo, push=False) == []  # clean tree, no push, no remote: nothing to do
    assert "git pull --ff-only" in notebook_cell("d", "run", "https://example/repo.git")
    assert main(["--dry-run", "--no-push", "--remote-dir", "d"]) == 0
