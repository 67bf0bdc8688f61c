"""End-to-end 4-D runtime (examples/train_4d.py) on CPU with 4 gloo ranks.

Covers the parallel layouts of the reference's integration matrix (PP x EP
with ZeRO-2, TP x PP, EP folded into DP with ZeRO-1) and exact resume from a
checkpoint: a run interrupted after 3 steps and resumed must log the same
losses for steps 3..5 as an uninterrupted run. Recovery after a failure: a rank
killed on the host (between steps, or while the checkpoint is being written)
ends the job, and the relaunch resumes from the last complete checkpoint.
"""
import os
import re
import subprocess
import sys

import pytest

from conftest import ROOT, free_port

SCRIPT = os.path.join(ROOT, "examples", "train_4d.py")
STEP_RE = re.compile(r"step=(\d+) task=([-\d.e]+) aux=([-\d.e]+) total=([-\d.e]+)")


def _run(args, world=4, timeout=300, env_extra=None, expect_ok=True):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", f"--master-port={free_port()}", SCRIPT,
           "--batch_size", "8", "--num_samples", "64", "--seq_len", "16", "--epochs", "2", "--log_every", "1",
           "--hidden_size", "64", "--num_layers", "3", "--num_heads", "4", "--num_kv_heads", "4",
           "--intermediate_size", "128", "--moe_intermediate_size", "64", "--vocab_size", "128",
           "--q_lora_rank", "32", "--kv_lora_rank", "16", "--dist-timeout-s", "120"] + args
    env = dict(os.environ, OMP_NUM_THREADS="1", PYTHONPATH=ROOT, **(env_extra or {}))
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env, cwd=ROOT)
    out = p.stdout + p.stderr
    if not expect_ok:
        assert p.returncode != 0, out[-4000:]
        return out, {int(m.group(1)): float(m.group(4)) for m in STEP_RE.finditer(out)}
    assert p.returncode == 0, out[-4000:]
    steps = {int(m.group(1)): float(m.group(4)) for m in STEP_RE.finditer(out)}
    return out, steps


@pytest.mark.parametrize("layout", [
    ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "2", "--expert-model-parallel-size", "2",
     "--use-distributed-optimizer", "--data-parallel-sharding-strategy", "optim_grads", "--num_microbatches", "2"],
    ["--tensor-model-parallel-size", "2", "--pipeline-model-parallel-size", "2", "--expert-model-parallel-size", "1",
     "--num_microbatches", "2"],
    ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "1", "--expert-model-parallel-size", "2",
     "--expert-layout", "fold_dp", "--use-distributed-optimizer", "--data-parallel-sharding-strategy", "optim"],
], ids=["pp2_ep2_zero2", "tp2_pp2", "ep2_fold_dp_zero1"])
def test_train_4d_layouts(layout):
    out, steps = _run(layout + ["--max_steps", "3"])
    assert "Training completed" in out
    assert sorted(steps) == [0, 1, 2]
    assert all(v == v and abs(v) < 100 for v in steps.values())  # finite


@pytest.mark.parametrize("layout", [
    ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "1", "--expert-model-parallel-size", "2",
     "--use-distributed-optimizer", "--data-parallel-sharding-strategy", "optim_grads"],
    ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "2", "--expert-model-parallel-size", "2",
     "--num_microbatches", "2"],
], ids=["ep2_dp2_zero2", "pp2_ep2"])
def test_train_4d_resume_is_exact(tmp_path, layout):
    _, full = _run(layout + ["--max_steps", "6"])
    ck = str(tmp_path / "ckpt")
    _run(layout + ["--max_steps", "3", "--checkpoint-dir", ck, "--save-every", "3"])
    out, resumed = _run(layout + ["--max_steps", "6", "--checkpoint-dir", ck, "--save-every", "3"])
    assert sorted(resumed) == [3, 4, 5], out[-2000:]
    for s in (3, 4, 5):
        assert abs(resumed[s] - full[s]) < 1e-6 * max(1.0, abs(full[s])), (s, resumed[s], full[s])


def test_train_4d_recovers_from_a_killed_rank(tmp_path):
    """Run -> kill -> resume from the v2 (ZeRO-2) checkpoint files -> compare losses. The fault is made on
    the host: rank 1 leaves like a crashed process (os._exit, no teardown). (a) Between steps, after step
    3 (the checkpoint after 3 steps is complete): the relaunch logs steps 3..5 as the uninterrupted run
    did. (b) While the checkpoint after 4 steps is being written (rank 1's files are on disk, the completion
    barrier is not reached): that directory has no COMPLETE marker, is skipped, and the relaunch resumes
    from the checkpoint after 2 steps."""
    layout = ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "1",
              "--expert-model-parallel-size", "2", "--use-distributed-optimizer",
              "--data-parallel-sharding-strategy", "optim_grads"]
    _, full = _run(layout + ["--max_steps", "6"])

    ck = str(tmp_path / "between_steps")
    args = layout + ["--max_steps", "6", "--checkpoint-dir", ck, "--save-every", "3"]
    out, seen = _run(args, env_extra={"NTB_FAULT_STEP": "3", "NTB_FAULT_RANK": "1"}, expect_ok=False)
    assert "injected fault: rank 1 at step_end of step 3" in out, out[-3000:]
    assert max(seen) <= 3 and "Training completed" not in out
    _, resumed = _run(args)
    assert sorted(resumed) == [3, 4, 5]
    for s in (3, 4, 5):
        assert abs(resumed[s] - full[s]) < 1e-6 * max(1.0, abs(full[s])), (s, resumed[s], full[s])

    ck = str(tmp_path / "in_save")
    args = layout + ["--max_steps", "6", "--checkpoint-dir", ck, "--save-every", "2"]
    out, _ = _run(args, env_extra={"NTB_FAULT_STEP": "4", "NTB_FAULT_RANK": "1", "NTB_FAULT_POINT": "checkpoint_save"},
                  expect_ok=False)
    assert "injected fault: rank 1 at checkpoint_save of step 4" in out, out[-3000:]
    assert os.path.exists(os.path.join(ck, "step_00000004", "model_rank1.pt"))
    assert not os.path.exists(os.path.join(ck, "step_00000004", "COMPLETE"))
    assert os.path.exists(os.path.join(ck, "step_00000002", "COMPLETE"))
    _, resumed = _run(args)
    assert sorted(resumed) == [2, 3, 4, 5]
    for s in (2, 3, 4, 5):
        assert abs(resumed[s] - full[s]) < 1e-6 * max(1.0, abs(full[s])), (s, resumed[s], full[s])
    assert os.path.exists(os.path.join(ck, "step_00000006", "COMPLETE"))


def test_train_4d_heartbeat_ends_the_job_when_a_rank_wedges():
    """A rank that wedges between steps (host-side stall: its heartbeat stops, it sleeps) while its peers
    wait for it in the next step's collectives: with --heartbeat-timeout-s the peers end within seconds,
    naming the silent rank, long before the 120 s process-group timeout."""
    import time

    layout = ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "1",
              "--expert-model-parallel-size", "2"]
    t0 = time.time()
    out, seen = _run(layout + ["--max_steps", "6", "--heartbeat-timeout-s", "5"],
                     env_extra={"NTB_FAULT_STEP": "1", "NTB_FAULT_RANK": "2", "NTB_FAULT_MODE": "stall",
                                "NTB_FAULT_STALL_S": "90"}, expect_ok=False)
    elapsed = time.time() - t0
    assert "injected fault: rank 2 at step_end of step 1" in out, out[-3000:]
    assert "no heartbeat from ranks [2]" in out, out[-3000:]
    assert max(seen) <= 1 and elapsed < 75, (seen, elapsed)


def test_train_4d_heartbeat_clean_run_completes():
    """Ranks that finish at slightly different times record a clean end, so the heartbeat does not fail
    a completed run."""
    out, steps = _run(["--tensor-model-parallel-size", "2", "--pipeline-model-parallel-size", "2",
                       "--expert-model-parallel-size", "1", "--num_microbatches", "2", "--max_steps", "3",
                       "--heartbeat-timeout-s", "10"])
    assert "Training completed" in out and sorted(steps) == [0, 1, 2]
    assert "no heartbeat" not in out


def test_train_4d_full_4d_layout_eight_ranks():
    """BASELINE config #4's layout at toy size: TP2 x PP2 x DP2 with EP2 folded inside DP, ZeRO-2, 1F1B
    with 8 microbatches, on 8 gloo ranks."""
    out, steps = _run(["--tensor-model-parallel-size", "2", "--pipeline-model-parallel-size", "2",
                       "--expert-model-parallel-size", "2", "--expert-layout", "fold_dp", "--use-distributed-optimizer",
                       "--data-parallel-sharding-strategy", "optim_grads", "--num_microbatches", "8",
                       "--num_experts", "16", "--max_steps", "2"], world=8, timeout=600)
    assert "Training completed" in out
    assert sorted(steps) == [0, 1]
    assert all(v == v and abs(v) < 100 for v in steps.values())

