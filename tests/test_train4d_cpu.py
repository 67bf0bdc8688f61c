"""End-to-end 4-D runtime (examples/train_4d.py) on CPU with 4 gloo ranks.

Covers the parallel layouts of the reference's integration matrix (PP x EP
with ZeRO-2, TP x PP, EP folded into DP with ZeRO-1) and exact resume from a
checkpoint: a run interrupted after 3 steps and resumed must log the same
losses for steps 3..5 as an uninterrupted run.
"""
import os
import re
import subprocess
import sys

import pytest

from conftest import ROOT, free_port

SCRIPT = os.path.join(ROOT, "examples", "train_4d.py")
STEP_RE = re.compile(r"step=(\d+) task=([-\d.e]+) aux=([-\d.e]+) total=([-\d.e]+)")


def _run(args, world=4, timeout=300):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", f"--master-port={free_port()}", SCRIPT,
           "--batch_size", "8", "--num_samples", "64", "--seq_len", "16", "--epochs", "2", "--log_every", "1",
           "--hidden_size", "64", "--num_layers", "3", "--num_heads", "4", "--num_kv_heads", "4",
           "--intermediate_size", "128", "--moe_intermediate_size", "64", "--vocab_size", "128",
           "--q_lora_rank", "32", "--kv_lora_rank", "16", "--dist-timeout-s", "120"] + args
    env = dict(os.environ, OMP_NUM_THREADS="1", PYTHONPATH=ROOT)
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env, cwd=ROOT)
    out = p.stdout + p.stderr
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

