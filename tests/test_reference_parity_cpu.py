"""Loss parity with the reference on BASELINE config #1 (CPU, 4 gloo ranks, TP1 PP2 EP2, ZeRO-2,
2 microbatches, DeepSeek tiny with 8 experts top-2 and one shared expert, fp32, seed 0).

The expected values are the reference's own engine log lines for the same command, run on this
machine with the unmodified reference (its examples/train_4d.py over the installed copy):

    torchrun --nproc-per-node 4 examples/train_4d.py <ARGS>

step=0 task=5.572248 aux=3.019414 total=5.602442 drop=0.1001
step=1 task=5.581793 aux=3.016708 total=5.611961 drop=0.0984

Matching them needs the same initial weights (same module construction order and per-rank
seeds), the same batch order (the epoch shuffle seed drawn from the global RNG) and the same
math; the optimizer step may differ in the last bits (fused flat AdamW).
"""
import os
import re
import subprocess
import sys

from conftest import ROOT, free_port

ARGS = ("--tensor-model-parallel-size 1 --pipeline-model-parallel-size 2 --expert-model-parallel-size 2 "
        "--use-distributed-optimizer --data-parallel-sharding-strategy optim_grads --num_microbatches 2 "
        "--batch_size 4 --seq_len 64 --vocab_size 256 --hidden_size 128 --num_layers 4 --num_heads 4 "
        "--num_kv_heads 4 --moe_intermediate_size 256 --num_experts 8 --top_k 2 --n_shared_experts 1 --seed 0 "
        "--lr 1e-3 --max_steps 2 --log_every 1").split()
REFERENCE = {0: (5.572248, 3.019414, 5.602442, 0.1001), 1: (5.581793, 3.016708, 5.611961, 0.0984)}
STEP_RE = re.compile(r"step=(\d+) task=([-\d.]+) aux=([-\d.]+) total=([-\d.]+) drop=([-\d.]+)")


def test_config1_losses_match_reference():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=4", "--master-addr",
           "127.0.0.1", f"--master-port={free_port()}", os.path.join(ROOT, "examples", "train_4d.py")] + ARGS
    env = dict(os.environ, OMP_NUM_THREADS="1", PYTHONPATH=ROOT)
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    out = p.stdout + p.stderr
    assert p.returncode == 0, out[-4000:]
    got = {int(m.group(1)): tuple(float(m.group(i)) for i in range(2, 6)) for m in STEP_RE.finditer(out)}
    assert sorted(got) == [0, 1], out[-2000:]
    for step, want in REFERENCE.items():
        for g, w, tol in zip(got[step], want, (2e-6, 2e-6, 2e-6, 1e-4)):
            assert abs(g - w) <= tol, (step, got[step], want)
