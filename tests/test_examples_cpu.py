"""The utility examples run on CPU from a clean working directory: the analytic reports (the
DeepSeek-V3 preset on the meta device, the GPT-2 model report with its sweep), the tiny DeepSeek preset
training on synthetic tokens, device info with the launch command it suggests, the logging demo and the
cross-entropy demo (reference: examples/deepseek.py, model_info.py, device_info.py, logging_demo.py,
loss_demo.py)."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT


def _run(args, cwd, timeout=600):
    env = dict(os.environ, OMP_NUM_THREADS="2", PYTHONPATH=ROOT)
    p = subprocess.run([sys.executable] + args, capture_output=True, text=True, timeout=timeout, cwd=str(cwd),
                       env=env)
    out = p.stdout + p.stderr
    assert p.returncode == 0, out[-3000:]
    return out


def test_deepseek_v3_meta_report(tmp_path):
    out = _run([os.path.join(ROOT, "examples", "deepseek.py"), "--report", str(tmp_path / "r.md")], tmp_path)
    assert "report:" in out
    text = (tmp_path / "r.md").read_text()
    assert text.startswith("# Model report") and "Architecture" in text
    assert (tmp_path / "r.json").exists() and (tmp_path / "r_roofline.svg").exists()


def test_deepseek_tiny_preset_trains(tmp_path):
    out = _run([os.path.join(ROOT, "examples", "deepseek.py"), "--model-preset", "tiny", "--no-meta-init",
                "--steps", "3", "--seq_len", "32"], tmp_path)
    assert "step 0 loss" in out


def test_model_info_report_and_sweep(tmp_path):
    out = _run([os.path.join(ROOT, "examples", "model_info.py"), "--model", "gpt2_125m", "--seq_len", "256",
                "--batch", "2", "--out", str(tmp_path / "m.md")], tmp_path)
    assert "decode batch" in out
    assert (tmp_path / "m.md").read_text().startswith("# Model report")
    assert (tmp_path / "m_decode_sweep.svg").exists()


@pytest.mark.parametrize("script,expect", [
    ("device_info.py", "examples/launch.py"),
    ("logging_demo.py", "info message"),
    ("loss_demo.py", "tensor("),
])
def test_small_demos(tmp_path, script, expect):
    out = _run([os.path.join(ROOT, "examples", script)], tmp_path)
    assert expect in out
