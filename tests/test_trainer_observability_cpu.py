"""Trainer observability: the tag families a logged step writes, the monitors' arming, the
runtime-step API a runtime-engine script drives, and the loss-spike alerts.

Behaviour follows the reference's Trainer (src/trainer.py: activation / residual hooks 579-740,
Attention/* 386-474, Tokens/* and Time/* 823-960, loss-spike alerts 808-922, histograms 1938-2070)."""
import math

import pytest
import torch

from nano_train_b200.config import Config, ModelConfig, TrainingConfig, _NoOpPrecisionResolver
from nano_train_b200.dataset import SyntheticTokenDataset, create_dataloader
from nano_train_b200.models.transformer import TransformerModel
from nano_train_b200.trainer import Trainer, _TrainTotals, _TrainWindow


class _Rec:
    def __init__(self):
        self.scalars, self.hists = {}, {}

    def add_scalar(self, tag, v, step):
        self.scalars[(tag, step)] = float(v)

    def add_histogram(self, tag, v, step):
        self.hists[(tag, step)] = v.numel()

    def flush(self):
        pass

    def close(self):
        pass


def _trainer(tmp_path, mode="standard", **train_kw):
    mcfg = ModelConfig(param_dtype=torch.float32, param_device=torch.device("cpu"),
                       precision_resolver=_NoOpPrecisionResolver(), hidden_size=32, num_layers=3,
                       num_attention_heads=4, intermediate_size=64, vocab_size=64, max_position_embeddings=64,
                       dropout=0.0)
    tk = dict(batch_size=4, micro_batch_size=2, learning_rate=1e-3, max_steps=4, warmup_steps=1, log_steps=2,
              eval_steps=100, save_steps=0, clip_grad=1.0)
    tk.update(train_kw)
    cfg = Config(model=mcfg, training=TrainingConfig(**tk), output_dir=str(tmp_path / "o"),
                 log_dir=str(tmp_path / "l"))
    cfg.monitoring.mode = mode
    cfg.monitoring.histogram_steps = 2
    cfg.monitoring.probe_steps = 0
    torch.manual_seed(0)
    ds = SyntheticTokenDataset(32, 16, 64, seed=0)
    tr = Trainer(TransformerModel(mcfg), cfg, create_dataloader(ds, 4, shuffle=False), "cpu")
    tr.writer = _Rec()
    return tr


def test_logged_steps_write_every_tag_family(tmp_path):
    tr = _trainer(tmp_path)
    tr.train()
    tags = {t for t, _ in tr.writer.scalars}
    fam = {t.split("/")[0] for t in tags}
    for f in ("Loss", "LR", "Tokens", "Time", "Throughput", "Perf", "Gradients", "Weights", "Activations",
              "Residual", "Attention", "Data", "Final"):
        assert f in fam, f
    # sentinel activation sites and every sentinel block's residual / attention readings
    assert ("Activations/ln_f/rms", 2) in tr.writer.scalars
    assert any(t.startswith("Residual/blocks.0/") for t in tags)
    assert ("Attention/block_0/attn_entropy_norm", 2) in tr.writer.scalars
    # tokens: 4 x 16 per step, all labels effective (no padding in the synthetic set)
    assert tr.writer.scalars[("Tokens/total", 4)] == 4 * 4 * 16
    assert tr.writer.scalars[("Tokens/effective_total", 4)] == 4 * 4 * 16
    wait, comp = tr.writer.scalars[("Time/data_wait_frac", 2)], tr.writer.scalars[("Time/compute_frac", 2)]
    assert 0.0 <= wait <= 1.0 and wait + comp == pytest.approx(1.0)
    # weight and gradient histograms every histogram_steps
    assert any(t.startswith("Hist/weights/") for t, _ in tr.writer.hists)
    assert any(t.startswith("Hist/gradients/") for t, _ in tr.writer.hists)
    # monitors are disarmed outside logged forwards
    assert not tr._act_watch.armed and not tr._res_watch.armed
    assert all(a is None or not a._monitor_enabled for a in tr._attn_by_block)


def test_minimal_mode_installs_no_monitors(tmp_path):
    tr = _trainer(tmp_path, mode="minimal")
    tr.train()
    assert tr._act_watch is None and tr._res_watch is None
    assert not any(t.startswith(("Activations/", "Residual/", "Attention/")) for t, _ in tr.writer.scalars)


def test_runtime_step_api_drives_a_step(tmp_path):
    """The three-call step a runtime-engine script makes (the reference's MVP example does this)."""
    tr = _trainer(tmp_path)
    batch = next(iter(tr.train_loader))
    totals, window = _TrainTotals(), _TrainWindow(start_time=0.0)
    tr.optimizer.zero_grad()
    loss, st = tr.runtime_forward_loss(batch, step=0, log_this_step=True, use_internal_autocast=True)
    loss.backward()
    gnorm = tr.runtime_post_backward_metrics(step=0, step_state=st)
    assert gnorm is not None and math.isfinite(gnorm) and gnorm > 0
    w0 = next(tr.model.parameters()).detach().clone()
    tr.runtime_apply_optimizer_step(step=0, step_applied=True)
    assert not torch.equal(w0, next(tr.model.parameters()).detach())
    totals.update(tokens=st.tokens, effective_tokens=st.effective_tokens, samples=st.samples)
    window.update(tokens=st.tokens, effective_tokens=st.effective_tokens, samples=st.samples,
                  clipped=tr._is_step_clipped(gnorm))
    ema, ratio = tr._update_loss_ema(float(loss))
    tr._log_train_step(step=0, lr_used=1e-3, loss_value=float(loss), loss_ema=ema, loss_spike_ratio=ratio,
                       tokens=st.tokens, effective_tokens=st.effective_tokens, step_seconds=0.1,
                       data_wait_seconds=0.1, totals=totals, window=window)
    assert tr.writer.scalars[("Time/data_wait_frac", 0)] == pytest.approx(0.5)
    assert window.steps == 0  # the logged step reset the window
    # a non-logged step does not compute the gradient norm (no host read)
    tr.optimizer.zero_grad()
    loss, st = tr.runtime_forward_loss(batch, step=1, log_this_step=False)
    loss.backward()
    assert tr.runtime_post_backward_metrics(step=1, step_state=st) is None


def test_loss_spike_alerts(tmp_path, caplog):
    tr = _trainer(tmp_path)
    tr._update_loss_ema(1.0)
    with caplog.at_level("WARNING"):
        _, r = tr._update_loss_ema(tr.config.alerts.loss_spike_warn * 1.5)
    assert r > tr.config.alerts.loss_spike_warn and "loss spike" in caplog.text
    with pytest.raises(RuntimeError, match="stop threshold"):
        tr._update_loss_ema(1e6)


def test_fixed_probe_batch_change_is_detected(tmp_path):
    """The fixed probe batch is hashed when captured; a later change of its contents raises instead of
    silently evaluating another batch (reference: src/trainer.py:524-531)."""
    tr = _trainer(tmp_path)
    tr._run_fixed_probe(step=1)
    assert ("Probe/loss", 1) in tr.writer.scalars
    ids, _ = tr._probe
    ids[0, 0] = (ids[0, 0] + 1) % 64
    with pytest.raises(RuntimeError, match="hash mismatch"):
        tr._run_fixed_probe(step=2)
