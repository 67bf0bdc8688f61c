"""Single-process Trainer for the MVP path (reference: src/trainer.py:119-2070).

``Trainer(model, config, train_loader, device, val_loader=None).train()`` trains with this
framework's pieces: the flat-buffer fused AdamW of ``create_optimizer`` (gradient clipping at
``training.clip_grad`` is a device-side scale inside the update), ``CosineAnnealingScheduler``,
gradient accumulation over ``training.micro_batch_size`` slices, and the loss through
``model.forward_loss`` when the model has it (fused cross-entropy) or ``CrossEntropyLoss``.

Structure. One step is three calls, which ``train()`` makes and which a runtime-engine script
(the reference's MVP example among them) can make itself:

* ``runtime_forward_loss(batch, step=, log_this_step=, use_internal_autocast=)`` -> (loss,
  step state): moves the batch, arms the monitors when the step is logged, runs the forward;
* ``runtime_post_backward_metrics(step=, step_state=)`` -> pre-clip gradient norm (or None),
  after the caller's backward: gradient / data-health scalars and the attention, activation and
  residual readings of a logged step;
* ``runtime_apply_optimizer_step(step=, step_applied=)``: optimizer step (unless a loss-scaling
  controller skipped it), scheduler, refresh of persistent low-bit weight copies.

Monitors never synchronise with the host inside the forward: activation (norm outputs) and
residual (block outputs) forward hooks are armed only on logged steps and leave their statistics
(RMS, max |x|, outlier fraction, residual growth) as device scalars, read in one transfer when the
step is logged. Logged tag families: Loss/*, LR, Tokens/*, Time/* (step, data wait, compute and
data-wait fractions), Throughput/*, Perf/* (achieved TFLOP/s, MFU), Gradients/*, Weights/*,
Activations/*, Residual/*, Attention/block_i/*, Data/*, Memory/*, GPU/*, Probe/*, Eval/*,
Checkpoint/*, Hist/* (weight and gradient histograms every ``monitoring.histogram_steps``).
Alerts follow ``AlertThresholdsConfig``: loss spikes against the loss EMA (warn / stop) on every
step whose loss is known on the host, gradient norm and clip coefficient bounds, activation and
residual bounds, attention logits and entropy, data-wait fraction, reserved-memory fraction, and
fail-fast on non-finite loss, gradient norm or optimizer state.

Scalars go to TensorBoard when it is importable, else to ``<log_dir>/<run_name>/metrics.jsonl``.
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn

from .config import Config, config_to_serializable_dict
from .distributed.failure import NonFiniteError
from .logging import get_logger
from .losses import CrossEntropyLoss
from .monitoring import (achieved_tflops, candidate_sentinel_param_names, clip_coef, eval_artifact_hash,
                         global_update_ratio, mfu, resolve_sentinel_blocks, update_ratio)
from .optimizer import create_optimizer
from .scheduler import CosineAnnealingScheduler

logger = get_logger(__name__)


# ----------------------------------------------------------------------------- counters
@dataclass
class _TrainTotals:
    """Totals since the start of training."""

    tokens: int = 0
    effective_tokens: int = 0
    samples: int = 0

    def update(self, *, tokens: int, effective_tokens: int, samples: int) -> None:
        self.tokens += int(tokens)
        self.effective_tokens += int(effective_tokens)
        self.samples += int(samples)


@dataclass
class _TrainWindow:
    """Counters since the last logged step (throughput and clip rate are window rates)."""

    start_time: float
    tokens: int = 0
    effective_tokens: int = 0
    samples: int = 0
    steps: int = 0
    clipped_steps: int = 0

    def update(self, *, tokens: int, effective_tokens: int, samples: int, clipped: bool) -> None:
        self.tokens += int(tokens)
        self.effective_tokens += int(effective_tokens)
        self.samples += int(samples)
        self.steps += 1
        self.clipped_steps += int(bool(clipped))

    def reset(self, *, start_time: float) -> None:
        self.start_time = float(start_time)
        self.tokens = self.effective_tokens = self.samples = self.steps = self.clipped_steps = 0

    def clip_rate(self) -> float:
        return self.clipped_steps / self.steps if self.steps else 0.0

    def elapsed_seconds(self, *, now: float) -> float:
        return max(1e-9, float(now) - self.start_time)


@dataclass
class _RuntimeStepState:
    """What the forward of a step leaves for its post-backward metrics."""

    labels_used: torch.Tensor
    tokens: int
    samples: int
    hist_this_step: bool
    blocks_to_monitor: set = field(default_factory=set)
    log_this_step: bool = False
    _effective: Optional[torch.Tensor] = None  # device count of non-ignored labels
    _effective_host: Optional[int] = None

    @property
    def effective_tokens(self) -> int:
        """Non-ignored label count (read from the device on first use)."""
        if self._effective_host is None:
            self._effective_host = int(self._effective) if self._effective is not None else self.tokens
        return self._effective_host


# ----------------------------------------------------------------------------- monitors
class _StatWatch:
    """Forward hooks on named modules that, while armed, record device-side statistics of the
    module output (and for ``residual`` watches, of its growth over the input)."""

    OUTLIER_SIGMAS = 6.0

    def __init__(self, sites: dict[str, nn.Module], *, residual: bool, model: Optional[nn.Module] = None,
                 block_ids: Optional[dict[int, str]] = None):
        """Forward hooks on ``sites``; or, for a residual watch on a model with block observers,
        one observer recording the blocks in ``block_ids`` (index -> site name)."""
        self.residual = residual
        self.armed = False
        self.pending: dict[str, torch.Tensor] = {}
        self.handles = [m.register_forward_hook(self._hook(name)) for name, m in sites.items()]
        if model is not None and block_ids:
            def observer(i, x, y):
                if self.armed and i in block_ids:
                    self.record(block_ids[i], x, y)
            self.handles.append(model.register_block_observer(observer))

    def _hook(self, name: str):
        def hook(_module, inputs, output):
            if self.armed:
                x = inputs[0] if inputs and torch.is_tensor(inputs[0]) else None
                self.record(name, x, output[0] if isinstance(output, (tuple, list)) else output)
        return hook

    def record(self, name: str, x: Optional[torch.Tensor], y) -> None:
        if not torch.is_tensor(y) or y.numel() == 0:
            return
        with torch.no_grad():
            yf = y.detach().float()
            rms = yf.pow(2).mean().sqrt()
            stats = [rms, yf.abs().amax(), (yf.abs() > self.OUTLIER_SIGMAS * rms).float().mean()]
            if self.residual:
                stats.append(rms / x.detach().float().pow(2).mean().sqrt().clamp_min(1e-12)
                             if x is not None else torch.ones_like(rms))
            self.pending[name] = torch.stack(stats)

    def collect(self) -> dict[str, list[float]]:
        """Every recorded site's statistics with one device-to-host transfer; clears them."""
        if not self.pending:
            return {}
        names = list(self.pending)
        vals = torch.stack([self.pending[n] for n in names]).tolist()
        self.pending.clear()
        return dict(zip(names, vals))

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []


class _JsonlWriter:
    def __init__(self, path: str):
        os.makedirs(os.path.dirname(path), exist_ok=True)
        self._f = open(path, "a", encoding="utf-8")

    def add_scalar(self, tag: str, value: float, step: int) -> None:
        self._f.write(json.dumps({"tag": tag, "value": float(value), "step": int(step)}) + "\n")

    def add_histogram(self, tag: str, values, step: int) -> None:
        v = values.detach().float().flatten()
        q = torch.quantile(v, torch.tensor([0.0, 0.25, 0.5, 0.75, 1.0])) if v.numel() else torch.zeros(5)
        for name, x in zip(("min", "p25", "p50", "p75", "max"), q.tolist()):
            self.add_scalar(f"{tag}/{name}", x, step)

    def flush(self) -> None:
        self._f.flush()

    def close(self) -> None:
        self._f.close()


def _make_writer(log_dir: str, run_name: str, config: Config):
    path = os.path.join(log_dir, run_name)
    try:
        from torch.utils.tensorboard import SummaryWriter

        return SummaryWriter(path, max_queue=config.monitoring.tensorboard_max_queue,
                             flush_secs=config.monitoring.tensorboard_flush_secs)
    except Exception:  # tensorboard not installed
        return _JsonlWriter(os.path.join(path, "metrics.jsonl"))


class _NoProgress:
    def update(self, *a, **k) -> None:
        pass


# ----------------------------------------------------------------------------- trainer
class Trainer:
    def __init__(self, model, config: Config, train_loader, device, val_loader=None, precision_controller=None):
        """``precision_controller`` (a ``MixedPrecisionController``, optional): forward passes run in its
        autocast context, backward passes through its loss scaling, and a step whose unscaled gradients
        are not finite on some rank is skipped (the scale backs off), as the reference's scripts do."""
        self.precision_controller = precision_controller
        # modules keeping persistent low-bit weight copies refresh them after every applied step
        self._persistent_lowbit = [m for m in model.modules()
                                   if callable(getattr(m, "_persistent_mode", None)) and m._persistent_mode() != "off"]
        self.device = torch.device(device)
        self.model = model.to(self.device)
        self.config = config
        self.train_loader = train_loader
        self.val_loader = val_loader
        tc, mc = config.training, config.monitoring
        self.monitoring_mode = mc.mode
        self.log_steps = max(1, int(tc.log_steps))
        self.histogram_steps = max(1, int(mc.histogram_steps or 0) or 10 ** 9)
        self.micro_batch_size = max(1, int(tc.micro_batch_size))
        self.optimizer = create_optimizer(model, tc.learning_rate, tc.weight_decay,
                                          max_grad_norm=tc.clip_grad if tc.clip_grad and tc.clip_grad > 0 else None)
        self.scheduler = CosineAnnealingScheduler(self.optimizer, tc.warmup_steps, tc.max_steps, min_lr=0.0)
        self.criterion = CrossEntropyLoss(ignore_index=-100)
        os.makedirs(config.output_dir, exist_ok=True)
        os.makedirs(config.log_dir, exist_ok=True)
        self.writer = _make_writer(config.log_dir, config.run_name, config)
        self.global_step = 0
        self._loss_ema: Optional[float] = None
        self.num_params = sum(p.numel() for p in model.parameters())
        blocks = getattr(model, "blocks", None)
        nl = int(getattr(getattr(model, "config", None), "num_layers", 0) or (len(blocks) if blocks is not None else 0))
        self._sentinel_blocks = resolve_sentinel_blocks(nl, mc.sentinel_blocks)
        named = dict(model.named_parameters())
        self._sentinels = {n: named[n] for n in sorted(candidate_sentinel_param_names(
            sentinel_blocks=self._sentinel_blocks)) if n in named}
        self._prev_sentinel: dict[str, torch.Tensor] = {}
        self._attn_by_block = [getattr(b, "attention", None) if hasattr(getattr(b, "attention", None),
                                                                        "set_monitoring") else None
                               for b in (blocks if blocks is not None else [])]
        self._act_watch, self._res_watch = self._install_watches(blocks)
        self._probe = self._probe_hash = self._probe_prev_logp = None
        self._pending_step: Optional[dict] = None
        self._nvml = self._nvml_handle = None
        if self.device.type == "cuda":
            try:
                import pynvml

                pynvml.nvmlInit()
                self._nvml = pynvml
                self._nvml_handle = pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)
            except Exception:
                self._nvml = None
        self._peak_tflops = mc.peak_tflops or (1649.0 if self.device.type == "cuda" else 0.0)

    # ------------------------------------------------------------------ monitor set-up
    def _install_watches(self, blocks):
        if self.monitoring_mode == "minimal":
            return None, None
        sites = {}
        choice = self.config.monitoring.activation_sites
        if choice == "sentinel" and blocks is not None:
            for i in self._sentinel_blocks:
                if 0 <= i < len(blocks) and hasattr(blocks[i], "attn_norm"):
                    sites[f"blocks.{i}.attn_norm"] = blocks[i].attn_norm
            if hasattr(self.model, "ln_f"):
                sites["ln_f"] = self.model.ln_f
        elif choice == "all_lns":
            from .layers import LayerNorm, RMSNorm

            sites = {n: m for n, m in self.model.named_modules() if isinstance(m, (LayerNorm, RMSNorm))}
        act = _StatWatch(sites, residual=False) if sites else None
        res = None
        if blocks is not None and len(blocks):
            idx = range(len(blocks)) if self.monitoring_mode == "debug" else self._sentinel_blocks
            ids = {i: f"blocks.{i}" for i in idx if 0 <= i < len(blocks)}
            if ids and callable(getattr(self.model, "register_block_observer", None)):
                res = _StatWatch({}, residual=True, model=self.model, block_ids=ids)
            elif ids:
                res = _StatWatch({n: blocks[i] for i, n in ids.items()}, residual=True)
        return act, res

    def _blocks_to_monitor(self, log_this_step: bool) -> set:
        if not log_this_step or self.monitoring_mode == "minimal":
            return set()
        idx = range(len(self._attn_by_block)) if self.monitoring_mode == "debug" else self._sentinel_blocks
        return {i for i in idx if 0 <= i < len(self._attn_by_block) and self._attn_by_block[i] is not None}

    def _arm(self, log_this_step: bool, blocks: set) -> None:
        """Arm the monitors for one forward; disarming keeps the readings already taken (the
        attention modules' ``_monitor_stats``) for the post-backward logging."""
        for i, attn in enumerate(self._attn_by_block):
            if attn is None:
                continue
            if log_this_step:
                attn.set_monitoring(i in blocks, tau=float(self.config.monitoring.attn_tau))
            else:
                attn._monitor_enabled = False
        for w in (self._act_watch, self._res_watch):
            if w is not None:
                w.armed = log_this_step

    # ------------------------------------------------------------------ loss
    def _loss(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        if hasattr(self.model, "forward_loss"):
            return self.model.forward_loss(input_ids, labels)
        logits = self.model(input_ids)
        return self.criterion(logits, labels)

    def _autocast(self, use_internal_autocast: bool):
        if use_internal_autocast and self.precision_controller is not None:
            return self.precision_controller.autocast_context()
        return torch.autograd.graph.saved_tensors_hooks(lambda x: x, lambda x: x)  # no-op context

    # ------------------------------------------------------------------ runtime step API
    def runtime_forward_loss(self, batch, *, step: int, log_this_step: bool,
                             use_internal_autocast: bool = True) -> tuple[torch.Tensor, _RuntimeStepState]:
        """Forward and loss of one batch (no backward); arms the monitors on a logged step."""
        ids = batch["input_ids"].to(self.device, non_blocking=True)
        lab = batch["labels"].to(self.device, non_blocking=True)
        blocks = self._blocks_to_monitor(log_this_step)
        self._arm(log_this_step, blocks)
        try:
            with self._autocast(use_internal_autocast):
                loss = self._loss(ids, lab)
        finally:
            self._arm(False, set())
        used = lab  # labels are aligned with the logits (the data pipeline shifts them)
        st = _RuntimeStepState(labels_used=used, tokens=int(ids.numel()), samples=int(ids.shape[0]),
                               hist_this_step=step > 0 and step % self.histogram_steps == 0,
                               blocks_to_monitor=blocks, log_this_step=log_this_step,
                               _effective=(used != -100).sum())
        return loss, st

    def runtime_post_backward_metrics(self, *, step: int, step_state: _RuntimeStepState) -> Optional[float]:
        """After the backward: the pre-clip gradient norm on logged and histogram steps (None on the
        others, which therefore never wait for the device) and the data-health, attention, activation
        and residual readings of a logged step. Clipping itself is applied on the device inside the
        optimizer's update, on every step."""
        tc, mc = self.config.training, self.config.monitoring
        need = step_state.log_this_step or step_state.hist_this_step
        gnorm = float(self.optimizer.grad_norm()) if need else None
        if gnorm is not None and mc.fail_fast_nonfinite and not math.isfinite(gnorm):
            raise NonFiniteError(f"step {step}: gradient norm {gnorm}")
        if step_state.log_this_step:
            used = step_state.labels_used
            ign = 1.0 - step_state.effective_tokens / max(1, used.numel())
            self._scalar("Data/ignore_frac", ign, step)
            self._band("ignore fraction", ign, step, warn_hi=self.config.alerts.ignore_frac_warn,
                       bad_hi=self.config.alerts.ignore_frac_bad)
            if gnorm is not None:
                cc = clip_coef(gnorm, tc.clip_grad) if tc.clip_grad and tc.clip_grad > 0 else 1.0
                self._scalar("Gradients/norm", gnorm, step)
                self._scalar("Gradients/clipped", float(self._is_step_clipped(gnorm)), step)
                self._band("clip coefficient", cc, step, warn_lo=self.config.alerts.clip_coef_warn,
                           bad_lo=self.config.alerts.clip_coef_bad)
            self._log_attention_metrics(step, blocks_to_monitor=step_state.blocks_to_monitor)
            self._log_watches(step)
        if step_state.hist_this_step:
            self._log_gradient_histograms(step)
        return gnorm

    def runtime_apply_optimizer_step(self, *, step: int, step_applied: bool = True) -> float:
        """Optimizer step (unless skipped), scheduler step and persistent low-bit refresh; returns the
        learning rate the step used."""
        lr = self.scheduler.step()
        if step_applied:
            self.optimizer.step()
            for m in self._persistent_lowbit:
                m.refresh_persistent_lowbit_params()
        return lr

    def training_step(self, batch) -> tuple[torch.Tensor, int]:
        """Forward + backward over ``micro_batch_size`` slices of ``batch``; returns (mean loss on the
        device, non-ignored label count)."""
        B = batch["input_ids"].shape[0]
        mb = min(self.micro_batch_size, B)
        n_mb = max(1, (B + mb - 1) // mb)
        total = torch.zeros((), device=self.device, dtype=torch.float32)
        tokens = 0
        pcc = self.precision_controller
        for i in range(n_mb):
            part = {k: v[i * mb:(i + 1) * mb] for k, v in batch.items() if torch.is_tensor(v)}
            loss, st = self.runtime_forward_loss(part, step=self.global_step, log_this_step=False)
            (pcc.backward(loss / n_mb) if pcc is not None else (loss / n_mb).backward())
            total += loss.detach().float()
            tokens += st.effective_tokens
        return total / n_mb, tokens

    # ------------------------------------------------------------------ small hooks (scripts call these)
    def _maybe_sync_cuda_timing(self) -> None:
        if self.config.monitoring.sync_cuda_timing and self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _is_step_clipped(self, grad_norm: Optional[float]) -> bool:
        clip = self.config.training.clip_grad
        return bool(clip and clip > 0 and grad_norm is not None and grad_norm > clip)

    def _update_loss_ema(self, loss_value: float) -> tuple[float, float]:
        """(new EMA, loss / previous EMA); the spike ratio is 1 on the first call. Raises when the
        ratio passes ``alerts.loss_spike_stop`` and warns past ``loss_spike_warn``."""
        prev = self._loss_ema
        beta = self.config.monitoring.loss_ema_beta
        self._loss_ema = loss_value if prev is None else beta * prev + (1.0 - beta) * loss_value
        ratio = 1.0 if prev is None or prev <= 0 else loss_value / prev
        al = self.config.alerts
        if ratio > al.loss_spike_stop:
            raise RuntimeError(f"loss {loss_value:.4f} is {ratio:.1f}x its EMA {prev:.4f} "
                               f"(stop threshold {al.loss_spike_stop})")
        if ratio > al.loss_spike_warn:
            logger.warning("loss spike: %.4f is %.1fx the EMA %.4f", loss_value, ratio, prev)
        return self._loss_ema, ratio

    def _flush_writer(self) -> None:
        self.writer.flush()

    # ------------------------------------------------------------------ logging
    def _scalar(self, tag: str, value, step: int) -> None:
        self.writer.add_scalar(tag, float(value), step)

    def _band(self, what: str, value: float, step: int, *, warn_lo=None, bad_lo=None, warn_hi=None,
              bad_hi=None) -> None:
        if not math.isfinite(value):
            return
        if (bad_lo is not None and value < bad_lo) or (bad_hi is not None and value > bad_hi):
            logger.warning("step %d: %s %.4g is in the BAD range", step, what, value)
        elif (warn_lo is not None and value < warn_lo) or (warn_hi is not None and value > warn_hi):
            logger.warning("step %d: %s %.4g is in the warning range", step, what, value)

    def _log_watches(self, step: int) -> None:
        al = self.config.alerts
        if self._act_watch is not None:
            for site, (rms, amax, outl) in self._act_watch.collect().items():
                self._scalar(f"Activations/{site}/rms", rms, step)
                self._scalar(f"Activations/{site}/max_abs", amax, step)
                self._band(f"activation rms at {site}", rms, step, warn_lo=al.activation_rms_warn_low,
                           bad_lo=al.activation_rms_bad_low, warn_hi=al.activation_rms_warn_high,
                           bad_hi=al.activation_rms_bad_high)
                self._band(f"activation max|x| at {site}", amax, step, warn_hi=al.activation_max_abs_warn,
                           bad_hi=al.activation_max_abs_bad)
        if self._res_watch is not None:
            for site, (rms, amax, outl, growth) in self._res_watch.collect().items():
                self._scalar(f"Residual/{site}/rms", rms, step)
                self._scalar(f"Residual/{site}/max_abs", amax, step)
                self._scalar(f"Residual/{site}/outlier_rate", outl, step)
                self._scalar(f"Residual/{site}/growth", growth, step)
                self._band(f"residual outlier rate at {site}", outl, step, warn_hi=al.residual_outlier_rate_warn,
                           bad_hi=al.residual_outlier_rate_bad)

    def _log_attention_metrics(self, step: int, *, blocks_to_monitor: set) -> None:
        al = self.config.alerts
        for i in sorted(blocks_to_monitor):
            attn = self._attn_by_block[i] if i < len(self._attn_by_block) else None
            stats = getattr(attn, "_monitor_stats", None) if attn is not None else None
            if not stats:
                continue
            for key in ("max_attn_logit", "attn_entropy", "attn_entropy_norm"):
                self._scalar(f"Attention/block_{i}/{key}", stats.get(key, float("nan")), step)
            if self.monitoring_mode == "debug" and "frac_logits_gt_tau" in stats:
                self._scalar(f"Attention/block_{i}/frac_logits_gt_tau", stats["frac_logits_gt_tau"], step)
            self._band(f"max attention logit of block {i}", stats.get("max_attn_logit", float("nan")), step,
                       warn_hi=al.max_attn_logit_warn, bad_hi=al.max_attn_logit_crit)
            self._band(f"normalised attention entropy of block {i}", stats.get("attn_entropy_norm", float("nan")),
                       step, warn_lo=al.attn_entropy_norm_warn)

    def _histogram_params(self):
        if self.monitoring_mode == "debug":
            return [(n, p) for n, p in self.model.named_parameters() if p.requires_grad]
        return list(self._sentinels.items())

    def _log_weight_histograms(self, step: int) -> None:
        for name, p in self._histogram_params():
            self.writer.add_histogram(f"Hist/weights/{name}", p.detach().float().cpu(), step)

    def _log_gradient_histograms(self, step: int) -> None:
        for name, p in self._histogram_params():
            g = getattr(p, "main_grad", None)
            g = p.grad if g is None else g
            if g is not None:
                self.writer.add_histogram(f"Hist/gradients/{name}", g.detach().float().cpu(), step)

    def _param_norm(self) -> float:
        sq = torch.zeros((), device=self.device)
        for p in self.model.parameters():
            sq += p.detach().float().pow(2).sum()
        return float(sq.sqrt())

    def _log_train_step(self, *, progress=None, step: int, lr_used: float, loss_value: float, loss_ema: float,
                        loss_spike_ratio: float, tokens: int, effective_tokens: int, step_seconds: float,
                        data_wait_seconds: float, totals: _TrainTotals, window: _TrainWindow,
                        grad_norm: Optional[float] = None) -> dict:
        """Scalars, console line and alerts of a logged step; resets ``window``."""
        cfg, mc = self.config, self.config.monitoring
        now = time.time()
        wall = window.elapsed_seconds(now=now)
        tps = window.effective_tokens / wall
        self._scalar("Loss/train", loss_value, step)
        self._scalar("Loss/train_ema", loss_ema, step)
        self._scalar("Loss/spike_ratio", loss_spike_ratio, step)
        self._scalar("Loss/perplexity", math.exp(min(loss_value, 50.0)), step)
        self._scalar("LR", lr_used, step)
        self._scalar("Tokens/step", tokens, step)
        self._scalar("Tokens/effective_step", effective_tokens, step)
        self._scalar("Tokens/total", totals.tokens, step)
        self._scalar("Tokens/effective_total", totals.effective_tokens, step)
        self._scalar("Tokens/samples_total", totals.samples, step)
        busy = step_seconds + data_wait_seconds
        wait_frac = data_wait_seconds / busy if busy > 0 else 0.0
        self._scalar("Time/step_seconds", step_seconds, step)
        self._scalar("Time/data_wait_seconds", data_wait_seconds, step)
        self._scalar("Time/data_wait_frac", wait_frac, step)
        self._scalar("Time/compute_frac", 1.0 - wait_frac, step)
        self._band("data-wait fraction", wait_frac, step, warn_hi=cfg.alerts.data_wait_frac_warn,
                   bad_hi=cfg.alerts.data_wait_frac_bad)
        self._scalar("Throughput/tokens_per_second", tps, step)
        self._scalar("Throughput/samples_per_second", window.samples / wall, step)
        self._scalar("Throughput/steps_per_second", window.steps / wall, step)
        self._scalar("Gradients/clip_rate", window.clip_rate(), step)
        tf = achieved_tflops(tps, self.num_params, flops_multiplier=mc.mfu_flops_multiplier)
        self._scalar("Perf/achieved_tflops", tf, step)
        self._scalar("Perf/mfu", mfu(tf, self._peak_tflops), step)
        line = {"step": step, "loss": loss_value, "lr": lr_used, "tokens_per_second": tps}
        if grad_norm is not None and math.isfinite(grad_norm):
            tc = cfg.training
            cc = clip_coef(grad_norm, tc.clip_grad) if tc.clip_grad and tc.clip_grad > 0 else 1.0
            pn = self._param_norm()
            self._scalar("Gradients/global_norm_pre_clip", grad_norm, step)
            self._scalar("Gradients/clip_coef", cc, step)
            self._scalar("Weights/global_norm", pn, step)
            self._scalar("Weights/global_update_ratio",
                         global_update_ratio(lr_used, grad_norm_pre_clip=grad_norm, clip_coef_value=cc, param_norm=pn),
                         step)
            al = cfg.alerts
            if grad_norm > al.grad_norm_stop_max:
                raise RuntimeError(f"step {step}: gradient norm {grad_norm:.3e} > {al.grad_norm_stop_max}")
            self._band("gradient norm", grad_norm, step, warn_lo=al.grad_norm_warn_min, warn_hi=al.grad_norm_warn_max)
            line.update(grad_norm=grad_norm, clip_coef=cc)
        logger.info("step %d | loss %.4f | lr %.3e | grad_norm %s | %.0f tok/s | data wait %.0f%%", step, loss_value,
                    lr_used, f"{grad_norm:.3f}" if grad_norm is not None else "-", tps, 100 * wait_frac)
        window.reset(start_time=now)
        return line

    def _log_gpu(self, step: int) -> None:
        if self.device.type != "cuda":
            return
        alloc = torch.cuda.memory_allocated(self.device)
        reserved = torch.cuda.memory_reserved(self.device)
        total = torch.cuda.get_device_properties(self.device).total_memory
        self._scalar("Memory/allocated_gb", alloc / 2**30, step)
        self._scalar("Memory/reserved_gb", reserved / 2**30, step)
        self._scalar("Memory/peak_allocated_gb", torch.cuda.max_memory_allocated(self.device) / 2**30, step)
        frac = reserved / max(total, 1)
        self._scalar("Memory/reserved_frac", frac, step)
        self._band("reserved memory fraction", frac, step, warn_hi=self.config.alerts.reserved_frac_warn,
                   bad_hi=self.config.alerts.reserved_frac_bad)
        if self._nvml is not None:
            nv, h = self._nvml, self._nvml_handle
            try:
                self._scalar("GPU/power_w", nv.nvmlDeviceGetPowerUsage(h) / 1000.0, step)
                self._scalar("GPU/sm_clock_mhz", nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), step)
                self._scalar("GPU/utilization_pct", nv.nvmlDeviceGetUtilizationRates(h).gpu, step)
                self._scalar("GPU/temperature_c", nv.nvmlDeviceGetTemperature(h, nv.NVML_TEMPERATURE_GPU), step)
            except Exception:
                pass

    def _log_sentinels(self, step: int, lr: float) -> None:
        al = self.config.alerts
        for name, p in self._sentinels.items():
            w = p.detach().float()
            wn = float(w.norm())
            self._scalar(f"Weights/norm/{name}", wn, step)
            prev = self._prev_sentinel.get(name)
            if prev is not None:
                ratio = float((w - prev).norm()) / (wn + 1e-12)
                self._scalar(f"Weights/update_ratio/{name}", ratio, step)
                self._band(f"update ratio of {name}", ratio, step, warn_lo=al.update_ratio_warn_low,
                           warn_hi=al.update_ratio_warn_high, bad_hi=al.update_ratio_stop_high)
            mg = getattr(p, "main_grad", None)
            if mg is not None:
                gn = float(mg.float().norm())
                self._scalar(f"Gradients/norm/{name}", gn, step)
                self._scalar(f"Gradients/update_ratio_proxy/{name}", update_ratio(lr, grad_norm=gn, weight_norm=wn),
                             step)
            self._prev_sentinel[name] = w.clone()

    def _check_opt_state_finite(self) -> None:
        for i, sh in enumerate(self.optimizer.state_tensors()):
            for k in ("master", "exp_avg", "exp_avg_sq"):
                if not bool(torch.isfinite(sh[k]).all()):
                    raise NonFiniteError(f"optimizer state {k} of buffer {i} is not finite")

    # ------------------------------------------------------------------ probe and evaluation
    def _capture_probe(self) -> None:
        src = self.val_loader if self.val_loader is not None else self.train_loader
        batch = next(iter(src))
        ids = batch["input_ids"][:1].clone().cpu()
        lab = batch["labels"][:1].clone().cpu()
        self._probe = (ids, lab)
        self._probe_hash = self._hash_probe(ids, lab)

    def _hash_probe(self, ids, lab) -> str:
        cfg = self.config
        return eval_artifact_hash(input_ids_bytes=ids.numpy().tobytes(), labels_bytes=lab.numpy().tobytes(),
                                  input_dtype=str(ids.dtype), labels_dtype=str(lab.dtype),
                                  input_shape=tuple(ids.shape), labels_shape=tuple(lab.shape),
                                  vocab_size=cfg.model.vocab_size, max_seq_length=cfg.data.max_seq_length,
                                  seed=cfg.seed)

    @torch.no_grad()
    def _run_fixed_probe(self, *, step: int) -> None:
        """Loss and last-token log-probability drift on a fixed batch whose hash must not change."""
        if self._probe is None:
            self._capture_probe()
        ids, lab = self._probe
        if self._hash_probe(ids, lab) != self._probe_hash:
            raise RuntimeError("fixed probe batch changed (hash mismatch)")
        was = self.model.training
        self.model.eval()
        try:
            self._scalar("Probe/loss", float(self._loss(ids.to(self.device), lab.to(self.device))), step)
            logp = torch.log_softmax(self.model(ids.to(self.device)).float()[0, -1], -1)
            if self._probe_prev_logp is not None:
                self._scalar("Probe/last_token_logprob_drift", float((logp - self._probe_prev_logp).abs().mean()),
                             step)
            self._probe_prev_logp = logp
        finally:
            self.model.train(was)

    @torch.no_grad()
    def evaluate(self, loader=None, *, step: int = 0, max_batches: Optional[int] = None) -> dict[str, float]:
        loader = loader if loader is not None else self.val_loader
        if loader is None:
            return {}
        self.model.eval()
        tot = torch.zeros((), device=self.device)
        n = 0
        for i, batch in enumerate(loader):
            if max_batches is not None and i >= max_batches:
                break
            tot += self._loss(batch["input_ids"].to(self.device), batch["labels"].to(self.device)).float()
            n += 1
        self.model.train()
        if n == 0:
            return {}
        loss = float(tot) / n
        out = {"loss": loss, "perplexity": math.exp(min(loss, 50.0))}
        self._scalar("Eval/loss", out["loss"], step)
        self._scalar("Eval/perplexity", out["perplexity"], step)
        return out

    # ------------------------------------------------------------------ checkpoint
    def save_checkpoint(self, step: int, final: bool = False) -> str:
        d = os.path.join(self.config.output_dir, f"checkpoint-step-{step}")
        os.makedirs(d, exist_ok=True)
        torch.save(self.model.state_dict(), os.path.join(d, "model.pt"))
        torch.save(self.optimizer.state_dict(), os.path.join(d, "optimizer.pt"))
        torch.save(self.scheduler.state_dict(), os.path.join(d, "scheduler.pt"))
        with open(os.path.join(d, "config.json"), "w") as f:
            json.dump(config_to_serializable_dict(self.config), f, indent=1)
        with open(os.path.join(d, "trainer_state.json"), "w") as f:
            json.dump({"global_step": step, "final": final}, f)
        size = sum(os.path.getsize(os.path.join(d, x)) for x in os.listdir(d))
        self._scalar("Checkpoint/ok", 1.0, step)
        self._scalar("Checkpoint/size_mb", size / 2**20, step)
        logger.info("saved checkpoint %s (%.1f MB)", d, size / 2**20)
        return d

    def load_checkpoint(self, path: str) -> int:
        self.model.load_state_dict(torch.load(os.path.join(path, "model.pt"), map_location=self.device))
        self.optimizer.load_state_dict(torch.load(os.path.join(path, "optimizer.pt"), map_location="cpu",
                                                  weights_only=False))
        self.scheduler.load_state_dict(torch.load(os.path.join(path, "scheduler.pt"), weights_only=False))
        with open(os.path.join(path, "trainer_state.json")) as f:
            self.global_step = int(json.load(f)["global_step"])
        return self.global_step

    def _finalize_training(self, *, step: int, totals: _TrainTotals, elapsed_seconds: float,
                           final_loss: float) -> None:
        self._scalar("Final/loss", final_loss, step)
        self._scalar("Final/tokens", totals.tokens, step)
        self._scalar("Final/effective_tokens", totals.effective_tokens, step)
        self._scalar("Final/elapsed_seconds", elapsed_seconds, step)
        self._scalar("Final/tokens_per_second", totals.effective_tokens / max(elapsed_seconds, 1e-9), step)
        logger.info("training finished at step %d: loss %.4f, %d tokens in %.1f s", step, final_loss, totals.tokens,
                    elapsed_seconds)
        self.writer.flush()

    # ------------------------------------------------------------------ the loop
    def _batches(self):
        while True:
            for batch in self.train_loader:
                yield batch

    def train(self) -> dict:
        tc, mc = self.config.training, self.config.monitoring
        self.model.train()
        self._capture_probe()
        totals = _TrainTotals()
        window = _TrainWindow(start_time=time.time())
        t_start = time.time()
        last: dict = {}
        loss_value = float("nan")
        batches = self._batches()
        pcc = self.precision_controller
        step = self.global_step
        prev_end = time.time()
        clip = tc.clip_grad if tc.clip_grad and tc.clip_grad > 0 else None
        # device-side window accumulators, read on logged steps only
        eff_acc = torch.zeros((), dtype=torch.int64, device=self.device)
        clip_acc = torch.zeros((), dtype=torch.float32, device=self.device)
        while step < tc.max_steps:
            batch = next(batches)
            t0 = time.time()
            data_wait = t0 - prev_end
            log_this = (step + 1) % self.log_steps == 0 or step + 1 == tc.max_steps
            self.optimizer.zero_grad()
            # gradient accumulation: the logged forward is the first micro-batch's
            B = batch["input_ids"].shape[0]
            mb = min(self.micro_batch_size, B)
            n_mb = max(1, (B + mb - 1) // mb)
            loss_dev = torch.zeros((), device=self.device)
            st0 = None
            for i in range(n_mb):
                part = {k: v[i * mb:(i + 1) * mb] for k, v in batch.items() if torch.is_tensor(v)}
                loss, st = self.runtime_forward_loss(part, step=step + 1, log_this_step=log_this and i == 0)
                (pcc.backward(loss / n_mb) if pcc is not None else (loss / n_mb).backward())
                loss_dev += loss.detach().float() / n_mb
                if st0 is None:
                    st0 = st
                else:
                    st0._effective = st0._effective + st._effective
                    st0.tokens += st.tokens
                    st0.samples += st.samples
            applied = True
            if pcc is not None and pcc.uses_loss_scaling:
                applied = pcc.prepare_optimizer_step(self.model)
            gnorm = self.runtime_post_backward_metrics(step=step + 1, step_state=st0)
            lr = self.runtime_apply_optimizer_step(step=step + 1, step_applied=applied)
            if pcc is not None and pcc.uses_loss_scaling:
                pcc.update_after_step(step_applied=applied)
            step += 1
            eff_acc += st0._effective
            if clip is not None and applied and self.optimizer.last_grad_norm is not None:
                clip_acc += (self.optimizer.last_grad_norm.reshape(()) > clip).float()
            self._maybe_sync_cuda_timing()
            t1 = time.time()
            window.update(tokens=st0.tokens, effective_tokens=0, samples=st0.samples, clipped=False)
            totals.update(tokens=st0.tokens, effective_tokens=0, samples=st0.samples)
            if log_this:
                eff, clipped = (int(v) for v in torch.stack([eff_acc.float(), clip_acc]).tolist())
                eff_acc.zero_()
                clip_acc.zero_()
                window.effective_tokens += eff
                window.clipped_steps += clipped
                totals.effective_tokens += eff
                loss_value = float(loss_dev)
                if mc.fail_fast_nonfinite and not math.isfinite(loss_value):
                    raise NonFiniteError(f"step {step}: loss {loss_value}")
                ema, ratio = self._update_loss_ema(loss_value)
                last = self._log_train_step(step=step, lr_used=lr, loss_value=loss_value, loss_ema=ema,
                                            loss_spike_ratio=ratio, tokens=st0.tokens,
                                            effective_tokens=st0.effective_tokens, step_seconds=t1 - t0,
                                            data_wait_seconds=data_wait, totals=totals, window=window,
                                            grad_norm=gnorm)
            if mc.gpu_metrics_steps and step % mc.gpu_metrics_steps == 0 and mc.log_memory:
                self._log_gpu(step)
            if mc.mode != "minimal" and mc.update_ratio_steps and step % mc.update_ratio_steps == 0:
                self._log_sentinels(step, lr)
            if mc.opt_state_check_steps and step % mc.opt_state_check_steps == 0:
                self._check_opt_state_finite()
            if mc.probe_steps and step % mc.probe_steps == 0:
                self._run_fixed_probe(step=step)
            if st0.hist_this_step:
                self._log_weight_histograms(step)
            if self.val_loader is not None and tc.eval_steps and step % tc.eval_steps == 0:
                last["eval"] = self.evaluate(step=step)
            if tc.save_steps and step % tc.save_steps == 0:
                self.save_checkpoint(step)
            if mc.tensorboard_flush_on_log and log_this:
                self._flush_writer()
            prev_end = time.time()
        self.global_step = step
        if self.val_loader is not None:
            last["eval"] = self.evaluate(step=step)
        self.save_checkpoint(step, final=True)
        self._finalize_training(step=step, totals=totals, elapsed_seconds=time.time() - t_start,
                                final_loss=loss_value)
        return last
