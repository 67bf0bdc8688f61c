"""Single-process Trainer for the MVP path (reference: src/trainer.py:119-2070).

``Trainer(model, config, train_loader, device, val_loader=None).train()``
runs the reference's loop on this framework's pieces:

* optimizer ``create_optimizer`` (flat-buffer fused AdamW; gradient clipping
  at ``training.clip_grad`` is a device-side scale inside the update, so a
  step does not synchronise with the host), ``CosineAnnealingScheduler``
  (linear warm-up, cosine to 0), gradient accumulation from
  ``training.batch_size / training.micro_batch_size``;
* loss through ``model.forward_loss`` when the model has it (fused
  cross-entropy, logits never materialised in fp32), else
  ``CrossEntropyLoss`` on the logits;
* periodic evaluation (mean loss, perplexity) and a fixed probe batch whose
  SHA-256 (``monitoring.eval_artifact_hash``) must not change;
* metrics every ``log_steps``: loss, EMA, perplexity, LR, gradient norm
  before clipping, clip coefficient, global update ratio, tokens/s,
  achieved TFLOP/s and MFU, CUDA memory, NVML power/clock/utilisation, and
  per-sentinel-tensor weight norms and update ratios;
* alerts from ``AlertThresholdsConfig`` (loss spikes, gradient norm) and
  fail-fast on non-finite loss, gradient norm or optimizer state;
* checkpoints ``checkpoint-step-{N}/`` with model.pt, optimizer.pt,
  scheduler.pt and config.json (``save_checkpoint`` / ``load_checkpoint``).

Scalars go to TensorBoard when it is importable, else to
``<log_dir>/<run_name>/metrics.jsonl``.
"""
from __future__ import annotations

import json
import math
import os
import time
from typing import Optional

import torch

from .config import Config, config_to_serializable_dict
from .distributed.failure import NonFiniteError
from .logging import get_logger
from .losses import CrossEntropyLoss
from .monitoring import (achieved_tflops, candidate_sentinel_param_names, clip_coef, eval_artifact_hash,
                         global_update_ratio, mfu, resolve_sentinel_blocks, update_ratio)
from .optimizer import create_optimizer
from .scheduler import CosineAnnealingScheduler

logger = get_logger(__name__)


class _JsonlWriter:
    def __init__(self, path: str):
        os.makedirs(os.path.dirname(path), exist_ok=True)
        self._f = open(path, "a", encoding="utf-8")

    def add_scalar(self, tag: str, value: float, step: int) -> None:
        self._f.write(json.dumps({"tag": tag, "value": float(value), "step": int(step)}) + "\n")

    def add_histogram(self, tag: str, values, step: int) -> None:
        v = values.detach().float().flatten()
        self.add_scalar(tag + "/mean", float(v.mean()), step)
        self.add_scalar(tag + "/std", float(v.std()) if v.numel() > 1 else 0.0, step)

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
        self.log_steps = max(1, int(tc.log_steps))
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
        # Sentinel tensors (bounded monitoring): fixed names, filtered to what the model has.
        nl = int(getattr(getattr(model, "config", None), "num_layers", 0) or len(getattr(model, "blocks", [])))
        self._sentinel_blocks = resolve_sentinel_blocks(nl, mc.sentinel_blocks)
        named = dict(model.named_parameters())
        self._sentinels = {n: named[n] for n in sorted(candidate_sentinel_param_names(
            sentinel_blocks=self._sentinel_blocks)) if n in named}
        self._prev_sentinel = {}
        self._probe = None
        self._probe_hash = None
        self._probe_prev_logp = None
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

    # ------------------------------------------------------------------ loss
    def _loss(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        if hasattr(self.model, "forward_loss"):
            return self.model.forward_loss(input_ids, labels)
        logits = self.model(input_ids)
        return self.criterion(logits, labels)

    def training_step(self, batch) -> tuple[torch.Tensor, int]:
        """Forward + backward over micro-batches of ``batch``; returns (mean loss on device, tokens)."""
        ids = batch["input_ids"].to(self.device, non_blocking=True)
        lab = batch["labels"].to(self.device, non_blocking=True)
        B = ids.shape[0]
        mb = min(self.micro_batch_size, B)
        n_mb = max(1, (B + mb - 1) // mb)
        total = torch.zeros((), device=self.device, dtype=torch.float32)
        pcc = self.precision_controller
        for i in range(n_mb):
            if pcc is not None:
                with pcc.autocast_context():
                    loss = self._loss(ids[i * mb:(i + 1) * mb], lab[i * mb:(i + 1) * mb])
                pcc.backward(loss / n_mb)
            else:
                loss = self._loss(ids[i * mb:(i + 1) * mb], lab[i * mb:(i + 1) * mb])
                (loss / n_mb).backward()
            total += loss.detach().float()
        return total / n_mb, int((lab != -100).sum())

    # ------------------------------------------------------------------ monitoring
    def _scalar(self, tag: str, value, step: int) -> None:
        self.writer.add_scalar(tag, float(value), step)

    def _param_norm(self) -> float:
        sq = torch.zeros((), device=self.device)
        for p in self.model.parameters():
            sq += p.detach().float().pow(2).sum()
        return float(sq.sqrt())

    def _check_opt_state_finite(self) -> None:
        for i, sh in enumerate(self.optimizer.state_tensors()):
            for k in ("master", "exp_avg", "exp_avg_sq"):
                if not bool(torch.isfinite(sh[k]).all()):
                    raise NonFiniteError(f"optimizer state {k} of buffer {i} is not finite")

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
        if frac > self.config.alerts.reserved_frac_bad:
            logger.warning("step %d: reserved memory fraction %.3f above %.2f", step, frac,
                           self.config.alerts.reserved_frac_bad)
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
        for name, p in self._sentinels.items():
            w = p.detach().float()
            wn = float(w.norm())
            self._scalar(f"Weights/norm/{name}", wn, step)
            prev = self._prev_sentinel.get(name)
            if prev is not None:
                delta = float((w - prev).norm())
                self._scalar(f"Weights/update_ratio/{name}", delta / (wn + 1e-12), step)
            mg = getattr(p, "main_grad", None)
            if mg is not None:
                self._scalar(f"Gradients/norm/{name}", float(mg.float().norm()), step)
                self._scalar(f"Gradients/update_ratio_proxy/{name}",
                             update_ratio(lr, grad_norm=float(mg.float().norm()), weight_norm=wn), step)
            self._prev_sentinel[name] = w.clone()

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
    def _run_probe(self, step: int) -> None:
        ids, lab = self._probe
        if self._hash_probe(ids, lab) != self._probe_hash:
            raise RuntimeError("fixed probe batch changed (hash mismatch)")
        self.model.eval()
        loss = float(self._loss(ids.to(self.device), lab.to(self.device)))
        self.model.train()
        self._scalar("Probe/loss", loss, step)
        if hasattr(self.model, "forward"):
            self.model.eval()
            logits = self.model(ids.to(self.device)).float()
            self.model.train()
            logp = torch.log_softmax(logits[0, -1], -1)
            if self._probe_prev_logp is not None:
                self._scalar("Probe/last_token_logprob_drift", float((logp - self._probe_prev_logp).abs().mean()), step)
            self._probe_prev_logp = logp

    @torch.no_grad()
    def evaluate(self, loader=None, *, step: int = 0, max_batches: Optional[int] = None) -> dict[str, float]:
        loader = loader if loader is not None else self.val_loader
        if loader is None:
            return {}
        self.model.eval()
        tot, n = 0.0, 0
        for i, batch in enumerate(loader):
            if max_batches is not None and i >= max_batches:
                break
            tot += float(self._loss(batch["input_ids"].to(self.device), batch["labels"].to(self.device)))
            n += 1
        self.model.train()
        if n == 0:
            return {}
        loss = tot / n
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

    # ------------------------------------------------------------------ loop
    def train(self) -> dict:
        cfg, tc, mc, al = self.config, self.config.training, self.config.monitoring, self.config.alerts
        self.model.train()
        self._capture_probe()
        step = self.global_step
        t_window = time.perf_counter()
        tokens_window = 0
        last = {}
        done = False
        while not done:
            for batch in self.train_loader:
                if step >= tc.max_steps:
                    done = True
                    break
                self.optimizer.zero_grad()
                loss_t, tokens = self.training_step(batch)
                lr = self.scheduler.step()
                pcc = self.precision_controller
                applied = True
                if pcc is not None and pcc.uses_loss_scaling:
                    applied = pcc.prepare_optimizer_step(self.model)  # unscale; skip on inf/nan
                    if applied:
                        self.optimizer.step()
                    pcc.update_after_step(step_applied=applied)
                else:
                    self.optimizer.step()
                if applied:
                    for m in self._persistent_lowbit:
                        m.refresh_persistent_lowbit_params()
                step += 1
                tokens_window += tokens
                if step % self.log_steps == 0 or step == tc.max_steps:
                    if mc.sync_cuda_timing and self.device.type == "cuda":
                        torch.cuda.synchronize(self.device)
                    loss = float(loss_t)
                    if mc.fail_fast_nonfinite and not math.isfinite(loss):
                        raise NonFiniteError(f"step {step}: loss {loss}")
                    beta = mc.loss_ema_beta
                    prev_ema = self._loss_ema
                    self._loss_ema = loss if prev_ema is None else beta * prev_ema + (1 - beta) * loss
                    gnorm = float(self.optimizer.last_grad_norm) if self.optimizer.last_grad_norm is not None \
                        else float("nan")
                    if mc.fail_fast_nonfinite and tc.clip_grad and not math.isfinite(gnorm):
                        raise NonFiniteError(f"step {step}: gradient norm {gnorm}")
                    cc = clip_coef(gnorm, tc.clip_grad) if math.isfinite(gnorm) else 1.0
                    pn = self._param_norm()
                    now = time.perf_counter()
                    tps = tokens_window / max(now - t_window, 1e-9)
                    t_window, tokens_window = now, 0
                    tf = achieved_tflops(tps, self.num_params, flops_multiplier=mc.mfu_flops_multiplier)
                    self._scalar("Loss/train", loss, step)
                    self._scalar("Loss/train_ema", self._loss_ema, step)
                    self._scalar("Loss/perplexity", math.exp(min(loss, 50.0)), step)
                    self._scalar("LR", lr, step)
                    self._scalar("Gradients/global_norm_pre_clip", gnorm, step)
                    self._scalar("Gradients/clip_coef", cc, step)
                    self._scalar("Weights/global_norm", pn, step)
                    self._scalar("Weights/global_update_ratio",
                                 global_update_ratio(lr, grad_norm_pre_clip=gnorm if math.isfinite(gnorm) else 0.0,
                                                     clip_coef_value=cc, param_norm=pn), step)
                    self._scalar("Throughput/tokens_per_second", tps, step)
                    self._scalar("Perf/achieved_tflops", tf, step)
                    self._scalar("Perf/mfu", mfu(tf, self._peak_tflops), step)
                    if prev_ema is not None and loss > al.loss_spike_stop * prev_ema:
                        raise RuntimeError(f"step {step}: loss {loss:.4f} > {al.loss_spike_stop}x EMA {prev_ema:.4f}")
                    if prev_ema is not None and loss > al.loss_spike_warn * prev_ema:
                        logger.warning("step %d: loss spike %.4f vs EMA %.4f", step, loss, prev_ema)
                    if math.isfinite(gnorm):
                        if gnorm > al.grad_norm_stop_max:
                            raise RuntimeError(f"step {step}: gradient norm {gnorm:.3e} > {al.grad_norm_stop_max}")
                        if gnorm > al.grad_norm_warn_max or gnorm < al.grad_norm_warn_min:
                            logger.warning("step %d: gradient norm %.3e outside [%g, %g]", step, gnorm,
                                           al.grad_norm_warn_min, al.grad_norm_warn_max)
                    logger.info("step %d | loss %.4f | lr %.3e | grad_norm %.3f | clip %.3f | %.0f tok/s", step,
                                loss, lr, gnorm, cc, tps)
                    last = {"step": step, "loss": loss, "lr": lr, "grad_norm": gnorm, "tokens_per_second": tps}
                if mc.gpu_metrics_steps and step % mc.gpu_metrics_steps == 0 and mc.log_memory:
                    self._log_gpu(step)
                if mc.mode != "minimal" and mc.update_ratio_steps and step % mc.update_ratio_steps == 0:
                    self._log_sentinels(step, lr)
                if mc.opt_state_check_steps and step % mc.opt_state_check_steps == 0:
                    self._check_opt_state_finite()
                if mc.probe_steps and step % mc.probe_steps == 0:
                    self._run_probe(step)
                if mc.mode == "debug" and mc.histogram_steps and step % mc.histogram_steps == 0:
                    for name, p in self._sentinels.items():
                        self.writer.add_histogram(f"Hist/{name}", p.detach().float().cpu(), step)
                if self.val_loader is not None and tc.eval_steps and step % tc.eval_steps == 0:
                    last["eval"] = self.evaluate(step=step)
                if tc.save_steps and step % tc.save_steps == 0:
                    self.save_checkpoint(step)
                if mc.tensorboard_flush_on_log:
                    self.writer.flush()
        self.global_step = step
        if self.val_loader is not None:
            last["eval"] = self.evaluate(step=step)
        self.save_checkpoint(step, final=True)
        self.writer.flush()
        return last
