"""Shared mixed-precision CLI flags of every entry script.

Flag names, defaults and choices are the reference's
(src/runtime/precision_args.py:13-220) so existing command lines work; the
fp8/fp4 backends additionally accept ``native`` (sm_100a e4m3 / NVFP4 path).
"""
from __future__ import annotations

import argparse

import torch

from ..runtime.contracts import PrecisionConfig
from .mixed_precision import resolve_precision_config

_DT = ["fp32", "bf16", "fp16"]


def add_mixed_precision_args(parser: argparse.ArgumentParser) -> None:
    a = parser.add_argument
    a("--precision-recipe", type=str, default="default", choices=["default", "deepseek_v3"],
      help="Precision policy preset. deepseek_v3 enables DeepSeek-V3 FP8 defaults.")
    a("--bf16", action="store_true", help="Enable BF16 mixed precision")
    a("--fp16", action="store_true", help="Enable FP16 mixed precision")
    a("--fp8", action="store_true", help="Enable FP8 mixed precision")
    a("--fp4", action="store_true", help="Enable FP4 mixed precision")
    a("--fp8-backend", type=str, default="transformer_engine", choices=["transformer_engine", "emulated", "native"],
      help="FP8 backend implementation (native = sm_100a e4m3 kernels)")
    a("--fp8-format", type=str, default="e4m3", choices=["e4m3", "hybrid"], help="FP8 format recipe")
    a("--fp8-amax-history-len", type=int, default=16, help="FP8 amax history length")
    a("--fp8-amax-compute-algo", type=str, default="most_recent", choices=["most_recent", "max"],
      help="FP8 amax update algorithm")
    a("--fp4-backend", type=str, default="emulated", choices=["emulated", "native"],
      help="FP4 backend implementation (native = NVFP4 numerics)")
    a("--params-dtype", type=str, default=None, choices=_DT, help="Model parameter dtype")
    a("--main-params-dtype", type=str, default=None, choices=_DT, help="Optimizer main parameter dtype")
    a("--main-grads-dtype", type=str, default=None, choices=_DT, help="Optimizer main grad dtype")
    a("--exp-avg-dtype", type=str, default=None, choices=_DT, help="Optimizer first-moment dtype")
    a("--exp-avg-sq-dtype", type=str, default=None, choices=_DT, help="Optimizer second-moment dtype")
    a("--loss-scale-init", type=float, default=65536.0)
    a("--loss-scale-growth-factor", type=float, default=2.0)
    a("--loss-scale-backoff-factor", type=float, default=0.5)
    a("--loss-scale-growth-interval", type=int, default=2000)
    a("--loss-scale-min", type=float, default=1.0)
    a("--loss-scale-max", type=float, default=16777216.0)
    a("--fp8-param", action="store_true", help="Enable persistent FP8 parameter storage for selected modules")
    a("--fp4-param", action="store_true", help="Enable persistent FP4 (NF4) parameter storage for selected modules")
    a("--fp4-param-format", type=str, default="nf4", choices=["nf4"], help="Persistent FP4 storage format")
    a("--persistent-scale-granularity", type=str, default="per_channel", choices=["per_tensor", "per_channel"],
      help="Scale granularity for persistent low-bit parameter quantization")
    a("--module-pattern-type", type=str, default="regex", choices=["regex", "glob"],
      help="Pattern matcher used by per-module low-bit include/exclude flags")
    a("--compute-lowbit-mode", type=str, default=None, choices=["fp8", "fp4"],
      help="Per-module low-bit compute mode override")
    a("--compute-lowbit-include", action="append", default=None,
      help="Repeatable include patterns for low-bit compute module selection")
    a("--compute-lowbit-exclude", action="append", default=None,
      help="Repeatable exclude patterns for low-bit compute module selection")
    a("--persistent-lowbit-mode", type=str, default="off", choices=["off", "fp8", "fp4"],
      help="Per-module persistent low-bit parameter mode override")
    a("--persistent-lowbit-include", action="append", default=None,
      help="Repeatable include patterns for persistent low-bit module selection")
    a("--persistent-lowbit-exclude", action="append", default=None,
      help="Repeatable exclude patterns for persistent low-bit module selection")
    a("--module-compute-dtype-rule", action="append", default=None,
      help="Repeatable per-module compute dtype override rule in '<pattern>=<fp32|bf16|fp16>' format")
    a("--lowbit-master-ownership", type=str, default="optimizer", choices=["module", "optimizer"],
      help="Ownership mode for trainable master weights in low-bit persistent paths")
    a("--fp8-rounding", type=str, default=None, choices=["nearest", "stochastic"],
      help="Rounding mode for FP8 quantization recipe")
    a("--fp8-activation-granularity", type=str, default=None, choices=["tile_1x128", "tensor", "channel"],
      help="Activation quantization granularity for FP8 recipe")
    a("--fp8-weight-granularity", type=str, default=None, choices=["block_128x128", "tensor", "channel"],
      help="Weight quantization granularity for FP8 recipe")
    a("--fp8-comm-quant", action=argparse.BooleanOptionalAction, default=None,
      help="Enable or disable FP8 communication quantization in MoE dispatch/combine")
    a("--fp8-comm-granularity", type=str, default=None, choices=["block_128x128", "tensor", "channel"],
      help="Communication quantization granularity for FP8 recipe")


def normalize_and_resolve_precision(args: argparse.Namespace, device: torch.device) -> PrecisionConfig:
    return resolve_precision_config(args, device)


def build_precision_runtime(args: argparse.Namespace, device: torch.device):
    """``(precision_config, module_resolver, controller)`` from the shared flags: the resolver is passed
    to every layer's constructor (then ``finalize_module_precision_resolver``), the controller gives the
    autocast context, loss scaling and the non-finite skip of a training step."""
    from .mixed_precision import MixedPrecisionController, build_module_precision_resolver

    pc = normalize_and_resolve_precision(args, device)
    return pc, build_module_precision_resolver(pc), MixedPrecisionController(pc, device=device)
