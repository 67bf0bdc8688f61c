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
_SR = ["nearest", "stochastic"]

# (flag, argparse keywords) in the order they are registered, by topic. The help texts describe
# what each flag does in this framework.
_FLAGS: tuple = (
    # compute precision
    ("--precision-recipe", dict(type=str, default="default", choices=["default", "deepseek_v3"],
                                help="preset of the per-module precision policy; deepseek_v3 turns on the FP8 "
                                     "training recipe (1x128 activation and 128x128 weight scales)")),
    ("--bf16", dict(action="store_true", help="compute in bfloat16 (fp32 master weights)")),
    ("--fp16", dict(action="store_true", help="compute in float16 with dynamic loss scaling")),
    ("--fp8", dict(action="store_true", help="run the selected linears with e4m3 operands")),
    ("--fp4", dict(action="store_true", help="run the selected linears with 4-bit operands")),
    ("--fp8-backend", dict(type=str, default="transformer_engine", choices=["transformer_engine", "emulated", "native"],
                           help="who executes the FP8 math: Transformer Engine modules, a PyTorch emulation, or "
                                "this framework's block-scaled e4m3 tensor-core GEMMs (native)")),
    ("--fp8-format", dict(type=str, default="e4m3", choices=["e4m3", "hybrid"],
                          help="e4m3 everywhere, or e4m3 forward / e5m2 gradients (hybrid)")),
    ("--fp8-amax-history-len", dict(type=int, default=16, help="steps of amax history kept per tensor")),
    ("--fp8-amax-compute-algo", dict(type=str, default="most_recent", choices=["most_recent", "max"],
                                     help="scale from the latest amax or from the maximum of the history")),
    ("--fp4-backend", dict(type=str, default="emulated", choices=["emulated", "native"],
                           help="who executes the FP4 math: a PyTorch emulation, or NVFP4 (e2m1 in 1x16 blocks with "
                                "e4m3 scales) on the fp4 tensor cores (native)")),
    # storage dtypes of parameters and optimizer state
    ("--params-dtype", dict(type=str, default=None, choices=_DT, help="dtype the model's parameters are stored in")),
    ("--main-params-dtype", dict(type=str, default=None, choices=_DT, help="dtype of the optimizer's master weights")),
    ("--main-grads-dtype", dict(type=str, default=None, choices=_DT,
                                help="dtype of the gradient buffers the optimizer reads")),
    ("--exp-avg-dtype", dict(type=str, default=None, choices=_DT, help="dtype of Adam's first moment")),
    ("--exp-avg-sq-dtype", dict(type=str, default=None, choices=_DT, help="dtype of Adam's second moment")),
    # dynamic loss scaling
    ("--loss-scale-init", dict(type=float, default=65536.0, help="initial loss scale")),
    ("--loss-scale-growth-factor", dict(type=float, default=2.0, help="multiplier after a run of finite steps")),
    ("--loss-scale-backoff-factor", dict(type=float, default=0.5, help="multiplier after a non-finite step")),
    ("--loss-scale-growth-interval", dict(type=int, default=2000, help="finite steps between two growths")),
    ("--loss-scale-min", dict(type=float, default=1.0, help="lower bound of the loss scale")),
    ("--loss-scale-max", dict(type=float, default=16777216.0, help="upper bound of the loss scale")),
    # persistent low-bit weights
    ("--fp8-param", dict(action="store_true", help="keep an e4m3 copy of the selected weights for the forward")),
    ("--fp4-param", dict(action="store_true", help="keep an NF4 copy of the selected weights for the forward")),
    ("--fp4-param-format", dict(type=str, default="nf4", choices=["nf4"], help="encoding of the 4-bit weight copy")),
    ("--persistent-scale-granularity", dict(type=str, default="per_channel", choices=["per_tensor", "per_channel"],
                                            help="one scale per weight tensor or per output channel")),
    # per-module selection
    ("--module-pattern-type", dict(type=str, default="regex", choices=["regex", "glob"],
                                   help="how the include / exclude patterns below match module paths")),
    ("--compute-lowbit-mode", dict(type=str, default=None, choices=["fp8", "fp4"],
                                   help="low-bit compute for the modules the include / exclude patterns select")),
    ("--compute-lowbit-include", dict(action="append", default=None,
                                      help="module-path pattern that gets low-bit compute (repeatable)")),
    ("--compute-lowbit-exclude", dict(action="append", default=None,
                                      help="module-path pattern kept at full compute precision (repeatable)")),
    ("--persistent-lowbit-mode", dict(type=str, default="off", choices=["off", "fp8", "fp4"],
                                      help="persistent low-bit weight copy for the selected modules")),
    ("--persistent-lowbit-include", dict(action="append", default=None,
                                         help="module-path pattern that keeps a low-bit weight copy (repeatable)")),
    ("--persistent-lowbit-exclude", dict(action="append", default=None,
                                         help="module-path pattern without a low-bit weight copy (repeatable)")),
    ("--module-compute-dtype-rule", dict(action="append", default=None,
                                         help="'<pattern>=<fp32|bf16|fp16>': compute dtype of matching modules "
                                              "(repeatable)")),
    ("--lowbit-master-ownership", dict(type=str, default="optimizer", choices=["module", "optimizer"],
                                       help="whether the trainable master of a low-bit weight lives in the module "
                                            "or in the optimizer's master store")),
    # DeepSeek-V3 FP8 recipe details
    ("--fp8-rounding", dict(type=str, default=None, choices=_SR,
                            help="rounding of values quantised to e4m3 (stochastic: unbiased in expectation)")),
    ("--fp8-activation-granularity", dict(type=str, default=None, choices=["tile_1x128", "tensor", "channel"],
                                          help="scale granularity of FP8 activations")),
    ("--fp8-weight-granularity", dict(type=str, default=None, choices=["block_128x128", "tensor", "channel"],
                                      help="scale granularity of FP8 weights")),
    ("--fp8-comm-quant", dict(action=argparse.BooleanOptionalAction, default=None,
                              help="send the MoE dispatch / combine payload as e4m3 with scales")),
    ("--fp8-comm-granularity", dict(type=str, default=None, choices=["block_128x128", "tensor", "channel"],
                                    help="scale granularity of the e4m3 MoE payload")),
)


def add_mixed_precision_args(parser: argparse.ArgumentParser) -> None:
    """Register every shared precision flag on ``parser``."""
    for flag, kw in _FLAGS:
        parser.add_argument(flag, **kw)


def normalize_and_resolve_precision(args: argparse.Namespace, device: torch.device) -> PrecisionConfig:
    return resolve_precision_config(args, device)


def build_precision_runtime(args: argparse.Namespace, device: torch.device):
    """``(precision_config, module_resolver, controller)`` from the shared flags: the resolver is passed
    to every layer's constructor (then ``finalize_module_precision_resolver``), the controller gives the
    autocast context, loss scaling and the non-finite skip of a training step."""
    from .mixed_precision import MixedPrecisionController, build_module_precision_resolver

    pc = normalize_and_resolve_precision(args, device)
    return pc, build_module_precision_resolver(pc), MixedPrecisionController(pc, device=device)
