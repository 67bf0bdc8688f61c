"""Run-level precision policy: flag resolution, per-module resolver, loss scaling.

Behaviour (flags, defaults, validation messages) follows the reference's
src/runtime/mixed_precision.py:635-880 so the same command lines resolve to
the same plan:

* at most one of --bf16/--fp16/--fp8/--fp4; default bf16 on bf16-capable CUDA
  else fp32; ``--precision-recipe deepseek_v3`` implies fp8;
* per-module include/exclude patterns (regex or glob) for low-bit compute and
  persistent low-bit params, dtype override rules ``<pattern>=<dtype>``, the
  DeepSeek-V3 high-precision exceptions (embeddings, lm_head, norms, router);
* ``MixedPrecisionController``: autocast, static-then-dynamic loss scale
  (backoff x0.5 on overflow, growth x2 every N good steps) with a world-wide
  MIN reduction of the local finite flag.

B200 additions: the fp8 backend may be ``native`` (real e4m3 + block scales
on sm_100a kernels) and the fp4 backend ``native`` (NVFP4 numerics); the
finite check and unscale run as one fused multi-tensor kernel on the flat
gradient buffers.
"""
from __future__ import annotations

import fnmatch
import re
from contextlib import contextmanager, nullcontext
from dataclasses import replace
from typing import Iterable, Iterator, Optional

import torch
import torch.distributed as dist

from ..runtime.contracts import (DeepSeekV3PrecisionRecipe, ModulePrecisionAssignment, ModulePrecisionInitState,
                                 ModulePrecisionPolicy, ModulePrecisionSummary, PrecisionConfig,
                                 PrecisionRuntimeState)
from .backends import build_lowbit_backend_for_mode

_DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
_LOWBIT_CAPABLE = {"linear", "column_parallel_linear", "row_parallel_linear"}


def dtype_alias_to_torch(alias: str) -> torch.dtype:
    try:
        return _DTYPES[alias]
    except KeyError as exc:
        raise ValueError(f"Unsupported precision dtype alias: {alias}") from exc


def _bf16_cuda(device: torch.device) -> bool:
    return device.type == "cuda" and torch.cuda.is_available() and torch.cuda.is_bf16_supported()


def _default_mode_for_device(device: torch.device) -> str:
    return "bf16" if _bf16_cuda(device) else "fp32"


def _resolve_mode_from_flags(args) -> Optional[str]:
    chosen = [m for m in ("bf16", "fp16", "fp8", "fp4") if bool(getattr(args, m, False))]
    if len(chosen) > 1:
        raise ValueError("At most one of --bf16/--fp16/--fp8/--fp4 may be set")
    return chosen[0] if chosen else None


def _default_low_dtype(mode: str, device: torch.device) -> str:
    if mode in ("bf16", "fp16"):
        return mode
    if mode in ("fp8", "fp4"):
        if _bf16_cuda(device):
            return "bf16"
        return "fp16" if device.type == "cuda" else "fp32"
    return "fp32"


def _iter_patterns(value) -> tuple[str, ...]:
    if value is None:
        return ()
    if isinstance(value, str):
        return (value.strip(),) if value.strip() else ()
    if isinstance(value, Iterable):
        return tuple(str(v).strip() for v in value if str(v).strip())
    s = str(value).strip()
    return (s,) if s else ()


def _one_of(raw, allowed, default, message):
    value = str(raw if raw is not None else default)
    if value not in allowed:
        raise ValueError(message)
    return value


def _parse_dtype_rules(raw) -> tuple[tuple[str, str], ...]:
    out = []
    for rule in _iter_patterns(raw):
        if "=" not in rule:
            raise ValueError("--module-compute-dtype-rule must use '<pattern>=<fp32|bf16|fp16>' format")
        pattern, dt = (x.strip() for x in rule.split("=", 1))
        if not pattern:
            raise ValueError("--module-compute-dtype-rule pattern cannot be empty")
        if dt not in _DTYPES:
            raise ValueError("--module-compute-dtype-rule dtype must be one of fp32, bf16, fp16")
        out.append((pattern, dt))
    return tuple(out)


def _granularity(raw, flag: str) -> str:
    v = str(raw)
    if v not in ("tensor", "channel", "tile_1x128", "block_128x128"):
        raise ValueError(f"{flag} must be one of tensor, channel, tile_1x128, block_128x128")
    return v


def default_deepseek_v3_recipe() -> DeepSeekV3PrecisionRecipe:
    """1x128 activation tiles, 128x128 weight blocks, stochastic rounding, fp8 MoE payloads;
    embeddings, LM head, norms and the router stay in high precision."""
    return DeepSeekV3PrecisionRecipe(
        activation_quant_granularity="tile_1x128", weight_quant_granularity="block_128x128",
        rounding_mode="stochastic", comm_quant_enabled=True, comm_quant_granularity="block_128x128",
        high_precision_module_patterns=(r"(^|\.)token_embeddings$", r"(^|\.)position_embeddings$",
                                        r"(^|\.)lm_head$", r"(^|\.)final_norm$", r"(^|\.).*norm$",
                                        r"(^|\.).*router(\.|$)"),
        high_precision_grad_patterns=(r"(^|\.)lm_head(\.|$)", r"(^|\.).*router(\.|$)"))


_default_deepseek_v3_recipe = default_deepseek_v3_recipe


def _recipe_from_args(args) -> DeepSeekV3PrecisionRecipe:
    d = default_deepseek_v3_recipe()
    act = getattr(args, "fp8_activation_granularity", None)
    wgt = getattr(args, "fp8_weight_granularity", None)
    rnd = getattr(args, "fp8_rounding", None)
    cq = getattr(args, "fp8_comm_quant", None)
    cg = getattr(args, "fp8_comm_granularity", None)
    if rnd is not None and str(rnd) not in ("nearest", "stochastic"):
        raise ValueError("--fp8-rounding must be nearest or stochastic")
    return replace(
        d,
        activation_quant_granularity=_granularity(act, "--fp8-activation-granularity") if act is not None
        else d.activation_quant_granularity,
        weight_quant_granularity=_granularity(wgt, "--fp8-weight-granularity") if wgt is not None
        else d.weight_quant_granularity,
        rounding_mode=str(rnd) if rnd is not None else d.rounding_mode,
        comm_quant_enabled=bool(cq) if cq is not None else d.comm_quant_enabled,
        comm_quant_granularity=_granularity(cg, "--fp8-comm-granularity") if cg is not None
        else d.comm_quant_granularity)


def resolve_module_precision_policy(args, precision_config: PrecisionConfig) -> ModulePrecisionPolicy:
    pattern_type = _one_of(getattr(args, "module_pattern_type", "regex"), ("regex", "glob"), "regex",
                           "--module-pattern-type must be regex or glob")
    raw_mode = getattr(args, "compute_lowbit_mode", None)
    explicit = None if raw_mode in (None, "", "none", "off") else str(raw_mode)
    if explicit is not None and explicit not in ("fp8", "fp4"):
        raise ValueError("--compute-lowbit-mode must be fp8 or fp4")
    compute_mode = precision_config.mode if (explicit is None and precision_config.mode in ("fp8", "fp4")) else explicit
    fp8_param = bool(getattr(args, "fp8_param", False))
    fp4_param = bool(getattr(args, "fp4_param", False))
    if fp8_param and fp4_param:
        raise ValueError("At most one of --fp8-param/--fp4-param may be set")
    raw_p = getattr(args, "persistent_lowbit_mode", None)
    pflag = "off" if raw_p in (None, "", "none") else str(raw_p)
    if pflag not in ("off", "fp8", "fp4"):
        raise ValueError("--persistent-lowbit-mode must be off, fp8, or fp4")
    if pflag == "off":
        persistent = "fp8" if fp8_param else ("fp4" if fp4_param else "off")
    else:
        if fp8_param and pflag != "fp8":
            raise ValueError("--fp8-param conflicts with --persistent-lowbit-mode")
        if fp4_param and pflag != "fp4":
            raise ValueError("--fp4-param conflicts with --persistent-lowbit-mode")
        persistent = pflag
    return ModulePrecisionPolicy(
        pattern_type=pattern_type, compute_lowbit_mode=compute_mode,
        compute_lowbit_include=_iter_patterns(getattr(args, "compute_lowbit_include", None)),
        compute_lowbit_exclude=_iter_patterns(getattr(args, "compute_lowbit_exclude", None)),
        persistent_lowbit_mode=persistent,
        persistent_lowbit_include=_iter_patterns(getattr(args, "persistent_lowbit_include", None)),
        persistent_lowbit_exclude=_iter_patterns(getattr(args, "persistent_lowbit_exclude", None)),
        persistent_scale_granularity=_one_of(getattr(args, "persistent_scale_granularity", "per_channel"),
                                             ("per_tensor", "per_channel"), "per_channel",
                                             "--persistent-scale-granularity must be per_tensor or per_channel"),
        fp4_persistent_format=_one_of(getattr(args, "fp4_param_format", "nf4"), ("nf4",), "nf4",
                                      "--fp4-param-format currently supports only nf4"),
        module_compute_dtype_rules=_iter_patterns(getattr(args, "module_compute_dtype_rule", None)))


def _match(name: str, pattern: str, pattern_type: str) -> bool:
    return re.search(pattern, name) is not None if pattern_type == "regex" else fnmatch.fnmatch(name, pattern)


class ModulePrecisionResolverImpl:
    """Resolves each module's precision at construction time from one run policy."""

    def __init__(self, config: PrecisionConfig) -> None:
        self._config = replace(config)
        self._policy = config.module_precision_policy or ModulePrecisionPolicy()
        self._dtype_rules = _parse_dtype_rules(self._policy.module_compute_dtype_rules)
        self._seen: set[str] = set()
        self._compute_hits: set[str] = set()
        self._persistent_hits: set[str] = set()
        self._hp_hits: set[str] = set()
        self._rule_hits: set[tuple[str, str]] = set()
        self._counts = dict(param=0, capable=0, compute=0, persistent=0, hp=0)
        self.assignments: dict[str, ModulePrecisionAssignment] = {}

    def _select(self, path, include, exclude, default_all):
        pt = self._policy.pattern_type
        hit = False
        if include:
            hit = any(_match(path, p, pt) for p in include)
            sel = hit
        else:
            sel = default_all
        if sel and any(_match(path, p, pt) for p in exclude):
            sel = False
        return sel, hit

    def resolve_module_init_state(self, *, module_path: str, module_type: str, lowbit_capable_type=None,
                                  kernel_spec=None) -> ModulePrecisionInitState:
        if not module_path:
            raise ValueError("module_path must be non-empty for precision resolution")
        if module_path in self._seen:
            raise ValueError(f"Duplicate module_path for precision resolution: {module_path}")
        self._seen.add(module_path)
        self._counts["param"] += 1
        capable = lowbit_capable_type in _LOWBIT_CAPABLE
        if capable:
            self._counts["capable"] += 1
        pol = self._policy
        c_sel, c_hit = self._select(module_path, pol.compute_lowbit_include, pol.compute_lowbit_exclude,
                                    pol.compute_lowbit_mode is not None and capable)
        if c_hit:
            self._compute_hits.add(module_path)
        p_sel, p_hit = self._select(module_path, pol.persistent_lowbit_include, pol.persistent_lowbit_exclude,
                                    pol.persistent_lowbit_mode != "off" and capable)
        if p_hit:
            self._persistent_hits.add(module_path)
        if c_sel and not capable and pol.compute_lowbit_mode is not None:
            raise ValueError("compute_lowbit patterns matched modules without low-bit support: "
                             f"{module_path} ({module_type})")
        if p_sel and not capable and pol.persistent_lowbit_mode != "off":
            raise ValueError("persistent_lowbit patterns matched modules without low-bit support: "
                             f"{module_path} ({module_type})")
        compute_mode = pol.compute_lowbit_mode if (capable and c_sel) else None
        persistent = pol.persistent_lowbit_mode if (capable and p_sel) else "off"
        recipe = self._config.deepseek_v3_recipe
        if recipe is not None and recipe.high_precision_module_patterns and any(
                re.search(p, module_path) for p in recipe.high_precision_module_patterns):
            self._hp_hits.add(module_path)
            self._counts["hp"] += 1
            compute_mode, persistent = None, "off"
        override = None
        for pattern, dt in self._dtype_rules:
            if _match(module_path, pattern, pol.pattern_type):
                override = dt
                self._rule_hits.add((pattern, dt))
        if compute_mode is not None and override is not None:
            raise ValueError(f"module matched both low-bit compute and compute-dtype override: {module_path}. "
                             "Adjust --compute-lowbit-* or --module-compute-dtype-rule.")
        if compute_mode is not None:
            self._counts["compute"] += 1
        if persistent != "off":
            self._counts["persistent"] += 1
        assignment = ModulePrecisionAssignment(module_name=module_path, module_type=module_type,
                                               compute_lowbit_mode=compute_mode, persistent_lowbit_mode=persistent,
                                               persistent_scale_granularity=pol.persistent_scale_granularity,
                                               fp4_persistent_format=pol.fp4_persistent_format,
                                               compute_dtype_override=override,
                                               master_ownership=self._config.lowbit_master_ownership)
        self.assignments[module_path] = assignment
        backend = None
        if compute_mode is not None:
            spec = kernel_spec
            if spec is not None and recipe is not None:
                spec = replace(spec, activation_quant_granularity=recipe.activation_quant_granularity,
                               weight_quant_granularity=recipe.weight_quant_granularity,
                               rounding_mode=recipe.rounding_mode)
            backend = build_lowbit_backend_for_mode(self._config, mode=compute_mode, kernel_spec=spec)
            if backend is None:
                raise RuntimeError(f"No backend available for compute mode {compute_mode} at module {module_path}")
        return ModulePrecisionInitState(assignment=assignment, lowbit_backend=backend,
                                        lowbit_capable_type=lowbit_capable_type,
                                        master_ownership_mode=self._config.lowbit_master_ownership)

    def finalize(self) -> ModulePrecisionSummary:
        pol = self._policy
        if pol.compute_lowbit_include and not self._compute_hits:
            raise ValueError("compute_lowbit include patterns matched zero modules")
        if pol.persistent_lowbit_include and not self._persistent_hits:
            raise ValueError("persistent_lowbit include patterns matched zero modules")
        unmatched = [f"{p}={d}" for p, d in self._dtype_rules if (p, d) not in self._rule_hits]
        if unmatched:
            raise ValueError(f"module compute dtype rules matched zero modules: {unmatched[:3]}")
        if self._config.mode in ("fp8", "fp4") and self._counts["compute"] == 0:
            raise RuntimeError(
                f"Low-bit mode '{self._config.mode}' is active but zero modules were assigned for low-bit compute. "
                "Check --compute-lowbit-include/--compute-lowbit-exclude or verify the model uses low-bit-capable "
                "layers.")
        recipe = self._config.deepseek_v3_recipe
        if recipe is not None and recipe.high_precision_module_patterns and not self._hp_hits:
            raise ValueError("DeepSeek-V3 high_precision_module_patterns matched zero modules")
        c = self._counts
        return ModulePrecisionSummary(parameterized_module_count=c["param"], lowbit_capable_module_count=c["capable"],
                                      compute_lowbit_module_count=c["compute"],
                                      persistent_lowbit_module_count=c["persistent"],
                                      high_precision_exception_module_count=c["hp"])

    def deepseek_v3_recipe(self) -> Optional[DeepSeekV3PrecisionRecipe]:
        return self._config.deepseek_v3_recipe


_ModulePrecisionResolverImpl = ModulePrecisionResolverImpl


def build_module_precision_resolver(config: PrecisionConfig) -> ModulePrecisionResolverImpl:
    return ModulePrecisionResolverImpl(config)


def finalize_module_precision_resolver(resolver) -> ModulePrecisionSummary:
    return resolver.finalize()


def refresh_persistent_lowbit_params(model: torch.nn.Module) -> int:
    n = 0
    for m in model.modules():
        fn = getattr(m, "refresh_persistent_lowbit_params", None)
        if callable(fn):
            fn()
            n += 1
    return n


def resolve_precision_config(args, device: torch.device) -> PrecisionConfig:
    """PrecisionConfig from Megatron-style precision flags and the run device."""
    recipe_name = _one_of(getattr(args, "precision_recipe", "default"), ("default", "deepseek_v3"), "default",
                          "--precision-recipe must be default or deepseek_v3")
    explicit = _resolve_mode_from_flags(args)
    if recipe_name == "deepseek_v3":
        if explicit not in (None, "fp8"):
            raise ValueError("--precision-recipe deepseek_v3 requires --fp8 (or no explicit mode)")
        mode = "fp8"
    else:
        mode = explicit or _default_mode_for_device(device)
    recipe = _recipe_from_args(args) if recipe_name == "deepseek_v3" else None
    if mode == "bf16":
        if device.type != "cuda":
            raise ValueError("--bf16 requires CUDA")
        if not torch.cuda.is_bf16_supported():
            raise ValueError("--bf16 requires torch.cuda.is_bf16_supported()")
    if mode == "fp16" and device.type != "cuda":
        raise ValueError("--fp16 requires CUDA")
    fp8_backend = str(getattr(args, "fp8_backend", "transformer_engine"))
    fp8_format = str(getattr(args, "fp8_format", "e4m3"))
    hist = int(getattr(args, "fp8_amax_history_len", 16))
    algo = str(getattr(args, "fp8_amax_compute_algo", "most_recent"))
    fp4_backend = str(getattr(args, "fp4_backend", "emulated"))
    ownership = str(getattr(args, "lowbit_master_ownership", "optimizer"))
    if mode == "fp8" and fp8_backend not in ("transformer_engine", "emulated", "native"):
        raise ValueError("--fp8-backend must be transformer_engine or emulated")
    if mode == "fp8" and fp8_format not in ("e4m3", "hybrid"):
        raise ValueError("--fp8-format must be e4m3 or hybrid")
    if mode == "fp8" and algo not in ("most_recent", "max"):
        raise ValueError("--fp8-amax-compute-algo must be most_recent or max")
    if mode == "fp8" and hist < 1:
        raise ValueError("--fp8-amax-history-len must be >= 1")
    if mode == "fp4" and fp4_backend not in ("emulated", "native"):
        raise ValueError("--fp4-backend must be emulated or native")
    if ownership not in ("module", "optimizer"):
        raise ValueError("--lowbit-master-ownership must be module or optimizer")
    dts = {
        "params_dtype": getattr(args, "params_dtype", None) or _default_low_dtype(mode, device),
        "main_params_dtype": getattr(args, "main_params_dtype", None) or "fp32",
        "main_grads_dtype": getattr(args, "main_grads_dtype", None) or "fp32",
        "exp_avg_dtype": getattr(args, "exp_avg_dtype", None) or "fp32",
        "exp_avg_sq_dtype": getattr(args, "exp_avg_sq_dtype", None) or "fp32",
    }
    for k, v in dts.items():
        if v not in _DTYPES:
            raise ValueError(f"--{k.replace('_', '-')} must be fp32, bf16, or fp16")
    interval = int(getattr(args, "loss_scale_growth_interval", 2000))
    if interval < 1:
        raise ValueError("--loss-scale-growth-interval must be >= 1")
    cfg = PrecisionConfig(
        mode=mode, activation_dtype=_default_low_dtype(mode, device), fp8_backend=fp8_backend,
        fp8_format=fp8_format, fp8_amax_history_len=hist, fp8_amax_compute_algo=algo, fp4_backend=fp4_backend,
        fp8_param=bool(getattr(args, "fp8_param", False)), fp4_param=bool(getattr(args, "fp4_param", False)),
        fp4_param_format=_one_of(getattr(args, "fp4_param_format", "nf4"), ("nf4",), "nf4",
                                 "--fp4-param-format currently supports only nf4"),
        persistent_scale_granularity=_one_of(getattr(args, "persistent_scale_granularity", "per_channel"),
                                             ("per_tensor", "per_channel"), "per_channel",
                                             "--persistent-scale-granularity must be per_tensor or per_channel"),
        lowbit_master_ownership=ownership, precision_recipe_name=recipe_name, deepseek_v3_recipe=recipe,
        loss_scale_init=float(getattr(args, "loss_scale_init", 65536.0)),
        loss_scale_growth_factor=float(getattr(args, "loss_scale_growth_factor", 2.0)),
        loss_scale_backoff_factor=float(getattr(args, "loss_scale_backoff_factor", 0.5)),
        loss_scale_growth_interval=interval, loss_scale_min=float(getattr(args, "loss_scale_min", 1.0)),
        loss_scale_max=float(getattr(args, "loss_scale_max", 16777216.0)), **dts)
    if cfg.loss_scale_init <= 0:
        raise ValueError("--loss-scale-init must be > 0")
    if cfg.loss_scale_growth_factor <= 1.0:
        raise ValueError("--loss-scale-growth-factor must be > 1")
    if not (0.0 < cfg.loss_scale_backoff_factor < 1.0):
        raise ValueError("--loss-scale-backoff-factor must be in (0, 1)")
    if cfg.loss_scale_min <= 0.0:
        raise ValueError("--loss-scale-min must be > 0")
    if cfg.loss_scale_max < cfg.loss_scale_min:
        raise ValueError("--loss-scale-max must be >= --loss-scale-min")
    cfg.module_precision_policy = resolve_module_precision_policy(args, cfg)
    modes = set()
    if cfg.mode in ("fp8", "fp4"):
        modes.add(cfg.mode)
    if cfg.module_precision_policy.compute_lowbit_mode is not None:
        modes.add(cfg.module_precision_policy.compute_lowbit_mode)
    for m in modes:
        build_lowbit_backend_for_mode(cfg, mode=m, kernel_spec=None)
    return cfg


class MixedPrecisionController:
    """Autocast + dynamic loss scaling with a skip-step on non-finite gradients."""

    def __init__(self, config: PrecisionConfig, *, device: torch.device) -> None:
        self.config = replace(config)
        self.device = device
        self.runtime_state = PrecisionRuntimeState(loss_scale=float(config.loss_scale_init))

    @property
    def uses_loss_scaling(self) -> bool:
        return self.config.mode in ("fp16", "fp8", "fp4")

    def activation_torch_dtype(self) -> torch.dtype:
        return dtype_alias_to_torch(self.config.activation_dtype)

    @contextmanager
    def autocast_context(self) -> Iterator[None]:
        dt = self.activation_torch_dtype()
        if dt == torch.float32:
            ctx = nullcontext()
        elif self.device.type == "cuda":
            ctx = torch.autocast(device_type="cuda", dtype=dt)
        elif self.device.type == "cpu" and dt == torch.bfloat16:
            ctx = torch.autocast(device_type="cpu", dtype=dt)
        else:
            ctx = nullcontext()
        with ctx:
            yield

    def backward(self, loss: torch.Tensor) -> None:
        if self.uses_loss_scaling:
            (loss * float(self.runtime_state.loss_scale)).backward()
        else:
            loss.backward()

    def _grads(self, model):
        for p in model.parameters():
            g = p.grad if p.grad is not None else getattr(p, "main_grad", None)
            if g is not None:
                yield g

    def prepare_optimizer_step(self, model: torch.nn.Module) -> bool:
        """Unscale gradients; return False (skip the step) if any rank saw inf/nan."""
        from ..ops.optim import grad_stats_

        inv = None
        if self.uses_loss_scaling and self.runtime_state.loss_scale != 1.0:
            inv = 1.0 / float(self.runtime_state.loss_scale)
        stats = torch.zeros(2, dtype=torch.float32, device=self.device)
        inv_t = torch.tensor([inv], dtype=torch.float32, device=self.device) if inv is not None else None
        for g in self._grads(model):
            if g.is_cuda and g.is_contiguous():
                grad_stats_(g, stats, inv_t)
            else:
                if inv is not None:
                    g.mul_(inv)
                if not bool(torch.isfinite(g).all()):
                    stats[1] = 1.0
        finite = torch.tensor([0 if float(stats[1]) else 1], dtype=torch.int32, device=self.device)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(finite, op=dist.ReduceOp.MIN)
        ok = bool(int(finite.item()) == 1)
        if not ok:
            self.runtime_state.found_inf_steps += 1
            self.runtime_state.skipped_steps += 1
        return ok

    def update_after_step(self, *, step_applied: bool) -> None:
        if not self.uses_loss_scaling:
            return
        st = self.runtime_state
        if not step_applied:
            st.loss_scale = max(float(self.config.loss_scale_min), st.loss_scale * float(self.config.loss_scale_backoff_factor))
            st.growth_tracker = 0
            return
        st.growth_tracker += 1
        if st.growth_tracker < int(self.config.loss_scale_growth_interval):
            return
        st.loss_scale = min(float(self.config.loss_scale_max), st.loss_scale * float(self.config.loss_scale_growth_factor))
        st.growth_tracker = 0
