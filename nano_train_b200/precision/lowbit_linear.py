"""Per-module precision state bound at construction time.

Every parameterised layer asks the precision resolver for its assignment
(compute low-bit mode, persistent low-bit mode, dtype override) using its
``module_path``; linear layers additionally get a low-bit backend object.
Reference parity: src/layers.py:187-458 (_ModulePrecisionStateMixin,
_LowBitPrecisionLinearMixin).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops

_DTYPE_ALIASES = {"fp32": torch.float32, "float32": torch.float32, "bf16": torch.bfloat16,
                  "bfloat16": torch.bfloat16, "fp16": torch.float16, "float16": torch.float16}


def resolve_compute_torch_dtype(alias: str) -> torch.dtype:
    try:
        return _DTYPE_ALIASES[alias]
    except KeyError as e:
        raise ValueError(f"unsupported compute dtype alias: {alias}") from e


class ModulePrecisionStateMixin:
    def _init_module_precision_state(self, *, module_path: str, module_type: str, precision_resolver,
                                     lowbit_capable_type=None, kernel_spec=None) -> None:
        state = precision_resolver.resolve_module_init_state(module_path=module_path, module_type=module_type,
                                                             lowbit_capable_type=lowbit_capable_type,
                                                             kernel_spec=kernel_spec)
        self._module_path = module_path
        self._module_precision_state = state
        self._precision_assignment = getattr(state, "assignment", None)
        self._lowbit_backend = getattr(state, "lowbit_backend", None)

    @property
    def module_precision_assignment(self):
        return self._precision_assignment

    @property
    def module_path(self) -> str:
        return self._module_path

    def _module_compute_dtype_override(self) -> Optional[torch.dtype]:
        a = self._precision_assignment
        alias = getattr(a, "compute_dtype_override", None) if a is not None else None
        return resolve_compute_torch_dtype(alias) if alias else None


class LowBitLinearMixin(ModulePrecisionStateMixin):
    """Linear-layer precision behaviour: low-bit compute dispatch, dtype override,
    persistent low-bit weight copies (refreshed after each optimizer step)."""

    def _init_lowbit_precision_state(self, *, module_path: str, module_type: str, precision_resolver,
                                     lowbit_capable_type: str, in_features: int, out_features: int,
                                     has_bias: bool) -> None:
        from ..runtime.contracts import LowBitKernelSpec

        spec = LowBitKernelSpec(module_type=lowbit_capable_type, in_features=in_features,
                                out_features=out_features, has_bias=has_bias)
        self._init_module_precision_state(module_path=module_path, module_type=module_type,
                                          precision_resolver=precision_resolver,
                                          lowbit_capable_type=lowbit_capable_type, kernel_spec=spec)
        from .persistent import init_persistent_buffers

        init_persistent_buffers(self)
        bind = getattr(self._lowbit_backend, "bind_parameters", None)
        if callable(bind):  # backends that own a kernel module use the layer's trainable parameters
            bind(self.weight, self.bias)

    _PERSISTENT_SUFFIXES = ("_persistent_fp8_weight", "_persistent_fp4_codes", "_persistent_scale",
                            "_persistent_numel")

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        """Checkpoints written without the persistent low-bit buffers still load strictly; the
        buffers are then rebuilt from the loaded weight."""
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)
        optional = {prefix + k for k in self._PERSISTENT_SUFFIXES}
        absent = [k for k in missing_keys if k in optional]
        missing_keys[:] = [k for k in missing_keys if k not in optional]
        if absent and self._persistent_mode() != "off":
            self.refresh_persistent_lowbit_params()

    @property
    def master_ownership_mode(self) -> str:
        a = self._precision_assignment
        return getattr(a, "master_ownership", "module") if a is not None else "module"

    def _persistent_mode(self) -> str:
        a = self._precision_assignment
        return getattr(a, "persistent_lowbit_mode", "off") if a is not None else "off"

    def _persistent_granularity(self) -> str:
        a = self._precision_assignment
        return getattr(a, "persistent_scale_granularity", "per_channel") if a is not None else "per_channel"

    def _compute_lowbit_mode(self) -> Optional[str]:
        a = self._precision_assignment
        return getattr(a, "compute_lowbit_mode", None) if a is not None else None

    def _lowbit_active(self) -> bool:
        return self._lowbit_backend is not None and self._compute_lowbit_mode() in ("fp8", "fp4")

    def bind_optimizer_master_weight(self, master_weight: torch.nn.Parameter) -> None:
        """Make ``self.weight`` the optimizer-owned master parameter (persistent low-bit ownership)."""
        if tuple(master_weight.shape) != tuple(self.weight.shape):
            raise ValueError("master weight shape mismatch")
        self.weight = master_weight
        self.refresh_persistent_lowbit_params()

    def refresh_persistent_lowbit_params(self) -> None:
        from .persistent import refresh_persistent

        refresh_persistent(self)

    def _effective_weight(self) -> torch.Tensor:
        from .persistent import persistent_weight_ste

        if self._persistent_mode() != "off":
            return persistent_weight_ste(self)
        return self.weight

    def _linear(self, x: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
        w = self._effective_weight()
        if self._compute_lowbit_mode() is not None:
            if self._lowbit_backend is None:
                raise RuntimeError(f"Module {type(self).__name__} ({self._module_path}) requested compute mode "
                                   f"{self._compute_lowbit_mode()} without a bound low-bit backend")
            return self._lowbit_backend.linear(x, w, bias)
        dt = self._module_compute_dtype_override()
        if dt is not None:  # the override is the compute and the output dtype
            return ops.linear(x.to(dt), w.to(dt), None if bias is None else bias.to(dt))
        if w.dtype != x.dtype:
            w = w.to(x.dtype)
            bias = None if bias is None else bias.to(x.dtype)
        return ops.linear(x, w, bias)
