"""Optimizer-owned master weights for persistent low-bit layers.

When persistent low-bit parameters are enabled with optimizer ownership, the
trainable fp32/bf16 master of each selected layer lives in a store module on
the model (``_lowbit_master_store``), the layer's ``weight`` is rebound to
it, and the low-bit copy is refreshed from it after every step. The shard
domain (tensor / expert / data parallel) is recorded so gradient
synchronisation treats the master like the weight it replaced.

Reference parity: src/runtime/master_store.py:18-119.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch.nn as nn


@dataclass(frozen=True)
class MasterBindingMetadata:
    module_path: str
    parameter_name: str
    shard_domain: str
    shape: tuple[int, ...]


class LowBitMasterStore(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.masters = nn.ParameterDict()
        self.metadata: dict[str, MasterBindingMetadata] = {}

    def add_master(self, *, key: str, param: nn.Parameter, metadata: MasterBindingMetadata) -> nn.Parameter:
        self.masters[key] = param
        self.metadata[key] = metadata
        return self.masters[key]


def _infer_shard_domain(module: nn.Module, module_path: str) -> str:
    from ..layers import ColumnParallelLinear, RowParallelLinear

    if isinstance(module, (ColumnParallelLinear, RowParallelLinear)) and module.tp_size > 1:
        return "tensor_model_parallel"
    if ".experts." in module_path:
        return "expert_model_parallel"
    return "data_parallel"


def materialize_optimizer_owned_masters(model: nn.Module, *, precision_config) -> Optional[LowBitMasterStore]:
    if precision_config.lowbit_master_ownership != "optimizer":
        return None
    store = LowBitMasterStore()
    n = 0
    for _, module in model.named_modules():
        assignment = getattr(module, "module_precision_assignment", None)
        bind = getattr(module, "bind_optimizer_master_weight", None)
        weight = getattr(module, "weight", None)
        if assignment is None or not callable(bind) or not isinstance(weight, nn.Parameter):
            continue
        if getattr(assignment, "persistent_lowbit_mode", "off") == "off":
            continue
        path = str(getattr(module, "module_path", getattr(assignment, "module_name", "")))
        if not path:
            continue
        key = f"{path.replace('.', '__')}__weight"
        bound = store.add_master(key=key, param=nn.Parameter(weight.detach().clone()),
                                 metadata=MasterBindingMetadata(module_path=path, parameter_name="weight",
                                                                shard_domain=_infer_shard_domain(module, path),
                                                                shape=tuple(weight.shape)))
        bind(bound)
        n += 1
    if n == 0:
        return None
    model.add_module("_lowbit_master_store", store)
    return store


def get_lowbit_master_store(model: nn.Module) -> Optional[LowBitMasterStore]:
    s = getattr(model, "_lowbit_master_store", None)
    return s if isinstance(s, LowBitMasterStore) else None
