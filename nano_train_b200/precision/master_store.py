"""Optimizer-owned master weights for persistent low-bit layers.

With persistent low-bit parameters and ``lowbit_master_ownership == "optimizer"``, a layer's
trainable high-precision weight moves out of the layer into one store module on the model
(``model._lowbit_master_store``); the layer is re-pointed at it (its ``bind_optimizer_master_weight``
hook) and refreshes its low-bit copy from it after every optimizer step. So the optimizer, the
gradient synchronisation and checkpoints see one master per layer, in one place.

How the store is built: ``_lowbit_layers`` walks the model once and yields the layers whose
precision assignment asks for a persistent low-bit copy and that can be re-bound; the store
``adopt``s each one (copy of the current weight, binding, metadata). The metadata records which
parallel domain shards the master, asked of the layer itself: a tensor-parallel linear with
``tp_size > 1`` is tensor-sharded, a layer under an ``experts`` container is expert-sharded, all
others are replicated over data parallelism. ``parallel/sync.py`` reads it to route gradients.

State-dict interface (kept as the reference writes it, src/runtime/master_store.py:18-119, so
checkpoints carry over): ``_lowbit_master_store.masters.<path with '.' -> '__'>__weight`` and the
metadata fields ``module_path``, ``parameter_name``, ``shard_domain``, ``shape``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Optional

import torch.nn as nn

STORE_ATTR = "_lowbit_master_store"
TENSOR, EXPERT, DATA = "tensor_model_parallel", "expert_model_parallel", "data_parallel"


@dataclass(frozen=True)
class MasterBindingMetadata:
    module_path: str
    parameter_name: str
    shard_domain: str
    shape: tuple[int, ...]


def master_key(module_path: str, parameter_name: str = "weight") -> str:
    """Key of a master in the store's ParameterDict (dots are not allowed in its keys)."""
    return "__".join(module_path.split(".") + [parameter_name])


def shard_domain(module: nn.Module, module_path: str) -> str:
    if getattr(module, "tp_size", 1) > 1 and hasattr(module, "tp_group"):
        return TENSOR
    if "experts" in module_path.split(".")[:-1]:
        return EXPERT
    return DATA


class LowBitMasterStore(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.masters = nn.ParameterDict()
        self.metadata: dict[str, MasterBindingMetadata] = {}

    def add_master(self, *, key: str, param: nn.Parameter, metadata: MasterBindingMetadata) -> nn.Parameter:
        self.masters[key] = param
        self.metadata[key] = metadata
        return self.masters[key]

    def adopt(self, module: nn.Module, module_path: str) -> nn.Parameter:
        """Take over ``module.weight``: store a copy as the master and re-point the module at it."""
        w = module.weight
        meta = MasterBindingMetadata(module_path=module_path, parameter_name="weight",
                                     shard_domain=shard_domain(module, module_path), shape=tuple(w.shape))
        master = self.add_master(key=master_key(module_path), param=nn.Parameter(w.detach().clone()), metadata=meta)
        module.bind_optimizer_master_weight(master)
        return master

    def params_in(self, domain: str) -> Iterator[nn.Parameter]:
        for key, meta in self.metadata.items():
            if meta.shard_domain == domain and key in self.masters:
                yield self.masters[key]


def _lowbit_layers(model: nn.Module) -> Iterator[tuple[str, nn.Module]]:
    """(module path, layer) of every layer with a persistent low-bit copy that can be re-bound."""
    for module in model.modules():
        assignment = getattr(module, "module_precision_assignment", None)
        if assignment is None or getattr(assignment, "persistent_lowbit_mode", "off") == "off":
            continue
        if not callable(getattr(module, "bind_optimizer_master_weight", None)):
            continue
        if not isinstance(getattr(module, "weight", None), nn.Parameter):
            continue
        path = str(getattr(module, "module_path", "") or getattr(assignment, "module_name", ""))
        if path:
            yield path, module


def materialize_optimizer_owned_masters(model: nn.Module, *, precision_config) -> Optional[LowBitMasterStore]:
    """Build and attach the store when the optimizer owns the masters; None when it does not, or
    when no layer has a persistent low-bit copy."""
    if precision_config.lowbit_master_ownership != "optimizer":
        return None
    store = LowBitMasterStore()
    for path, layer in list(_lowbit_layers(model)):
        store.adopt(layer, path)
    if not store.masters:
        return None
    model.add_module(STORE_ATTR, store)
    return store


def get_lowbit_master_store(model: nn.Module) -> Optional[LowBitMasterStore]:
    s = getattr(model, STORE_ATTR, None)
    return s if isinstance(s, LowBitMasterStore) else None
