"""``import src.<module>`` resolved to this framework's modules.

Code written against the reference imports ``src.layers``, ``src.runtime.pipeline``,
``src.runtime.te_backend`` and so on. Its package tree is not this framework's (the pipeline lives
in ``parallel/``, the precision runtime in ``precision/``, attention and MLP in
``models/transformer.py``), so ``MODULE_MAP`` lists, for every reference module, the module of this
package that provides the same public names. ``install_src_alias()`` puts a finder at the front of
``sys.meta_path`` that answers ``src`` and ``src.*`` imports with those modules: the very same
module objects, so monkeypatching ``src.layers.X`` patches ``nano_train_b200.layers.X``.

Used by ``tests/test_reference_suite_cpu.py`` to run the reference's own test files against this
package, and usable by any script of the reference.
"""
from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import sys
from typing import Optional

_P = "nano_train_b200"

MODULE_MAP: dict[str, str] = {
    "src": _P,
    "src.config": f"{_P}.config",
    "src.dataset": f"{_P}.dataset",
    "src.distributed": f"{_P}.distributed",
    "src.distributed.device": f"{_P}.distributed.device",
    "src.distributed.launch": f"{_P}.distributed.launch",
    "src.distributed.topology": f"{_P}.distributed.topology",
    "src.distributed.zero": f"{_P}.distributed.zero",
    "src.layers": f"{_P}.layers",
    "src.logging": f"{_P}.logging",
    "src.losses": f"{_P}.losses",
    "src.models": f"{_P}.models",
    "src.models.attention": f"{_P}.models.transformer",
    "src.models.mlp": f"{_P}.models.transformer",
    "src.models.deepseek": f"{_P}.models.deepseek",
    "src.models.moe": f"{_P}.models.moe",
    "src.models.transformer": f"{_P}.models.transformer",
    "src.monitoring": f"{_P}.monitoring",
    "src.optimizer": f"{_P}.optimizer",
    "src.runtime": f"{_P}.runtime",
    "src.runtime.checkpoint": f"{_P}.runtime.checkpoint",
    "src.runtime.context": f"{_P}.runtime.context",
    "src.runtime.contracts": f"{_P}.runtime.contracts",
    "src.runtime.engine": f"{_P}.runtime.engine",
    "src.runtime.master_store": f"{_P}.precision.master_store",
    "src.runtime.mixed_precision": f"{_P}.precision.mixed_precision",
    "src.runtime.optimizer_runtime": f"{_P}.runtime.optimizer_runtime",
    "src.runtime.pipeline": f"{_P}.parallel.pipeline",
    "src.runtime.precision_args": f"{_P}.precision.precision_args",
    "src.runtime.schedules": f"{_P}.runtime.schedules",
    "src.runtime.schedules.non_pipeline": f"{_P}.runtime.schedules.non_pipeline",
    "src.runtime.schedules.pipeline_1f1b": f"{_P}.runtime.schedules.pipeline_1f1b",
    "src.runtime.schedules.selector": f"{_P}.runtime.schedules.selector",
    "src.runtime.sync": f"{_P}.parallel.sync",
    "src.runtime.te_backend": f"{_P}.precision.backends",
    "src.runtime.validation": f"{_P}.runtime.validation",
    "src.scheduler": f"{_P}.scheduler",
    "src.trainer": f"{_P}.trainer",
    "src.utils": f"{_P}.utils",
    "src.utils.model_info": f"{_P}.utils.model_info",
}


class _AliasLoader(importlib.abc.Loader):
    """Hands out the already-imported target module. The import machinery stamps the alias spec
    onto the module it gets from ``create_module``; ``exec_module`` puts the module's own spec
    back, so its relative imports, pickling and reloads keep working under both names."""

    def __init__(self, target: str):
        self.target = target
        self._own_spec = None

    def create_module(self, spec):
        module = importlib.import_module(self.target)
        self._own_spec = module.__spec__
        return module

    def exec_module(self, module):
        if self._own_spec is not None:
            module.__spec__ = self._own_spec


class _SrcAliasFinder(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname: str, path, target=None) -> Optional[importlib.machinery.ModuleSpec]:
        dest = MODULE_MAP.get(fullname)
        if dest is None:
            return None
        is_pkg = fullname.count(".") == 0 or fullname in ("src.distributed", "src.models", "src.runtime",
                                                           "src.runtime.schedules", "src.utils")
        spec = importlib.util.spec_from_loader(fullname, _AliasLoader(dest), is_package=is_pkg)
        return spec


_FINDER = _SrcAliasFinder()


def install_src_alias() -> None:
    """Answer ``src`` / ``src.*`` imports with this package (first in ``sys.meta_path``). Modules
    already imported under ``src`` (for example the reference itself) are dropped first."""
    for name in [m for m in sys.modules if m == "src" or m.startswith("src.")]:
        del sys.modules[name]
    if _FINDER not in sys.meta_path:
        sys.meta_path.insert(0, _FINDER)


def uninstall_src_alias() -> None:
    if _FINDER in sys.meta_path:
        sys.meta_path.remove(_FINDER)
    for name in [m for m in sys.modules if m == "src" or m.startswith("src.")]:
        del sys.modules[name]
