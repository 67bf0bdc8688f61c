"""Loader of the compiled sm_100a extension (``nano_train_b200/_C*.so``).

CUDA tensors always go through the extension; if it is missing on a machine
with a GPU the call raises instead of silently falling back to a library
kernel. CPU tensors use the PyTorch reference math of each op (the CPU/gloo
path that the tests and the tiny configs run).
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def ext():
    """Return the compiled extension module or raise a clear error."""
    global _C, _ERR
    if _C is not None:
        return _C
    if _ERR is not None:
        raise RuntimeError(
            "nano_train_b200 CUDA extension is not built; run `python setup.py build_ext --inplace`"
        ) from _ERR
    try:
        _C = importlib.import_module("nano_train_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        raise RuntimeError(
            "nano_train_b200 CUDA extension is not built; run `python setup.py build_ext --inplace`"
        ) from e
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def check_status(device: int = 0) -> None:
    """Raise if a kernel on ``device`` reported a bounded-wait timeout or a bad shape."""
    code = ext().read_and_clear_status(device)
    if code:
        raise KernelStatusError(code)


class KernelStatusError(RuntimeError):
    NAMES = {
        1: "TMA producer wait timed out",
        2: "MMA issuer wait timed out",
        3: "epilogue wait timed out",
        4: "drain wait timed out",
        5: "peer wait timed out",
        6: "bad shape",
        7: "flag wait timed out",
    }

    def __init__(self, code: int):
        self.code = code
        super().__init__(f"kernel status {code}: {self.NAMES.get(code, 'unknown')}")
