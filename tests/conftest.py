"""Shared fixtures and markers.

Tests marked ``gpu`` need a B200 (sm_100a) and the built extension; they are
skipped when CUDA is not available. Everything else runs on CPU, with gloo for
multi-process cases (rendezvous on 127.0.0.1).
"""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Tolerances:
    rtol = 1e-5
    atol = 1e-6


@pytest.fixture
def device():
    return torch.device("cpu")


def assert_tensor_close(a, b, rtol=Tolerances.rtol, atol=Tolerances.atol, msg=""):
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol, msg=msg or None)


def assert_grad_close(a, b, rtol=Tolerances.rtol, atol=Tolerances.atol):
    assert a.grad is not None and b.grad is not None
    torch.testing.assert_close(a.grad, b.grad, rtol=rtol, atol=atol)
