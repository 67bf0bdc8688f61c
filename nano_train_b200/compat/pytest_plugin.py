"""pytest plugin (``-p nano_train_b200.compat.pytest_plugin``): installs the ``src.*`` alias
before test modules are collected, so test files written for the reference import this package.

It also seeds torch's and Python's generators before every test (seed 0). Some of the reference's
tests draw unseeded random inputs and compare a statistic with a bound that sits close to the
statistic's typical value (the cross-entropy of standard-normal logits against log(num_classes) + 0.5
in tests/test_losses.py), so without a fixed seed their outcome would depend on which tests ran
before them."""
import random

import pytest
import torch

from .src_alias import install_src_alias

install_src_alias()


@pytest.fixture(autouse=True)
def _ntb_seed_each_test():
    random.seed(0)
    torch.manual_seed(0)
    yield
