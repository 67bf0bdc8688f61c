"""pytest plugin (``-p nano_train_b200.compat.pytest_plugin``): installs the ``src.*`` alias
before test modules are collected, so test files written for the reference import this package."""
from .src_alias import install_src_alias

install_src_alias()
