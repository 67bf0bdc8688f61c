"""Compatibility with code written against the reference's ``src.*`` import paths."""
from .src_alias import MODULE_MAP, install_src_alias, uninstall_src_alias

__all__ = ["MODULE_MAP", "install_src_alias", "uninstall_src_alias"]
