"""Logging setup: coloured console + optional file handler, rank-aware levels
(reference: src/logging.py:19-161)."""
from __future__ import annotations

import logging
import os
import sys
from typing import Optional

_COLORS = {"DEBUG": "\033[36m", "INFO": "\033[32m", "WARNING": "\033[33m", "ERROR": "\033[31m",
           "CRITICAL": "\033[35m"}
_RESET = "\033[0m"
_ROOT = "nano_train_b200"


class ColoredFormatter(logging.Formatter):
    def __init__(self, fmt: Optional[str] = None, datefmt: Optional[str] = None, use_colors: bool = True):
        super().__init__(fmt or "%(asctime)s | %(levelname)-8s | %(name)s | %(message)s", datefmt or "%H:%M:%S")
        self.use_colors = use_colors

    def format(self, record: logging.LogRecord) -> str:
        text = super().format(record)
        if self.use_colors and record.levelname in _COLORS:
            return f"{_COLORS[record.levelname]}{text}{_RESET}"
        return text


def setup_logging(log_level: str = "INFO", log_file: Optional[str] = None, use_colors: bool = True,
                  log_format: Optional[str] = None, *, level: Optional[str] = None) -> logging.Logger:
    """Configure the root logger: colour console handler (when the console is a terminal) and an
    optional plain-text file handler (appending). ``level`` is accepted as an alias of
    ``log_level``. Unknown level names raise ``ValueError``."""
    name = (level or log_level).upper()
    if not isinstance(getattr(logging, name, None), int):
        raise ValueError(f"Unsupported log level: {level or log_level}. "
                         "Expected one of DEBUG, INFO, WARNING, ERROR, CRITICAL.")
    lvl = int(getattr(logging, name))
    fmt = log_format or "%(asctime)s | %(levelname)-8s | %(name)s: %(message)s"
    datefmt = None if log_format else "%Y-%m-%d %H:%M:%S"
    root = logging.getLogger()
    root.setLevel(lvl)
    root.handlers.clear()
    h = logging.StreamHandler(sys.stdout)
    h.setLevel(lvl)
    h.setFormatter(ColoredFormatter(fmt, datefmt=datefmt, use_colors=use_colors and sys.stdout.isatty()))
    root.addHandler(h)
    if log_file:
        os.makedirs(os.path.dirname(os.path.abspath(log_file)), exist_ok=True)
        fh = logging.FileHandler(log_file, mode="a")
        fh.setLevel(lvl)
        fh.setFormatter(logging.Formatter(fmt, datefmt=datefmt))
        root.addHandler(fh)
    pkg = logging.getLogger(_ROOT)  # the package logger propagates to the configured root
    pkg.handlers.clear()
    pkg.setLevel(logging.NOTSET)
    pkg.propagate = True
    return root


def get_logger(name: str) -> logging.Logger:
    if not name.startswith(_ROOT):
        name = f"{_ROOT}.{name}"
    return logging.getLogger(name)


def quick_setup(level: str = "INFO") -> None:
    setup_logging(level=level)


def setup_process_logging(rank: int, level: str = "INFO") -> None:
    """INFO on rank 0, WARNING elsewhere."""
    setup_logging(level=level if rank == 0 else "WARNING")
