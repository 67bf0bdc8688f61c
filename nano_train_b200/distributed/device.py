"""Device and backend selection (reference: src/distributed/device.py:22-209).

NCCL on CUDA machines, gloo otherwise; ``cuda:{local_rank}`` placement.
"""
from __future__ import annotations

import os
import warnings
from dataclasses import dataclass
from typing import Literal, Optional

import torch


@dataclass
class DeviceInfo:
    device_type: Literal["cpu", "cuda"]
    device_count: int
    backend: Literal["gloo", "nccl"]
    world_size: int


def get_device_info(world_size: Optional[int] = None,
                    backend: Optional[Literal["gloo", "nccl", "auto"]] = None) -> DeviceInfo:
    """Detected device type/count and the backend to use (CPU: one process per core)."""
    cuda = torch.cuda.is_available()
    device_type: Literal["cpu", "cuda"] = "cuda" if cuda else "cpu"
    count = torch.cuda.device_count() if cuda else (os.cpu_count() or 1)
    if backend in (None, "auto"):
        backend = "nccl" if cuda else "gloo"
    elif backend == "nccl" and not cuda:
        raise RuntimeError("Requested 'nccl' backend but CUDA is not available. "
                           "Use backend='gloo' for CPU distributed training.")
    elif backend == "gloo" and cuda:
        warnings.warn("Using 'gloo' backend with CUDA available. Consider using 'nccl' for better performance on GPUs.",
                      UserWarning)
    return DeviceInfo(device_type=device_type, device_count=count, backend=backend,
                      world_size=count if world_size is None else world_size)


def get_device(device_type: Literal["cpu", "cuda"], rank: int = 0) -> torch.device:
    if device_type == "cpu":
        return torch.device("cpu")
    if device_type == "cuda":
        return torch.device(f"cuda:{rank}")
    raise ValueError(f"Unknown device type: {device_type}")


def get_backend(backend: Optional[Literal["gloo", "nccl", "auto"]] = None) -> Literal["gloo", "nccl"]:
    if backend in (None, "auto"):
        forced = os.environ.get("NTB_BACKEND")
        if forced in ("gloo", "nccl"):
            return forced  # type: ignore[return-value]
        return "nccl" if torch.cuda.is_available() else "gloo"
    if backend not in ("gloo", "nccl"):
        raise ValueError(f"Unknown backend: {backend}")
    if backend == "nccl" and not torch.cuda.is_available():
        raise RuntimeError("Requested 'nccl' backend but CUDA is not available. "
                           "Use backend='gloo' for CPU distributed training.")
    return backend


def validate_world_size(world_size: int, available_devices: int) -> None:
    if world_size > available_devices:
        raise ValueError(f"Requested world_size={world_size} but only {available_devices} devices are available")
    if world_size <= 0:
        raise ValueError(f"world_size must be positive, got {world_size}")


def print_device_info(info: DeviceInfo) -> None:
    print("=" * 60)
    print("Device Information")
    print("=" * 60)
    print(f"Device type:  {info.device_type}")
    print(f"Device count: {info.device_count}")
    print(f"Backend:      {info.backend}")
    print(f"World size:   {info.world_size}")
    print("=" * 60)
