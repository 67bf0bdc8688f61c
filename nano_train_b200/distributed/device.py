"""Where a rank runs and which process-group backend it uses.

``probe()`` takes one snapshot of the machine: CUDA or not, the device count, each device's name
and SM count, and whether every pair of GPUs can reach each other's memory directly (the NVLink /
NVSwitch peer path that the fused tensor-, expert- and data-parallel kernels load and store
through). The backend follows from a small policy table keyed by (requested backend, CUDA
present): NCCL on GPUs, gloo on CPU, an error for NCCL without CUDA, a warning for gloo on GPUs.
``NTB_BACKEND`` (set by the local launcher) overrides an ``auto`` request.

Public names and ``DeviceInfo`` fields are the reference's (src/distributed/device.py:22-209), so
scripts written against it keep working; one process per GPU, placed on ``cuda:<local rank>``.
"""
from __future__ import annotations

import os
import warnings
from dataclasses import dataclass, field
from typing import Literal, Optional

import torch

Backend = Literal["gloo", "nccl"]


@dataclass(frozen=True)
class Platform:
    kind: Literal["cpu", "cuda"]
    count: int  # GPUs, or CPU cores without CUDA
    names: tuple[str, ...] = ()
    sm_counts: tuple[int, ...] = ()
    all_pairs_peer: bool = False  # every GPU pair has direct peer access (NVLink / NVSwitch)


def probe() -> Platform:
    if not torch.cuda.is_available():
        return Platform("cpu", os.cpu_count() or 1)
    n = torch.cuda.device_count()
    props = [torch.cuda.get_device_properties(i) for i in range(n)]
    peer = all(torch.cuda.can_device_access_peer(i, j) for i in range(n) for j in range(n) if i != j)
    return Platform("cuda", n, tuple(p.name for p in props), tuple(p.multi_processor_count for p in props), peer)


def _nccl_without_cuda() -> Backend:
    raise RuntimeError("The 'nccl' backend needs CUDA devices and none are visible; "
                       "use backend='gloo' to run the ranks on CPU.")


def _gloo_on_gpus() -> Backend:
    warnings.warn("Backend 'gloo' selected although CUDA devices are visible; 'nccl' is the GPU backend "
                  "(collectives over NVLink).", UserWarning)
    return "gloo"


# (requested, cuda present) -> backend (or a raise / warn step)
_POLICY = {
    ("auto", True): lambda: "nccl",
    ("auto", False): lambda: "gloo",
    ("nccl", True): lambda: "nccl",
    ("nccl", False): _nccl_without_cuda,
    ("gloo", True): _gloo_on_gpus,
    ("gloo", False): lambda: "gloo",
}


def _resolve(requested: Optional[str], cuda: bool, *, honour_env: bool) -> Backend:
    req = "auto" if requested is None else requested
    if req == "auto" and honour_env and os.environ.get("NTB_BACKEND") in ("gloo", "nccl"):
        req = os.environ["NTB_BACKEND"]
    rule = _POLICY.get((req, cuda))
    if rule is None:
        raise ValueError(f"Unknown backend: {requested}")
    return rule()


@dataclass
class DeviceInfo:
    device_type: Literal["cpu", "cuda"]
    device_count: int
    backend: Backend
    world_size: int
    platform: Optional[Platform] = field(default=None, repr=False, compare=False)


def get_device_info(world_size: Optional[int] = None,
                    backend: Optional[Literal["gloo", "nccl", "auto"]] = None) -> DeviceInfo:
    """The machine snapshot plus the backend to use; world size defaults to one rank per device
    (per core on CPU)."""
    plat = probe()
    chosen = _resolve(backend, plat.kind == "cuda", honour_env=False)
    return DeviceInfo(device_type=plat.kind, device_count=plat.count, backend=chosen,
                      world_size=plat.count if world_size is None else world_size, platform=plat)


def get_backend(backend: Optional[Literal["gloo", "nccl", "auto"]] = None) -> Backend:
    return _resolve(backend, torch.cuda.is_available(), honour_env=True)


def get_device(device_type: Literal["cpu", "cuda"], rank: int = 0) -> torch.device:
    """``cuda:<rank>`` (the caller passes its local rank) or the CPU."""
    if device_type not in ("cpu", "cuda"):
        raise ValueError(f"Unknown device type: {device_type}")
    return torch.device("cpu") if device_type == "cpu" else torch.device("cuda", rank)


def validate_world_size(world_size: int, available_devices: int) -> None:
    if world_size <= 0:
        raise ValueError(f"world_size must be positive, got {world_size}")
    if world_size > available_devices:
        raise ValueError(f"Requested world_size={world_size} but only {available_devices} devices are available")


def describe(info: DeviceInfo) -> list[str]:
    """Human-readable lines for ``info`` (one per fact; GPUs listed with their SM counts)."""
    lines = [f"device type   {info.device_type}", f"device count  {info.device_count}",
             f"backend       {info.backend}", f"world size    {info.world_size}"]
    plat = info.platform
    if plat is not None and plat.kind == "cuda":
        for i, (name, sms) in enumerate(zip(plat.names, plat.sm_counts)):
            lines.append(f"cuda:{i}        {name}, {sms} SMs")
        lines.append(f"peer access   {'all pairs' if plat.all_pairs_peer else 'not between every pair'}")
    return lines


def print_device_info(info: DeviceInfo) -> None:
    print("\n".join(["-- devices --", *describe(info)]))
