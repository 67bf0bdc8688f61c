"""Process launchers (reference: src/distributed/launch.py:25-277).

``launch_multiprocessing`` spawns ``world_size`` local processes (gloo on
CPU, NCCL with one process per GPU), each importing the script as a module
and calling its ``main()`` with RANK / WORLD_SIZE / LOCAL_RANK set and the
script arguments in ``sys.argv``. ``get_launch_command`` prints the
equivalent ``torchrun`` command line.
"""
from __future__ import annotations

import importlib
import os
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import torch.multiprocessing as mp

from .device import DeviceInfo, get_device_info, print_device_info


@dataclass
class LaunchConfig:
    world_size: int
    backend: str
    script_path: str
    script_args: list[str]


def launch_multiprocessing(script_path: str, world_size: int, backend: str = "gloo",
                           script_args: Optional[list[str]] = None) -> None:
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    if not Path(script_path).exists():
        raise FileNotFoundError(f"script_path does not exist: {script_path}")
    script_args = list(script_args or [])
    print(f"Launching {world_size} processes with backend '{backend}'")
    print(f"Script: {script_path}")
    print(f"Args: {script_args}")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    os.environ["NTB_BACKEND"] = backend
    mp.start_processes(_train_worker, args=(world_size, backend, script_path, script_args), nprocs=world_size,
                       start_method="spawn")


def _train_worker(rank: int, world_size: int, backend: str, script_path: str, script_args: list[str]) -> None:
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world_size)
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["LOCAL_WORLD_SIZE"] = str(world_size)
    os.environ["NTB_BACKEND"] = backend
    script_dir = os.path.dirname(os.path.abspath(script_path))
    if script_dir not in sys.path:
        sys.path.insert(0, script_dir)
    module = importlib.import_module(os.path.basename(script_path).replace(".py", ""))
    if not hasattr(module, "main"):
        raise AttributeError(f"Script {script_path} must have a main() function")
    argv = sys.argv
    try:
        sys.argv = [script_path, *script_args]
        module.main()
    finally:
        sys.argv = argv


def get_launch_command(info: DeviceInfo, script_path: str, script_args: Optional[list[str]] = None) -> str:
    args = " ".join(script_args or [])
    if info.device_type == "cuda":
        return (f"torchrun --standalone --nproc_per_node={info.world_size} --master-addr 127.0.0.1 "
                f"{script_path} {args}").strip()
    return (f"python examples/launch.py --world-size {info.world_size} --backend gloo --script {script_path} "
            f"--script-args {args}").strip()


def print_launch_instructions(info: DeviceInfo, script_path: str) -> None:
    print_device_info(info)
    print("Launch with:")
    print("  " + get_launch_command(info, script_path))


def auto_detect_and_print(script_path: str = "examples/train_ddp.py") -> DeviceInfo:
    info = get_device_info()
    print_launch_instructions(info, script_path)
    return info
