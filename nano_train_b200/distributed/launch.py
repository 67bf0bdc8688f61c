"""Local multi-process launcher and the equivalent ``torchrun`` command line.

A job is a ``LaunchConfig`` (script, its arguments, world size, backend). ``launch_multiprocessing``
spawns one process per rank; each gets its rendezvous environment from ``rank_environment`` (a
pure function, so what a rank sees is testable without spawning) and then runs the script as
``__main__`` with ``runpy``, exactly as ``python script.py args...`` would. The rendezvous is
on 127.0.0.1; without ``MASTER_PORT`` in the environment a free port is picked, so two local
jobs do not collide. On GPUs, ``torchrun`` is the launcher of record (one process per GPU, NCCL);
``get_launch_command`` prints its command line.

Public names follow the reference (src/distributed/launch.py:25-277).
"""
from __future__ import annotations

import os
import runpy
import socket
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

import torch.multiprocessing as mp

from .device import DeviceInfo, get_device_info, print_device_info


@dataclass
class LaunchConfig:
    world_size: int
    backend: str
    script_path: str
    script_args: list[str] = field(default_factory=list)
    master_addr: str = "127.0.0.1"
    master_port: Optional[int] = None

    def check(self) -> "LaunchConfig":
        if self.world_size <= 0:
            raise ValueError("world_size must be positive")
        if not Path(self.script_path).is_file():
            raise FileNotFoundError(f"script_path does not exist: {self.script_path}")
        return self


def _free_port(addr: str) -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind((addr, 0))
        return s.getsockname()[1]


def rank_environment(cfg: LaunchConfig, rank: int) -> dict[str, str]:
    """Environment variables that make ``rank`` of the job join its process group."""
    return {
        "RANK": str(rank),
        "LOCAL_RANK": str(rank),
        "WORLD_SIZE": str(cfg.world_size),
        "LOCAL_WORLD_SIZE": str(cfg.world_size),
        "MASTER_ADDR": cfg.master_addr,
        "MASTER_PORT": str(cfg.master_port),
        "NTB_BACKEND": cfg.backend,
    }


def _run_rank(rank: int, cfg: LaunchConfig) -> None:
    os.environ.update(rank_environment(cfg, rank))
    script = os.path.abspath(cfg.script_path)
    sys.path.insert(0, os.path.dirname(script))
    saved = sys.argv
    sys.argv = [script, *cfg.script_args]
    try:
        runpy.run_path(script, run_name="__main__")
    finally:
        sys.argv = saved


def launch(cfg: LaunchConfig) -> None:
    """Run ``cfg`` as ``cfg.world_size`` local processes and wait for all of them."""
    cfg.check()
    if cfg.master_port is None:
        env_port = os.environ.get("MASTER_PORT")
        cfg.master_port = int(env_port) if env_port else _free_port(cfg.master_addr)
    print(f"launch: {cfg.world_size} x {cfg.script_path} {' '.join(cfg.script_args)} "
          f"(backend {cfg.backend}, rendezvous {cfg.master_addr}:{cfg.master_port})")
    mp.start_processes(_run_rank, args=(cfg,), nprocs=cfg.world_size, start_method="spawn")


def launch_multiprocessing(script_path: str, world_size: int, backend: str = "gloo",
                           script_args: Optional[list[str]] = None) -> None:
    launch(LaunchConfig(world_size=world_size, backend=backend, script_path=script_path,
                        script_args=list(script_args or [])))


def get_launch_command(info: DeviceInfo, script_path: str, script_args: Optional[list[str]] = None) -> str:
    tail = " ".join([script_path, *(script_args or [])])
    if info.device_type == "cuda":
        return f"torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node {info.world_size} {tail}"
    extra = f" --script-args {' '.join(script_args)}" if script_args else ""
    return f"python examples/launch.py --world-size {info.world_size} --backend gloo --script {script_path}{extra}"


def print_launch_instructions(info: DeviceInfo, script_path: str) -> None:
    print_device_info(info)
    print("launch with:\n  " + get_launch_command(info, script_path))


def auto_detect_and_print(script_path: str = "examples/train_ddp.py") -> DeviceInfo:
    info = get_device_info()
    print_launch_instructions(info, script_path)
    return info
