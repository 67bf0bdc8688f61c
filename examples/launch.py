"""Launch a training script on N local processes (reference: examples/launch.py).

    python examples/launch.py --world-size 4 --backend gloo --script examples/train_4d.py --script-args ...
    python examples/launch.py --dry-run --script examples/train_ddp.py

Without ``--world-size`` the number of devices is auto-detected. With
``--dry-run`` the equivalent ``torchrun`` command is printed instead.
Inside an existing torchrun job the script is run directly.
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.distributed.device import get_device_info  # noqa: E402
from nano_train_b200.distributed.launch import get_launch_command, launch_multiprocessing  # noqa: E402


def main():
    ap = argparse.ArgumentParser(description="Launch distributed training")
    ap.add_argument("--world-size", type=int, default=None)
    ap.add_argument("--backend", choices=["auto", "gloo", "nccl"], default="auto")
    ap.add_argument("--script", default="examples/train_ddp.py")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--script-args", nargs=argparse.REMAINDER, default=[])
    a = ap.parse_args()
    info = get_device_info(a.world_size)
    if a.dry_run:
        print(get_launch_command(info, a.script, a.script_args))
        return
    if "RANK" in os.environ and "WORLD_SIZE" in os.environ:
        sys.argv = [a.script] + list(a.script_args)
        with open(a.script) as f:
            code = compile(f.read(), a.script, "exec")
        exec(code, {"__name__": "__main__", "__file__": a.script})
        return
    backend = info.backend if a.backend == "auto" else a.backend
    launch_multiprocessing(a.script, info.world_size if a.world_size is None else a.world_size, backend,
                           list(a.script_args))


if __name__ == "__main__":
    main()
