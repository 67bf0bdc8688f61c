"""Print detected devices, the backend and the launch command (reference: examples/device_info.py)."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.distributed.device import get_device_info, print_device_info  # noqa: E402
from nano_train_b200.distributed.launch import print_launch_instructions  # noqa: E402

if __name__ == "__main__":
    info = get_device_info()
    print_device_info(info)
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            print(f"  cuda:{i} {p.name} sm_{p.major}{p.minor} {p.multi_processor_count} SMs "
                  f"{p.total_memory / 2**30:.0f} GiB")
    print_launch_instructions(info, "examples/train_ddp.py")
