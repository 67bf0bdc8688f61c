"""Distributed plumbing: device/backend selection, launchers, topology, ZeRO."""
from .device import DeviceInfo, get_backend, get_device, get_device_info, print_device_info, validate_world_size  # noqa: F401
from .launch import (LaunchConfig, auto_detect_and_print, get_launch_command, launch_multiprocessing,  # noqa: F401
                     print_launch_instructions)
from .topology import (ModelParallelTopology, ParallelSetup4D, coords_from_rank, init_parallel_4d,  # noqa: F401
                       initialize_model_parallel, rank_from_coords)
