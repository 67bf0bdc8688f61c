"""Section layout of a symmetric-memory region, with canary words after every section.

Each section starts 256-byte aligned and is followed by 256 bytes filled with
a fixed pattern. ``check`` (a host read, so a synchronisation; meant for tests
and debugging) names every section whose canary changed, i.e. a kernel that
wrote past the end of that section (its own or a peer's write into this
rank's memory).
"""
from __future__ import annotations

import torch

CANARY_BYTES = 256
PATTERN = 0xA5


def align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class RegionLayout:
    def __init__(self, start: int = 4096):
        self.off = align(start)
        self.sections: dict[str, tuple[int, int]] = {}
        self.canaries: list[tuple[str, int]] = []

    def add(self, name: str, nbytes: int) -> int:
        off = self.off
        self.sections[name] = (off, nbytes)
        c = align(off + nbytes)
        self.canaries.append((name, c))
        self.off = c + CANARY_BYTES
        return off

    @property
    def total(self) -> int:
        return self.off

    def _views(self, C, local_ptr: int, device_index: int):
        for name, c in self.canaries:
            yield name, C.symm_local_view(local_ptr, c, [CANARY_BYTES], torch.uint8, device_index)

    def fill(self, C, local_ptr: int, device_index: int) -> None:
        for _, v in self._views(C, local_ptr, device_index):
            v.fill_(PATTERN)

    def check(self, C, local_ptr: int, device_index: int) -> list[str]:
        bad = []
        for name, v in self._views(C, local_ptr, device_index):
            if not bool(torch.all(v == PATTERN)):
                bad.append(name)
        return bad
