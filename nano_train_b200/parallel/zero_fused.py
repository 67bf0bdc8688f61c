"""Symmetric flat buffers and the fused ZeRO step (csrc/zero_fused.cu) for one NVLink node.

The flat optimizer's parameter (bf16) and gradient (fp32) buffers of every
rank of the data-parallel group live in one symmetric region (CUDA IPC,
identical layout on every rank), so one step is three kernels per rank:
a pull reduce-scatter of this rank's gradient shards (+ the clipping partial
sums, exchanged through peer memory), AdamW on the shard that stores the new
bf16 shard into every rank's parameter buffer (the all-gather), and a
bounded wait for every rank's parameters. NCCL does not take part.

Reference parity: src/distributed/zero.py:392-499 (reduce-scatter or
all-reduce, AdamW on the shard, all-gather, per parameter); here one pass per
step over all buffers.

The reduce-scatter runs one launch per buffer in index order, so the flat optimizer can cut its
parameters into buckets (buffers, last layers first) and reduce each bucket while the backward
still produces the earlier layers' gradients (``FlatAdamW.overlap_next_backward``); the clipping
partials accumulate over the buckets and the last one publishes them.

Layout of the region:
    [0, 256)        flags u64 [3 kinds][8 source ranks]: gradients ready, partial norm, parameters written
    [256, 320)      partial sums of squares fp32 [8 source ranks][2]
    4 KiB ...       per buffer: parameters bf16 [numel], gradients fp32 [numel] (256-byte aligned,
                    each followed by a 256-byte canary, see parallel/region.py)
"""
from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist

from . import comm
from .region import RegionLayout

GRADS, STATS, PARAMS = range(3)
MAX_RANKS = 8
MAX_BUFFERS = 32  # buffers per launch of the step kernels (csrc/zero_fused.cu, kZMaxBufs)


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def fused_zero_available(dp_group, param_dtypes, *, grad_norm_group=None) -> bool:
    """Whether the peer-memory ZeRO step can run for this group (NTB_FUSED_ZERO=0 turns it off)."""
    if os.environ.get("NTB_FUSED_ZERO", "1") == "0":
        return False
    if not (torch.cuda.is_available() and dist.is_initialized()):
        return False
    n = comm.group_size(dp_group)
    if not (comm.min_fused_ranks() <= n <= MAX_RANKS) or dist.get_backend(dp_group) != "nccl":
        return False
    if any(dt != torch.bfloat16 for dt in param_dtypes):
        return False
    if grad_norm_group is not None and comm.group_size(grad_norm_group) > 1:
        return False  # the clipping norm would also need a tensor-parallel reduction
    hosts = [None] * n
    dist.all_gather_object(hosts, socket.gethostname(), group=dp_group)
    return len(set(hosts)) == 1


class ZeroSymm:
    """The data-parallel group's symmetric region and the three-kernel step."""

    def __init__(self, dp_group, numels: list[int], device):
        from ..ops._ext import ext

        self.group = dp_group
        self.n = comm.group_size(dp_group)
        self.rank = comm.group_rank(dp_group)
        self.device = device
        self.numels = list(numels)
        lay = RegionLayout(4096)
        self.poff, self.goff = [], []
        for i, k in enumerate(self.numels):
            self.poff.append(lay.add(f"params{i}", k * 2))
            self.goff.append(lay.add(f"grads{i}", k * 4))
        self.layout = lay
        self.bytes = lay.total
        C = ext()
        self._C = C
        self.local, handle = C.symm_alloc(self.bytes)
        handles = [None] * self.n
        dist.all_gather_object(handles, handle, group=dp_group)
        self.ptrs, self._opened = [], []
        for i, h in enumerate(handles):
            if i == self.rank:
                self.ptrs.append(self.local)
            else:
                p = C.symm_open(h)
                self.ptrs.append(p)
                self._opened.append(p)
        self.done = torch.zeros(1, dtype=torch.int32, device=device)
        self.stats_acc = torch.zeros(2, dtype=torch.float32, device=device)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=device)
        self.scale = torch.ones(1, dtype=torch.float32, device=device)
        self.epoch = 0
        self._open = False  # a step's first bucket was reduced and its adam launch has not run yet
        self._next = 0
        self.closed = False
        lay.fill(C, self.local, device.index)
        dist.barrier(group=dp_group)

    def views(self, i: int):
        """(param bf16 [numel], grad fp32 [numel]) views of buffer i in this rank's region."""
        k = self.numels[i]
        dev = self.device.index
        return (self._C.symm_local_view(self.local, self.poff[i], [k], torch.bfloat16, dev),
                self._C.symm_local_view(self.local, self.goff[i], [k], torch.float32, dev))

    def _flags(self, kind: int):
        return [p + (kind * MAX_RANKS + self.rank) * 8 for p in self.ptrs]

    def _open_step(self) -> int:
        """Epoch of the step in progress (a step opens with its first bucket reduction)."""
        if not self._open:
            self.epoch += 1
            self._open = True
            self._next = 0
        return self.epoch

    @property
    def next_bucket(self) -> int:
        """Index of the next buffer to reduce in the step in progress (0 when none is open)."""
        return self._next if self._open else 0

    @torch.no_grad()
    def reduce_through(self, k: int, shards: list[dict], classes, *, grid: int = 0) -> None:
        """Reduce-scatter buffers next_bucket..k in index order, each once every rank has signalled it
        (gradients-ready flag = epoch * nbuf + i + 1, monotonic over buckets and steps). Runs on the
        current stream; the last buffer of the step publishes the clipping partials."""
        C, n, me = self._C, self.n, self.rank
        e = self._open_step()
        dev = self.device.index
        nb = len(self.numels)
        for i in range(self._next, min(k, nb - 1) + 1):
            value = e * nb + i + 1
            C.ep_signal(self._flags(GRADS), value, dev)
            C.ep_wait(self.local + GRADS * MAX_RANKS * 8, n, value, dev)
            lo, hi = shards[i]["lo"], shards[i]["hi"]
            C.zero_reduce_scatter([[p + self.goff[i] + lo * 4 for p in self.ptrs]], [self.views(i)[1][lo:hi]],
                                  [int(classes[i])], self.stats_acc, [p + 256 + me * 8 for p in self.ptrs],
                                  self._flags(STATS), self.done, me, e, publish=(i == nb - 1), grid=grid)
            self._next = i + 1

    @torch.no_grad()
    def step(self, shards: list[dict], lrs, wds, classes, *, step: int, betas, eps: float, inv_dp: float,
             max_norm: float) -> None:
        """One optimizer step over every buffer; ``shards[i]`` holds lo/hi/master/exp_avg/exp_avg_sq.
        Buffers already reduced during the backward (``reduce_through``) are not reduced again."""
        C, n, me = self._C, self.n, self.rank
        e = self._open_step()
        dev = self.device.index
        self.reduce_through(len(self.numels) - 1, shards, classes)
        red, param_ptrs = [], []
        for i, sh in enumerate(shards):
            lo, hi = sh["lo"], sh["hi"]
            red.append(self.views(i)[1][lo:hi])
            param_ptrs.append([p + self.poff[i] + lo * 2 for p in self.ptrs])
        C.zero_adam_allgather(param_ptrs, red, [s["master"] for s in shards], [s["exp_avg"] for s in shards],
                              [s["exp_avg_sq"] for s in shards], [float(x) for x in lrs], [float(x) for x in wds],
                              self.local + 256, self.local + STATS * MAX_RANKS * 8, self._flags(PARAMS), self.done,
                              me, e, float(betas[0]), float(betas[1]), float(eps), int(step), float(inv_dp),
                              float(max_norm), self.grad_norm, self.scale)
        C.ep_wait(self.local + PARAMS * MAX_RANKS * 8, n, e, dev)
        self._open = False
        self._next = 0

    def check_canaries(self) -> list[str]:
        """Sections of this rank's region whose trailing canary was overwritten (synchronises)."""
        return self.layout.check(self._C, self.local, self.device.index)

    def close(self):
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize()
        for p in self._opened:
            self._C.symm_close(p)
        self._C.symm_free(self.local)
