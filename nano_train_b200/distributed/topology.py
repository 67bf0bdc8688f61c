"""Process topology: Megatron-style TP / PP / EP / CP / DP / EDP groups.

Rank layout (the reference's, EP fastest then CP; src/distributed/topology.py:159-224):

    rank = ((((dp * PP + pp) * TP + tp) * EP + ep) * CP + cp)

so on one 8-GPU node the fastest axes share NVSwitch ports evenly (every
peer has full bandwidth anyway). Groups are built by one generic routine:
"vary a set of axes, fix the others", iterated in the same order on every
rank so ``dist.new_group`` calls line up.

A second layout, ``expert_layout="fold_dp"`` (Megatron EP inside DP), is a
B200-build extension: EP ranks are carved out of the data-parallel axis so
each EP rank trains on its own data; the reference's layout
(``"separate"``) keeps EP as its own axis with replicated data.
"""
from __future__ import annotations

import itertools
import os
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

from .device import get_backend, get_device

AXES = ("dp", "pp", "tp", "ep", "cp")


@dataclass
class ModelParallelTopology:
    """Resolved topology of this process: sizes, ranks, groups and group tables."""

    rank: int
    world_size: int
    local_rank: int
    device: torch.device
    tensor_model_parallel_size: int
    pipeline_model_parallel_size: int
    expert_model_parallel_size: int
    context_parallel_size: int
    data_parallel_size: int
    expert_data_parallel_size: int
    tensor_model_parallel_rank: int
    pipeline_model_parallel_rank: int
    expert_model_parallel_rank: int
    context_parallel_rank: int
    data_parallel_rank: int
    tensor_model_parallel_group: Optional[object]
    pipeline_model_parallel_group: Optional[object]
    expert_model_parallel_group: Optional[object]
    context_parallel_group: Optional[object]
    data_parallel_group: Optional[object]
    expert_data_parallel_group: Optional[object]
    tensor_model_parallel_replica_group: Optional[object]
    expert_model_parallel_replica_group: Optional[object]
    pipeline_stage_replica_group: Optional[object]
    tensor_model_parallel_group_table: list[list[int]]
    pipeline_model_parallel_group_table: list[list[int]]
    expert_model_parallel_group_table: list[list[int]]
    context_parallel_group_table: list[list[int]]
    data_parallel_group_table: list[list[int]]
    expert_data_parallel_group_table: list[list[int]]
    expert_layout: str = "separate"
    extra: dict = field(default_factory=dict)

    def rank_from_coords(self, data_parallel_rank: int, pipeline_model_parallel_rank: int,
                         tensor_model_parallel_rank: int, expert_model_parallel_rank: int,
                         context_parallel_rank: int = 0) -> int:
        """Global rank of a coordinate. With ``expert_layout="fold_dp"`` the rank grid has no EP axis
        (the EP rank is ``data_parallel_rank % EP``), so the expert rank argument is not used."""
        fold = self.expert_layout == "fold_dp"
        return rank_from_coords(data_parallel_rank=data_parallel_rank,
                                pipeline_model_parallel_rank=pipeline_model_parallel_rank,
                                tensor_model_parallel_rank=tensor_model_parallel_rank,
                                expert_model_parallel_rank=0 if fold else expert_model_parallel_rank,
                                pipeline_model_parallel_size=self.pipeline_model_parallel_size,
                                tensor_model_parallel_size=self.tensor_model_parallel_size,
                                expert_model_parallel_size=1 if fold else self.expert_model_parallel_size,
                                context_parallel_rank=context_parallel_rank,
                                context_parallel_size=self.context_parallel_size)

    tp_size = property(lambda self: self.tensor_model_parallel_size)
    pp_size = property(lambda self: self.pipeline_model_parallel_size)
    ep_size = property(lambda self: self.expert_model_parallel_size)
    cp_size = property(lambda self: self.context_parallel_size)
    dp_size = property(lambda self: self.data_parallel_size)
    tp_rank = property(lambda self: self.tensor_model_parallel_rank)
    pp_rank = property(lambda self: self.pipeline_model_parallel_rank)
    ep_rank = property(lambda self: self.expert_model_parallel_rank)
    cp_rank = property(lambda self: self.context_parallel_rank)
    dp_rank = property(lambda self: self.data_parallel_rank)
    tp_group = property(lambda self: self.tensor_model_parallel_group)
    pp_group = property(lambda self: self.pipeline_model_parallel_group)
    ep_group = property(lambda self: self.expert_model_parallel_group)
    dp_group = property(lambda self: self.data_parallel_group)
    edp_group = property(lambda self: self.expert_data_parallel_group)
    tp_replica_group = property(lambda self: self.tensor_model_parallel_replica_group)
    ep_replica_group = property(lambda self: self.expert_model_parallel_replica_group)
    stage_replica_group = property(lambda self: self.pipeline_stage_replica_group)
    tp_group_table = property(lambda self: self.tensor_model_parallel_group_table)
    pp_group_table = property(lambda self: self.pipeline_model_parallel_group_table)
    ep_group_table = property(lambda self: self.expert_model_parallel_group_table)
    dp_group_table = property(lambda self: self.data_parallel_group_table)

    @property
    def is_first_pipeline_stage(self) -> bool:
        return self.pipeline_model_parallel_rank == 0

    @property
    def is_last_pipeline_stage(self) -> bool:
        return self.pipeline_model_parallel_rank == self.pipeline_model_parallel_size - 1


ParallelSetup4D = ModelParallelTopology


def rank_from_coords(data_parallel_rank: int, pipeline_model_parallel_rank: int, tensor_model_parallel_rank: int,
                     expert_model_parallel_rank: int, pipeline_model_parallel_size: int,
                     tensor_model_parallel_size: int, expert_model_parallel_size: int,
                     context_parallel_rank: int = 0, context_parallel_size: int = 1) -> int:
    """Global rank of (dp, pp, tp, ep, cp) in the EP-fastest layout."""
    r = data_parallel_rank
    r = r * pipeline_model_parallel_size + pipeline_model_parallel_rank
    r = r * tensor_model_parallel_size + tensor_model_parallel_rank
    r = r * expert_model_parallel_size + expert_model_parallel_rank
    return r * context_parallel_size + context_parallel_rank


def coords_from_rank(rank: int, pipeline_model_parallel_size: int, tensor_model_parallel_size: int,
                     expert_model_parallel_size: int, context_parallel_size: int = 1):
    """Inverse of rank_from_coords: returns (dp, pp, tp, ep, cp)."""
    cp = rank % context_parallel_size
    rest = rank // context_parallel_size
    ep = rest % expert_model_parallel_size
    rest //= expert_model_parallel_size
    tp = rest % tensor_model_parallel_size
    rest //= tensor_model_parallel_size
    pp = rest % pipeline_model_parallel_size
    dp = rest // pipeline_model_parallel_size
    return dp, pp, tp, ep, cp


def _new_group_if_needed(ranks: list[int], distributed: bool):
    if not distributed:
        return None
    return dist.new_group(ranks)


class _Grid:
    """Axis sizes of the rank grid and the generic group enumeration."""

    def __init__(self, sizes: dict[str, int]):
        self.sizes = sizes

    def rank(self, c: dict[str, int]) -> int:
        return rank_from_coords(c["dp"], c["pp"], c["tp"], c["ep"], self.sizes["pp"], self.sizes["tp"],
                                self.sizes["ep"], c["cp"], self.sizes["cp"])

    def groups(self, vary: tuple[str, ...]):
        """Yield (fixed coords, ranks) for every group varying ``vary``, in deterministic order."""
        fixed_axes = [a for a in AXES if a not in vary]
        for fixed in itertools.product(*[range(self.sizes[a]) for a in fixed_axes]):
            base = dict(zip(fixed_axes, fixed))
            ranks = []
            for var in itertools.product(*[range(self.sizes[a]) for a in vary]):
                c = dict(base)
                c.update(zip(vary, var))
                ranks.append(self.rank(c))
            yield base, ranks


def _build(grid: _Grid, vary: tuple[str, ...], me: dict[str, int], distributed: bool, create: bool = True):
    table, mine = [], None
    for fixed, ranks in grid.groups(vary):
        table.append(ranks)
        g = _new_group_if_needed(ranks, distributed) if create else None
        if all(me[a] == v for a, v in fixed.items()):
            mine = g
    return table, mine


def initialize_model_parallel(*, tensor_model_parallel_size: int, pipeline_model_parallel_size: int,
                              expert_model_parallel_size: int, context_parallel_size: int = 1,
                              expert_layout: str = "separate", timeout=None) -> ModelParallelTopology:
    """Initialise the default process group (if needed) and every parallel group.

    Reads RANK / WORLD_SIZE / LOCAL_RANK from the environment; the backend is
    NCCL on CUDA machines and gloo otherwise.
    """
    rank = int(os.environ.get("RANK", "0"))
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    for name, v in (("tensor_model_parallel_size", tensor_model_parallel_size),
                    ("pipeline_model_parallel_size", pipeline_model_parallel_size),
                    ("expert_model_parallel_size", expert_model_parallel_size),
                    ("context_parallel_size", context_parallel_size)):
        if v < 1:
            raise ValueError(f"{name} must be >= 1")
    if expert_layout not in ("separate", "fold_dp"):
        raise ValueError(f"unknown expert_layout {expert_layout}")
    ep_axis = expert_model_parallel_size if expert_layout == "separate" else 1
    model_parallel = tensor_model_parallel_size * pipeline_model_parallel_size * ep_axis * context_parallel_size
    if world_size % model_parallel != 0:
        raise ValueError("world_size must be divisible by tensor*pipeline*expert*context sizes: "
                         f"{world_size} vs {model_parallel}")
    backend = get_backend()
    device = get_device("cuda" if backend == "nccl" else "cpu", local_rank)
    if device.type == "cuda":
        torch.cuda.set_device(local_rank)
    distributed = world_size > 1
    if distributed and not dist.is_initialized():
        kwargs = dict(backend=backend, world_size=world_size, rank=rank)
        if timeout is not None:
            kwargs["timeout"] = timeout
        dist.init_process_group(**kwargs)
    dp_size = world_size // model_parallel
    sizes = dict(dp=dp_size, pp=pipeline_model_parallel_size, tp=tensor_model_parallel_size, ep=ep_axis,
                 cp=context_parallel_size)
    grid = _Grid(sizes)
    dp, pp, tp, ep, cp = coords_from_rank(rank, sizes["pp"], sizes["tp"], sizes["ep"], sizes["cp"])
    me = dict(dp=dp, pp=pp, tp=tp, ep=ep, cp=cp)

    tables = {}
    groups = {}
    # Creation order is fixed (identical on all ranks): TP, EP, PP, CP, DP, EDP, TP-replica, stage-replica.
    tables["tp"], groups["tp"] = _build(grid, ("tp",), me, distributed, sizes["tp"] > 1) if sizes["tp"] > 1 else ([], None)
    if expert_layout == "separate":
        tables["ep"], groups["ep"] = _build(grid, ("ep",), me, distributed) if sizes["ep"] > 1 else ([], None)
    tables["pp"], groups["pp"] = _build(grid, ("pp",), me, distributed) if sizes["pp"] > 1 else ([], None)
    tables["cp"], groups["cp"] = _build(grid, ("cp",), me, distributed) if sizes["cp"] > 1 else ([], None)
    tables["dp"], groups["dp"] = _build(grid, ("dp",), me, distributed) if sizes["dp"] > 1 else ([], None)
    if expert_layout == "separate":
        tables["edp"], groups["edp"] = _build(grid, ("dp", "tp"), me, distributed)
        edp_size = dp_size * sizes["tp"]
        ep_rank = ep
        ep_size = sizes["ep"]
    else:
        # EP folded into DP: EP groups are consecutive blocks of `ep` data-parallel ranks
        # (with pp, tp, cp fixed); expert replicas are the other blocks (and the TP ranks).
        epn = expert_model_parallel_size
        if dp_size % epn != 0:
            raise ValueError(f"data_parallel_size {dp_size} must be divisible by expert_model_parallel_size {epn}")
        ep_rank = dp % epn
        ep_size = epn
        t_ep, t_edp = [], []
        g_ep = g_edp = None
        for fixed, ranks in grid.groups(("dp",)):
            for blk in range(dp_size // epn):
                rs = ranks[blk * epn:(blk + 1) * epn]
                t_ep.append(rs)
                g = _new_group_if_needed(rs, distributed) if epn > 1 else None
                if rank in rs:
                    g_ep = g
        for fixed, _ in grid.groups(("dp", "tp")):
            for e in range(epn):
                rs = []
                for d in range(e, dp_size, epn):
                    for t in range(sizes["tp"]):
                        c = dict(fixed)
                        c.update(dp=d, tp=t)
                        rs.append(grid.rank(c))
                t_edp.append(rs)
                g = _new_group_if_needed(rs, distributed)
                if rank in rs:
                    g_edp = g
        tables["ep"], groups["ep"] = t_ep, g_ep
        tables["edp"], groups["edp"] = t_edp, g_edp
        edp_size = (dp_size // epn) * sizes["tp"]
    _, tp_replica = _build(grid, ("dp", "ep"), me, distributed)
    _, stage_replica = _build(grid, ("dp", "tp", "ep", "cp"), me, distributed)
    return ModelParallelTopology(
        rank=rank, world_size=world_size, local_rank=local_rank, device=device,
        tensor_model_parallel_size=sizes["tp"], pipeline_model_parallel_size=sizes["pp"],
        expert_model_parallel_size=ep_size, context_parallel_size=sizes["cp"], data_parallel_size=dp_size,
        expert_data_parallel_size=edp_size, tensor_model_parallel_rank=tp, pipeline_model_parallel_rank=pp,
        expert_model_parallel_rank=ep_rank, context_parallel_rank=cp, data_parallel_rank=dp,
        tensor_model_parallel_group=groups["tp"], pipeline_model_parallel_group=groups["pp"],
        expert_model_parallel_group=groups["ep"], context_parallel_group=groups["cp"],
        data_parallel_group=groups["dp"], expert_data_parallel_group=groups["edp"],
        tensor_model_parallel_replica_group=tp_replica, expert_model_parallel_replica_group=groups["edp"],
        pipeline_stage_replica_group=stage_replica,
        tensor_model_parallel_group_table=tables["tp"], pipeline_model_parallel_group_table=tables["pp"],
        expert_model_parallel_group_table=tables["ep"], context_parallel_group_table=tables["cp"],
        data_parallel_group_table=tables["dp"], expert_data_parallel_group_table=tables["edp"],
        expert_layout=expert_layout)


def init_parallel_4d(*, tensor_model_parallel_size: int = 1, pipeline_model_parallel_size: int = 1,
                     expert_model_parallel_size: int = 1, context_parallel_size: int = 1, **kw):
    """Alias of initialize_model_parallel with every size defaulting to 1."""
    return initialize_model_parallel(tensor_model_parallel_size=tensor_model_parallel_size,
                                     pipeline_model_parallel_size=pipeline_model_parallel_size,
                                     expert_model_parallel_size=expert_model_parallel_size,
                                     context_parallel_size=context_parallel_size, **kw)
