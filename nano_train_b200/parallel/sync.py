"""Parameter / gradient synchronisation across replica domains.

* ``collect_param_shard_info``: tensor-parallel sharded params (Column/Row
  linears with tp > 1), expert-parallel params (local experts of an EP MoE),
  plus optimizer-owned low-bit masters by their recorded shard domain.
* ``synchronize_initial_parameters``: broadcast from the first replica -
  TP-sharded params over the TP-replica group, expert params over the
  expert-data-parallel group, everything else over the stage-replica group.
* ``synchronize_gradients``: all-reduce + average over DP (dense) or EDP
  (expert), materialising zero gradients so every rank issues the same
  collectives in the same order. Gradients of one domain are flattened into
  one bucket and reduced with a single collective (the reference issues one
  collective per parameter).

Reference parity: src/runtime/sync.py:20-219.
"""
from __future__ import annotations


import torch
import torch.distributed as dist
import torch.nn as nn

from ..runtime.contracts import ParamShardInfo


def collect_param_shard_info(model: nn.Module, tensor_model_parallel_group=None) -> ParamShardInfo:
    from ..layers import ColumnParallelLinear, RowParallelLinear
    from ..models.moe import ExpertParallelMoE
    from ..precision.master_store import get_lowbit_master_store

    tp_ids: set[int] = set()
    ep_ids: set[int] = set()
    for m in model.modules():
        if isinstance(m, ColumnParallelLinear):
            if m.tp_size <= 1:
                continue
            if m.tp_group is not tensor_model_parallel_group:
                raise ValueError("Unsupported ColumnParallelLinear tp_group in model")
            tp_ids.add(id(m.weight))
            if m.bias is not None:
                tp_ids.add(id(m.bias))
        elif isinstance(m, RowParallelLinear):
            if m.tp_size <= 1:
                continue
            if m.tp_group is not tensor_model_parallel_group:
                raise ValueError("Unsupported RowParallelLinear tp_group in model")
            tp_ids.add(id(m.weight))
        elif isinstance(m, ExpertParallelMoE):
            for e in m.experts:
                for p in e.parameters():
                    ep_ids.add(id(p))
    store = get_lowbit_master_store(model)
    if store is not None:
        from ..precision.master_store import EXPERT, TENSOR

        tp_ids.update(id(p) for p in store.params_in(TENSOR))
        ep_ids.update(id(p) for p in store.params_in(EXPERT))
    return ParamShardInfo(tensor_model_parallel_sharded_param_ids=tp_ids, expert_model_parallel_sharded_param_ids=ep_ids)


def synchronize_initial_parameters(model: nn.Module, shard_info: ParamShardInfo, parallel) -> None:
    if parallel.world_size == 1:
        return
    rc = parallel.rank_from_coords
    tp_src = rc(data_parallel_rank=0, pipeline_model_parallel_rank=parallel.pipeline_model_parallel_rank,
                tensor_model_parallel_rank=parallel.tensor_model_parallel_rank, expert_model_parallel_rank=0,
                context_parallel_rank=parallel.context_parallel_rank)
    ep_src = rc(data_parallel_rank=0, pipeline_model_parallel_rank=parallel.pipeline_model_parallel_rank,
                tensor_model_parallel_rank=0, expert_model_parallel_rank=parallel.expert_model_parallel_rank,
                context_parallel_rank=parallel.context_parallel_rank)
    stage_src = rc(data_parallel_rank=0, pipeline_model_parallel_rank=parallel.pipeline_model_parallel_rank,
                   tensor_model_parallel_rank=0, expert_model_parallel_rank=0,
                   context_parallel_rank=parallel.context_parallel_rank)
    if getattr(parallel, "expert_layout", "separate") == "fold_dp":
        # EP ranks are data-parallel ranks: the first replica of each expert shard is its first EDP rank.
        edp_table = parallel.expert_data_parallel_group_table
        for ranks in edp_table:
            if parallel.rank in ranks:
                ep_src = ranks[0]
    for p in model.parameters():
        pid = id(p)
        if pid in shard_info.tensor_model_parallel_sharded_param_ids:
            if parallel.tensor_model_parallel_size > 1:
                dist.broadcast(p.data, src=tp_src, group=parallel.tensor_model_parallel_replica_group)
        elif pid in shard_info.expert_model_parallel_sharded_param_ids:
            if parallel.expert_data_parallel_size > 1:
                dist.broadcast(p.data, src=ep_src, group=parallel.expert_model_parallel_replica_group)
        else:
            dist.broadcast(p.data, src=stage_src, group=parallel.pipeline_stage_replica_group)
    for b in model.buffers():
        dist.broadcast(b.data, src=stage_src, group=parallel.pipeline_stage_replica_group)


def _flat_allreduce_mean(grads: list[torch.Tensor], group, size: int) -> None:
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    flat.div_(size)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off: off + n].view_as(g))
        off += n


def synchronize_gradients(model: nn.Module, shard_info: ParamShardInfo, data_parallel_size: int,
                          expert_data_parallel_size: int, data_parallel_group, expert_data_parallel_group) -> None:
    dense: dict = {}
    expert: dict = {}
    for p in model.parameters():
        is_expert = id(p) in shard_info.expert_model_parallel_sharded_param_ids
        need = (data_parallel_size > 1 and not is_expert) or (expert_data_parallel_size > 1 and is_expert)
        if p.grad is None:
            if not need:
                continue
            p.grad = torch.zeros_like(p)
        if not need:
            continue
        bucket = expert if is_expert else dense
        bucket.setdefault(p.grad.dtype, []).append(p.grad)
    for grads in dense.values():
        _flat_allreduce_mean(grads, data_parallel_group, data_parallel_size)
    for grads in expert.values():
        _flat_allreduce_mean(grads, expert_data_parallel_group, expert_data_parallel_size)
