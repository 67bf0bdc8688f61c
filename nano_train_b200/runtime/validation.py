"""Argument validation for the 4-D runtime path.

Same checks and error texts as the reference (src/runtime/validation.py:9-191)
so existing scripts and tests see identical failures. Two guards relax when
the B200-build option ``--expert-layout fold_dp`` is given (EP carved out of
the data-parallel axis, Megatron style): TP>1 with EP>1 becomes legal, and
dropout under TP/EP is allowed because expert replicas synchronise over the
expert-data-parallel group.
"""
from __future__ import annotations

import argparse
from typing import Optional


def parse_pp_layer_splits(raw_splits: Optional[str]) -> Optional[tuple[int, ...]]:
    if raw_splits is None:
        return None
    text = raw_splits.strip()
    if not text:
        return None
    parts = [p.strip() for p in text.split(",") if p.strip()]
    if not parts:
        return None
    try:
        return tuple(int(p) for p in parts)
    except ValueError as exc:
        raise ValueError("pp_layer_splits must be a comma-separated integer list") from exc


def _fold(args) -> bool:
    return getattr(args, "expert_layout", "separate") == "fold_dp"


def _validate_parallel_factorization(args: argparse.Namespace, world_size: int) -> None:
    sizes = (args.tensor_model_parallel_size, args.pipeline_model_parallel_size, args.expert_model_parallel_size,
             args.context_parallel_size)
    if any(s < 1 for s in sizes):
        raise ValueError("parallel sizes must be >= 1")
    ep_axis = 1 if _fold(args) else args.expert_model_parallel_size
    mp = args.tensor_model_parallel_size * args.pipeline_model_parallel_size * ep_axis * args.context_parallel_size
    if mp > world_size:
        raise ValueError("tensor*pipeline*expert*context cannot exceed world_size")
    if world_size % mp != 0:
        raise ValueError(f"world_size ({world_size}) must be divisible by tensor*pipeline*expert*context ({mp})")
    if _fold(args):
        dp = world_size // mp
        if dp % args.expert_model_parallel_size != 0:
            raise ValueError("data_parallel_size must be divisible by expert_model_parallel_size with fold_dp")


def _validate_model_dimension_compatibility(args: argparse.Namespace) -> None:
    tp = max(1, args.tensor_model_parallel_size)
    if args.intermediate_size % tp != 0:
        raise ValueError("intermediate_size must be divisible by tensor_model_parallel_size")
    if args.num_heads % tp != 0:
        raise ValueError("num_heads must be divisible by tensor_model_parallel_size")
    if args.num_experts % args.expert_model_parallel_size != 0:
        raise ValueError("num_experts must be divisible by expert_model_parallel_size")
    if args.seq_len < 2:
        raise ValueError("seq_len must be >= 2 for causal LM loss")
    if args.tensor_model_parallel_size > 1 and args.seq_len % args.tensor_model_parallel_size != 0:
        raise ValueError("seq_len must be divisible by tensor_model_parallel_size for sequence-parallel MoE")


def _validate_tutorial_guards(args: argparse.Namespace) -> None:
    if args.context_parallel_size != 1:
        raise ValueError("context_parallel_size > 1 is not yet implemented in this tutorial")
    if args.expert_tensor_parallel_size != 1:
        raise ValueError("expert_tensor_parallel_size must be 1 in this tutorial")
    if args.tensor_model_parallel_size > 1 and args.expert_model_parallel_size > 1 and not _fold(args):
        raise ValueError(
            "This tutorial disallows tensor_model_parallel_size>1 with expert_model_parallel_size>1 when "
            "expert_tensor_parallel_size=1. That setup replicates expert shards across TP lanes. "
            "Use tensor_model_parallel_size=1 for MoE EP runs.")
    if args.dropout > 0.0 and (args.tensor_model_parallel_size > 1 or args.expert_model_parallel_size > 1) \
            and not _fold(args):
        raise ValueError(
            "dropout must be 0.0 when tensor_model_parallel_size>1 or expert_model_parallel_size>1 in this "
            "tutorial. This keeps replicated non-sharded parameter paths deterministic without extra "
            "model-parallel gradient synchronization.")


def _validate_zero_optimizer_settings(args: argparse.Namespace) -> None:
    strategy = args.data_parallel_sharding_strategy
    if strategy not in {"no_shard", "optim", "optim_grads", "optim_grads_params"}:
        raise ValueError("data_parallel_sharding_strategy must be one of no_shard, optim, optim_grads, "
                         "optim_grads_params")
    if strategy == "optim_grads_params":
        raise ValueError("optim_grads_params (ZeRO-3) is out of scope in this tutorial. "
                         "Use no_shard, optim, or optim_grads.")
    if args.num_distributed_optimizer_instances != 1:
        raise ValueError("num_distributed_optimizer_instances must be 1 in this tutorial implementation")
    if strategy != "no_shard" and not args.use_distributed_optimizer:
        raise ValueError("use_distributed_optimizer must be enabled when sharding strategy is not no_shard")
    if args.use_distributed_optimizer and strategy == "no_shard":
        raise ValueError("When use_distributed_optimizer is set, select sharding strategy optim or optim_grads")
    if bool(getattr(args, "zero_debug", False)) and not args.use_distributed_optimizer:
        raise ValueError("zero_debug requires use_distributed_optimizer=True")
    if int(getattr(args, "zero_debug_max_steps", 1)) < 1:
        raise ValueError("zero_debug_max_steps must be >= 1")
    if int(getattr(args, "zero_debug_max_params", 8)) < 1:
        raise ValueError("zero_debug_max_params must be >= 1")


def _validate_pipeline_batching(args: argparse.Namespace, pp_layer_splits: Optional[tuple[int, ...]]) -> None:
    if args.num_microbatches < 1:
        raise ValueError("num_microbatches must be >= 1")
    if args.batch_size % args.num_microbatches != 0:
        raise ValueError("batch_size must be divisible by num_microbatches for fixed-shape 1F1B")
    if pp_layer_splits is not None:
        if len(pp_layer_splits) != args.pipeline_model_parallel_size + 1:
            raise ValueError("pp_layer_splits length must equal pipeline_model_parallel_size + 1")
        if pp_layer_splits[0] != 0:
            raise ValueError("pp_layer_splits must start with 0")
        if pp_layer_splits[-1] != args.num_layers:
            raise ValueError("pp_layer_splits must end at num_layers")
        for i in range(1, len(pp_layer_splits)):
            if pp_layer_splits[i] <= pp_layer_splits[i - 1]:
                raise ValueError("pp_layer_splits must be strictly increasing")


def _validate_precision_args(args: argparse.Namespace) -> None:
    """Precision flags are validated where precision is resolved."""
    del args


def validate_args(args: argparse.Namespace, world_size: int, pp_layer_splits: Optional[tuple[int, ...]]) -> None:
    _validate_parallel_factorization(args, world_size)
    _validate_model_dimension_compatibility(args)
    _validate_tutorial_guards(args)
    _validate_zero_optimizer_settings(args)
    _validate_pipeline_batching(args, pp_layer_splits)
    _validate_precision_args(args)
