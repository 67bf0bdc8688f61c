"""Argument validation for the 4-D runtime path, as an ordered table of rules.

Each ``Rule`` states one constraint on the parsed arguments as a predicate over a ``_Layout`` (the
arguments plus the derived quantities: the model-parallel product, the expert axis that counts
against the world size, the data-parallel size); ``validate_args`` walks the table in order and
raises ``ValueError`` with the first broken rule's message. The rule set and the message texts are
those of the reference (src/runtime/validation.py:9-191), because existing launch scripts and
tests match on the texts; the table form is this framework's.

Two rules relax under ``--expert-layout fold_dp`` (EP carved out of the data-parallel axis, Megatron
style): TP > 1 with EP > 1 becomes legal, and dropout under TP / EP is allowed because expert
replicas synchronise over the expert-data-parallel group. In exchange the data-parallel size must
split into EP groups.
"""
from __future__ import annotations

import argparse
from dataclasses import dataclass
from typing import Callable, Optional, Union

SHARDING_STRATEGIES = ("no_shard", "optim", "optim_grads", "optim_grads_params")


def parse_pp_layer_splits(raw_splits: Optional[str]) -> Optional[tuple[int, ...]]:
    """``"0,3,8"`` -> ``(0, 3, 8)``; None or a blank / comma-only string -> None."""
    fields = [f.strip() for f in (raw_splits or "").split(",")]
    fields = [f for f in fields if f]
    if not fields:
        return None
    try:
        return tuple(int(f) for f in fields)
    except ValueError:
        raise ValueError("pp_layer_splits must be a comma-separated integer list") from None


@dataclass(frozen=True)
class _Layout:
    a: argparse.Namespace
    world: int
    splits: Optional[tuple[int, ...]]

    @property
    def fold(self) -> bool:
        return getattr(self.a, "expert_layout", "separate") == "fold_dp"

    @property
    def mp(self) -> int:
        """Ranks of one model replica: TP x PP x CP, times EP unless EP is folded into DP."""
        ep_axis = 1 if self.fold else self.a.expert_model_parallel_size
        return (self.a.tensor_model_parallel_size * self.a.pipeline_model_parallel_size * ep_axis
                * self.a.context_parallel_size)

    @property
    def tp_ep(self) -> bool:
        return self.a.tensor_model_parallel_size > 1 or self.a.expert_model_parallel_size > 1

    def get(self, name: str, default):
        return getattr(self.a, name, default)


Message = Union[str, Callable[[_Layout], str]]


@dataclass(frozen=True)
class Rule:
    broken: Callable[[_Layout], bool]
    message: Message

    def text(self, lay: _Layout) -> str:
        return self.message(lay) if callable(self.message) else self.message


def _sizes(lay: _Layout) -> tuple[int, ...]:
    a = lay.a
    return (a.tensor_model_parallel_size, a.pipeline_model_parallel_size, a.expert_model_parallel_size,
            a.context_parallel_size)


def _splits_broken(lay: _Layout) -> Optional[str]:
    s = lay.splits
    if s is None:
        return None
    if len(s) != lay.a.pipeline_model_parallel_size + 1:
        return "pp_layer_splits length must equal pipeline_model_parallel_size + 1"
    if s[0] != 0:
        return "pp_layer_splits must start with 0"
    if s[-1] != lay.a.num_layers:
        return "pp_layer_splits must end at num_layers"
    if any(b <= a for a, b in zip(s, s[1:])):
        return "pp_layer_splits must be strictly increasing"
    return None


_TP_EP_MSG = ("This tutorial disallows tensor_model_parallel_size>1 with expert_model_parallel_size>1 when "
              "expert_tensor_parallel_size=1. That setup replicates expert shards across TP lanes. "
              "Use tensor_model_parallel_size=1 for MoE EP runs.")
_DROPOUT_MSG = ("dropout must be 0.0 when tensor_model_parallel_size>1 or expert_model_parallel_size>1 in this "
                "tutorial. This keeps replicated non-sharded parameter paths deterministic without extra "
                "model-parallel gradient synchronization.")

RULES: tuple[Rule, ...] = (
    # parallel factorisation
    Rule(lambda l: any(s < 1 for s in _sizes(l)), "parallel sizes must be >= 1"),
    Rule(lambda l: l.mp > l.world, "tensor*pipeline*expert*context cannot exceed world_size"),
    Rule(lambda l: l.world % l.mp != 0,
         lambda l: f"world_size ({l.world}) must be divisible by tensor*pipeline*expert*context ({l.mp})"),
    Rule(lambda l: l.fold and (l.world // l.mp) % l.a.expert_model_parallel_size != 0,
         "data_parallel_size must be divisible by expert_model_parallel_size with fold_dp"),
    # model dimensions against the parallel sizes
    Rule(lambda l: l.a.intermediate_size % max(1, l.a.tensor_model_parallel_size) != 0,
         "intermediate_size must be divisible by tensor_model_parallel_size"),
    Rule(lambda l: l.a.num_heads % max(1, l.a.tensor_model_parallel_size) != 0,
         "num_heads must be divisible by tensor_model_parallel_size"),
    Rule(lambda l: l.a.num_experts % l.a.expert_model_parallel_size != 0,
         "num_experts must be divisible by expert_model_parallel_size"),
    Rule(lambda l: l.a.seq_len < 2, "seq_len must be >= 2 for causal LM loss"),
    Rule(lambda l: l.a.tensor_model_parallel_size > 1 and l.a.seq_len % l.a.tensor_model_parallel_size != 0,
         "seq_len must be divisible by tensor_model_parallel_size for sequence-parallel MoE"),
    # features the runtime does not have
    Rule(lambda l: l.a.context_parallel_size != 1, "context_parallel_size > 1 is not yet implemented in this tutorial"),
    Rule(lambda l: l.a.expert_tensor_parallel_size != 1, "expert_tensor_parallel_size must be 1 in this tutorial"),
    Rule(lambda l: l.a.tensor_model_parallel_size > 1 and l.a.expert_model_parallel_size > 1 and not l.fold,
         _TP_EP_MSG),
    Rule(lambda l: l.a.dropout > 0.0 and l.tp_ep and not l.fold, _DROPOUT_MSG),
    # ZeRO / distributed optimizer
    Rule(lambda l: l.a.data_parallel_sharding_strategy not in SHARDING_STRATEGIES,
         "data_parallel_sharding_strategy must be one of no_shard, optim, optim_grads, optim_grads_params"),
    Rule(lambda l: l.a.data_parallel_sharding_strategy == "optim_grads_params",
         "optim_grads_params (ZeRO-3) is out of scope in this tutorial. Use no_shard, optim, or optim_grads."),
    Rule(lambda l: l.a.num_distributed_optimizer_instances != 1,
         "num_distributed_optimizer_instances must be 1 in this tutorial implementation"),
    Rule(lambda l: l.a.data_parallel_sharding_strategy != "no_shard" and not l.a.use_distributed_optimizer,
         "use_distributed_optimizer must be enabled when sharding strategy is not no_shard"),
    Rule(lambda l: l.a.use_distributed_optimizer and l.a.data_parallel_sharding_strategy == "no_shard",
         "When use_distributed_optimizer is set, select sharding strategy optim or optim_grads"),
    Rule(lambda l: bool(l.get("zero_debug", False)) and not l.a.use_distributed_optimizer,
         "zero_debug requires use_distributed_optimizer=True"),
    Rule(lambda l: int(l.get("zero_debug_max_steps", 1)) < 1, "zero_debug_max_steps must be >= 1"),
    Rule(lambda l: int(l.get("zero_debug_max_params", 8)) < 1, "zero_debug_max_params must be >= 1"),
    # 1F1B batching and stage boundaries (precision flags are checked where precision is resolved)
    Rule(lambda l: l.a.num_microbatches < 1, "num_microbatches must be >= 1"),
    Rule(lambda l: l.a.batch_size % l.a.num_microbatches != 0,
         "batch_size must be divisible by num_microbatches for fixed-shape 1F1B"),
    Rule(lambda l: _splits_broken(l) is not None, lambda l: _splits_broken(l)),
)


def broken_rules(args: argparse.Namespace, world_size: int,
                 pp_layer_splits: Optional[tuple[int, ...]]) -> list[str]:
    """Messages of every rule the arguments break, in table order (to report all of them at once).
    A rule that cannot be evaluated (a division by a zero parallel size, itself reported by the
    first rule) is skipped."""
    lay = _Layout(args, world_size, pp_layer_splits)
    out = []
    for rule in RULES:
        try:
            if rule.broken(lay):
                out.append(rule.text(lay))
        except ZeroDivisionError:
            continue
    return out


def validate_args(args: argparse.Namespace, world_size: int, pp_layer_splits: Optional[tuple[int, ...]]) -> None:
    """Raise ValueError with the first broken rule's message."""
    lay = _Layout(args, world_size, pp_layer_splits)
    for rule in RULES:
        if rule.broken(lay):
            raise ValueError(rule.text(lay))
