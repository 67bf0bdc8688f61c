"""Components of the 4-D (TP x PP x EP x DP) DeepSeek training entry point.

``build_train_4d_components()`` returns the six runtime components that
``RuntimeEngine`` drives; ``parse_args()`` accepts the reference's
train_4d flags verbatim (examples/train_4d.py:131-249, mixed ``-``/``_``
spelling kept) plus B200-build options:

  --expert-layout {separate,fold_dp}  EP as its own axis (reference) or carved
                                      out of DP (each EP rank its own data)
  --scoring-func {sigmoid,softmax}    router scoring (reference hard-codes sigmoid)
  --checkpoint-dir / --save-every     real save + resume (the reference's
                                      train_4d checkpoint manager is a no-op)
  --dist-timeout-s / --heartbeat-timeout-s
                                      process-group timeout; fail-fast on a peer
                                      whose heartbeat stopped
"""
from __future__ import annotations

import argparse
import os
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.data import DataLoader, Dataset, DistributedSampler

from ..distributed.topology import initialize_model_parallel
from ..distributed.zero import DistributedOptimizerConfig, MegatronZeroOptimizer
from ..logging import get_logger, setup_logging
from ..models.deepseek import DeepSeekModel, DeepSeekModelConfig, DeepSeekParallelContext
from ..models.moe import ExpertParallelMoE, LocalRoutedMoE
from ..parallel.pipeline import train_step_pipeline
from ..parallel.sync import collect_param_shard_info, synchronize_gradients, synchronize_initial_parameters
from ..precision.master_store import materialize_optimizer_owned_masters
from ..precision.mixed_precision import (MixedPrecisionController, build_module_precision_resolver,
                                         dtype_alias_to_torch, finalize_module_precision_resolver,
                                         refresh_persistent_lowbit_params)
from ..precision.precision_args import add_mixed_precision_args, normalize_and_resolve_precision
from .checkpoint import DirectoryCheckpointManager, NoOpCheckpointManager
from .context import RunConfig, RuntimeContext
from .contracts import OptimizerState, ResumeState, RuntimeComponents, StepContext, StepOutput, TrainDataBundle
from .engine import RuntimeEngine
from .optimizer_runtime import PrecisionAdamW, step_with_sync_policy, zero_grad_optimizer
from .schedules import DefaultScheduleSelector, NonPipelineSchedule, Pipeline1F1BSchedule
from .validation import parse_pp_layer_splits, validate_args

logger = get_logger(__name__)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="4-D parallel DeepSeek training (TP x PP x EP x DP)")
    a = p.add_argument
    a("--tensor-model-parallel-size", type=int, required=True, help="Tensor model parallel size")
    a("--pipeline-model-parallel-size", type=int, required=True, help="Pipeline model parallel size")
    a("--expert-model-parallel-size", type=int, required=True, help="Expert model parallel size")
    a("--context-parallel-size", type=int, default=1, help="Context parallel size (must be 1)")
    a("--expert-tensor-parallel-size", type=int, default=1, help="Expert tensor parallel size (must be 1)")
    a("--num-layers-per-virtual-pipeline-stage", type=int, default=None, help="Reserved (unused)")
    a("--use-distributed-optimizer", action="store_true", help="Enable the ZeRO distributed optimizer")
    a("--data-parallel-sharding-strategy", type=str, default="no_shard",
      help="DP sharding strategy: no_shard | optim | optim_grads")
    a("--num-distributed-optimizer-instances", type=int, default=1, help="Distributed optimizer instances (1)")
    a("--zero-debug", action="store_true", help="Verbose ZeRO debug logging")
    a("--zero-debug-max-steps", type=int, default=1)
    a("--zero-debug-max-params", type=int, default=8)
    a("--num_microbatches", type=int, default=1, help="Pipeline microbatch count for 1F1B")
    a("--pp_layer_splits", type=str, default=None, help="Optional PP layer boundaries, e.g. '0,2,5'")
    a("--batch_size", type=int, default=16)
    a("--num_samples", type=int, default=256)
    a("--seq_len", type=int, default=32)
    a("--epochs", type=int, default=3)
    a("--max_steps", type=int, default=100)
    a("--lr", type=float, default=1e-3)
    a("--weight_decay", type=float, default=0.01)
    a("--vocab_size", type=int, default=512)
    a("--hidden_size", type=int, default=128)
    a("--num_layers", type=int, default=5)
    a("--num_heads", type=int, default=8)
    a("--num_kv_heads", type=int, default=8)
    a("--intermediate_size", type=int, default=256)
    a("--moe_intermediate_size", type=int, default=128)
    a("--q_lora_rank", type=int, default=64)
    a("--kv_lora_rank", type=int, default=32)
    a("--qk_nope_head_dim", type=int, default=8)
    a("--qk_rope_head_dim", type=int, default=8)
    a("--v_head_dim", type=int, default=8)
    a("--max_position_embeddings", type=int, default=256)
    a("--num_experts", type=int, default=8)
    a("--top_k", type=int, default=2)
    a("--n_group", type=int, default=4)
    a("--topk_group", type=int, default=2)
    a("--n_shared_experts", type=int, default=1)
    a("--first_k_dense_replace", type=int, default=1)
    a("--moe_layer_freq", type=int, default=1)
    a("--dropout", type=float, default=0.0)
    a("--capacity_factor", type=float, default=1.0)
    a("--aux_loss_coef", type=float, default=0.01)
    a("--seed", type=int, default=42)
    a("--log_every", type=int, default=10)
    # B200-build options
    a("--expert-layout", type=str, default="separate", choices=["separate", "fold_dp"])
    a("--scoring-func", type=str, default="sigmoid", choices=["sigmoid", "softmax"])
    a("--checkpoint-dir", type=str, default=None)
    a("--save-every", type=int, default=0)
    a("--dist-timeout-s", type=float, default=600.0, help="process-group timeout (failure detection)")
    a("--heartbeat-timeout-s", type=float, default=0.0,
      help="end a rank whose peer sent no heartbeat for this many seconds (0: off)")
    add_mixed_precision_args(p)
    return p


def parse_args(argv=None) -> argparse.Namespace:
    return build_parser().parse_args(argv)


class DummyTokenDataset(Dataset):
    """Deterministic token dataset (uniform ids from a seeded generator)."""

    def __init__(self, num_samples: int, seq_len: int, vocab_size: int, seed: int):
        g = torch.Generator().manual_seed(seed)
        self.input_ids = torch.randint(0, vocab_size, (num_samples, seq_len), generator=g)

    def __len__(self) -> int:
        return len(self.input_ids)

    def __getitem__(self, i: int) -> dict:
        return {"input_ids": self.input_ids[i]}


def build_tiny_deepseek_config(args, *, param_dtype, param_device, precision_resolver,
                               module_compute_dtype_overrides=None) -> DeepSeekModelConfig:
    return DeepSeekModelConfig(
        param_dtype=param_dtype, param_device=param_device, precision_resolver=precision_resolver,
        module_compute_dtype_overrides=dict(module_compute_dtype_overrides or {}), vocab_size=args.vocab_size,
        hidden_size=args.hidden_size, num_hidden_layers=args.num_layers, num_attention_heads=args.num_heads,
        num_key_value_heads=args.num_kv_heads, intermediate_size=args.intermediate_size,
        max_position_embeddings=max(args.max_position_embeddings, args.seq_len), q_lora_rank=args.q_lora_rank,
        kv_lora_rank=args.kv_lora_rank, qk_nope_head_dim=args.qk_nope_head_dim,
        qk_rope_head_dim=args.qk_rope_head_dim, v_head_dim=args.v_head_dim, attention_dropout=args.dropout,
        dropout=args.dropout, moe_intermediate_size=args.moe_intermediate_size, n_routed_experts=args.num_experts,
        n_shared_experts=args.n_shared_experts, num_experts_per_tok=args.top_k,
        first_k_dense_replace=args.first_k_dense_replace, moe_layer_freq=args.moe_layer_freq,
        scoring_func=getattr(args, "scoring_func", "sigmoid"), n_group=args.n_group, topk_group=args.topk_group,
        norm_topk_prob=True, routed_scaling_factor=1.0)


def create_data_loader(dataset: Dataset, batch_size: int, dp_size: int, dp_rank: int, seed: int) -> TrainDataBundle:
    """DP > 1: DistributedSampler(shuffle, seed). DP = 1: the reference's shuffle order (an epoch seed
    drawn from the global RNG, as DataLoader(shuffle=True) does), recorded for exact resume."""
    from ..dataset import EpochSeedRandomSampler

    if dp_size > 1:
        sampler = DistributedSampler(dataset, num_replicas=dp_size, rank=dp_rank, shuffle=True, seed=seed)
    else:
        sampler = EpochSeedRandomSampler(dataset)
    loader = DataLoader(dataset, batch_size=batch_size, shuffle=False, sampler=sampler, num_workers=0,
                        drop_last=False)
    return TrainDataBundle(loader=loader, sampler=sampler)


def gather_moe_metrics(model: nn.Module, device: torch.device):
    """Sum of aux losses and mean dropped fraction over all MoE layers of the last forward, both as
    device scalars: nothing is read back to the host here (callers read once per step)."""
    aux, drops = [], []
    for m in model.modules():
        if isinstance(m, (ExpertParallelMoE, LocalRoutedMoE)):
            aux.append(m.last_aux_loss.reshape(()))
            drops.append(m.last_dropped_fraction_tensor.to(device=device, dtype=torch.float32).reshape(()))
    a = torch.stack(aux).sum() if aux else torch.zeros((), device=device)
    d = torch.stack(drops).mean() if drops else torch.zeros((), device=device)
    return a, d


def _infer_mode(parallel) -> str:
    if parallel.world_size == 1:
        return "single"
    if parallel.pipeline_model_parallel_size > 1:
        return "tp_pp_ep_dp"
    if parallel.tensor_model_parallel_size == 1 and parallel.expert_model_parallel_size > 1:
        return "ep_only"
    return "tp_ep_dp"


def _build_model_for_context(ctx: RuntimeContext) -> DeepSeekModel:
    args = ctx.run_config.args
    par = ctx.parallel
    off = par.pipeline_model_parallel_rank * 1_000_003 + par.tensor_model_parallel_rank * 1009 + \
        par.expert_model_parallel_rank
    torch.manual_seed(args.seed + off)
    if par.device.type == "cuda":
        torch.cuda.manual_seed_all(args.seed + off)
    pc = ctx.run_config.precision_config
    if pc is None:
        raise RuntimeError("precision_config must be resolved in Train4PBootstrap")
    cfg = build_tiny_deepseek_config(args, param_dtype=dtype_alias_to_torch(pc.params_dtype), param_device=par.device,
                                     precision_resolver=build_module_precision_resolver(pc))
    pctx = DeepSeekParallelContext(
        tensor_model_parallel_rank=par.tensor_model_parallel_rank,
        tensor_model_parallel_size=par.tensor_model_parallel_size,
        tensor_model_parallel_group=par.tensor_model_parallel_group,
        expert_model_parallel_rank=par.expert_model_parallel_rank,
        expert_model_parallel_size=par.expert_model_parallel_size,
        expert_model_parallel_group=par.expert_model_parallel_group,
        pipeline_model_parallel_rank=par.pipeline_model_parallel_rank,
        pipeline_model_parallel_size=par.pipeline_model_parallel_size,
        pipeline_model_parallel_group=par.pipeline_model_parallel_group,
        context_parallel_rank=par.context_parallel_rank, context_parallel_size=par.context_parallel_size,
        context_parallel_group=par.context_parallel_group, pp_layer_splits=ctx.run_config.pp_layer_splits,
        capacity_factor=args.capacity_factor, expert_tensor_parallel_size=args.expert_tensor_parallel_size,
        sequence_parallel=True)
    model = DeepSeekModel(cfg, parallel_context=pctx)
    summary = finalize_module_precision_resolver(cfg.precision_resolver)
    store = materialize_optimizer_owned_masters(model, precision_config=pc)
    if par.rank == 0:
        logger.info("Per-module low-bit policy: compute_modules=%d persistent_modules=%d high_precision_exceptions=%d",
                    summary.compute_lowbit_module_count, summary.persistent_lowbit_module_count,
                    summary.high_precision_exception_module_count)
        logger.info("Low-bit master ownership: mode=%s bound_modules=%d", pc.lowbit_master_ownership,
                    0 if store is None else len(store.metadata))
    refresh_persistent_lowbit_params(model)
    return model


def _build_optimizer(*, model, shard_info, ctx: RuntimeContext, precision_config):
    args = ctx.run_config.args
    par = ctx.parallel
    if args.use_distributed_optimizer:
        r = precision_config.deepseek_v3_recipe
        return MegatronZeroOptimizer(
            model=model,
            config=DistributedOptimizerConfig(
                use_distributed_optimizer=True, data_parallel_sharding_strategy=args.data_parallel_sharding_strategy,
                num_distributed_optimizer_instances=args.num_distributed_optimizer_instances, learning_rate=args.lr,
                weight_decay=args.weight_decay, betas=(0.9, 0.999), eps=1e-8, use_reduce_scatter=True,
                main_params_dtype=precision_config.main_params_dtype,
                main_grads_dtype=precision_config.main_grads_dtype, exp_avg_dtype=precision_config.exp_avg_dtype,
                exp_avg_sq_dtype=precision_config.exp_avg_sq_dtype,
                precision_recipe_name=precision_config.precision_recipe_name,
                fp8_rounding="nearest" if r is None else r.rounding_mode,
                fp8_activation_quant_granularity="tensor" if r is None else r.activation_quant_granularity,
                fp8_weight_quant_granularity="tensor" if r is None else r.weight_quant_granularity,
                fp8_comm_quant_enabled=False if r is None else r.comm_quant_enabled,
                fp8_comm_quant_granularity="tensor" if r is None else r.comm_quant_granularity,
                debug=args.zero_debug, debug_max_steps=args.zero_debug_max_steps,
                debug_max_params=args.zero_debug_max_params),
            data_parallel_group=par.data_parallel_group, expert_data_parallel_group=par.expert_data_parallel_group,
            expert_param_ids=shard_info.expert_model_parallel_sharded_param_ids)
    return PrecisionAdamW(model.parameters(), lr=args.lr, weight_decay=args.weight_decay, betas=(0.9, 0.999),
                          eps=1e-8, main_params_dtype=precision_config.main_params_dtype,
                          main_grads_dtype=precision_config.main_grads_dtype,
                          exp_avg_dtype=precision_config.exp_avg_dtype,
                          exp_avg_sq_dtype=precision_config.exp_avg_sq_dtype)


@dataclass
class Train4PBootstrap:
    def build_context(self, args: argparse.Namespace) -> RuntimeContext:
        import datetime

        splits = parse_pp_layer_splits(getattr(args, "pp_layer_splits", None))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        validate_args(args, world, splits)
        par = initialize_model_parallel(tensor_model_parallel_size=args.tensor_model_parallel_size,
                                        pipeline_model_parallel_size=args.pipeline_model_parallel_size,
                                        expert_model_parallel_size=args.expert_model_parallel_size,
                                        context_parallel_size=args.context_parallel_size,
                                        expert_layout=getattr(args, "expert_layout", "separate"),
                                        timeout=datetime.timedelta(seconds=float(getattr(args, "dist_timeout_s",
                                                                                         600.0))))
        pc = normalize_and_resolve_precision(args, par.device)
        return RuntimeContext(parallel=par, mode=_infer_mode(par),
                              run_config=RunConfig(args=args, pp_layer_splits=splits, precision_config=pc))


@dataclass
class Train4PModelProvider:
    def build_model(self, ctx: RuntimeContext) -> torch.nn.Module:
        return _build_model_for_context(ctx)


@dataclass
class Train4PDataProvider:
    def build_train_data(self, ctx: RuntimeContext) -> TrainDataBundle:
        args = ctx.run_config.args
        par = ctx.parallel
        ds = DummyTokenDataset(args.num_samples, args.seq_len, args.vocab_size, args.seed)
        return create_data_loader(ds, args.batch_size, par.data_parallel_size, par.data_parallel_rank, args.seed)


@dataclass
class Train4POptimizerRuntime:
    def initialize(self, model: torch.nn.Module, ctx: RuntimeContext) -> OptimizerState:
        if not isinstance(model, DeepSeekModel):
            raise TypeError("Train4POptimizerRuntime requires a DeepSeekModel")
        pc = ctx.run_config.precision_config
        if pc is None:
            raise RuntimeError("precision_config must be resolved in Train4PBootstrap")
        info = collect_param_shard_info(model=model, tensor_model_parallel_group=ctx.parallel.tensor_model_parallel_group)
        synchronize_initial_parameters(model=model, shard_info=info, parallel=ctx.parallel)
        opt = _build_optimizer(model=model, shard_info=info, ctx=ctx, precision_config=pc)
        ctrl = MixedPrecisionController(pc, device=ctx.parallel.device)
        return OptimizerState(optimizer=opt, shard_info=info, extra_state={"precision_controller": ctrl})

    def zero_grad(self, state: OptimizerState) -> None:
        zero_grad_optimizer(state)

    def step(self, *, model, state: OptimizerState, ctx: RuntimeContext) -> None:
        step_with_sync_policy(model=model, state=state, ctx=ctx, synchronize_gradients_fn=synchronize_gradients)


@dataclass
class Train4PNonPipelineSchedule:
    optimizer_runtime: Train4POptimizerRuntime

    def run_step(self, step_ctx: StepContext) -> StepOutput:
        if step_ctx.batch is None:
            raise RuntimeError("Non-pipeline schedule requires a batch")
        args = step_ctx.runtime_context.run_config.args
        device = step_ctx.runtime_context.parallel.device
        ids = step_ctx.batch["input_ids"].to(device, non_blocking=True)
        ctrl = step_ctx.optimizer_state.extra_state.get("precision_controller")
        self.optimizer_runtime.zero_grad(step_ctx.optimizer_state)
        with (ctrl.autocast_context() if ctrl is not None else torch.autograd.graph.saved_tensors_hooks(
                lambda x: x, lambda x: x)):
            logits = step_ctx.model(ids)
            if ids.size(0) == 0 or ids.size(1) < 2:
                task = logits.sum() * 0.0
            else:
                task = F.cross_entropy(logits[:, :-1, :].reshape(-1, logits.size(-1)).float(), ids[:, 1:].reshape(-1))
            aux, drop = gather_moe_metrics(step_ctx.model, device=device)
            total = task + args.aux_loss_coef * aux
        if ctrl is None:
            total.backward()
            should_step = True
        else:
            ctrl.backward(total)
            should_step = ctrl.prepare_optimizer_step(step_ctx.model)
        if should_step:
            self.optimizer_runtime.step(model=step_ctx.model, state=step_ctx.optimizer_state,
                                        ctx=step_ctx.runtime_context)
            refresh_persistent_lowbit_params(step_ctx.model)
        if ctrl is not None:
            ctrl.update_after_step(step_applied=should_step)
            if (step_ctx.runtime_context.parallel.rank == 0 and args.log_every > 0
                    and step_ctx.train_state.global_step % args.log_every == 0 and ctrl.uses_loss_scaling):
                logger.info("precision step=%d mode=%s loss_scale=%.4f skipped_steps=%d",
                            step_ctx.train_state.global_step, ctrl.config.mode, ctrl.runtime_state.loss_scale,
                            ctrl.runtime_state.skipped_steps)
        vals = torch.stack([task.detach().float(), aux.detach().float().reshape(()), total.detach().float(),
                            drop.float().reshape(())]).tolist()
        return StepOutput(task_loss=vals[0], aux_loss=vals[1], total_loss=vals[2], drop_fraction=vals[3],
                          counters={"objective_count": 1, "drop_count": 1})


@dataclass
class Train4PPipelineSchedule:
    optimizer_runtime: Train4POptimizerRuntime

    def run_step(self, step_ctx: StepContext) -> StepOutput:
        args = step_ctx.runtime_context.run_config.args
        par = step_ctx.runtime_context.parallel
        model = step_ctx.model
        if not isinstance(model, DeepSeekModel):
            raise TypeError("Train4PPipelineSchedule requires a DeepSeekModel")
        ctrl = step_ctx.optimizer_state.extra_state.get("precision_controller")

        def apply_step(**kw) -> None:
            self.optimizer_runtime.step(model=model, state=step_ctx.optimizer_state, ctx=step_ctx.runtime_context)

        t, a, d, oc, dc = train_step_pipeline(
            model=model, optimizer=step_ctx.optimizer_state.optimizer,
            use_distributed_optimizer=args.use_distributed_optimizer, batch=step_ctx.batch, parallel=par,
            num_microbatches=args.num_microbatches, expected_local_batch=args.batch_size, seq_len=args.seq_len,
            aux_loss_coef=args.aux_loss_coef, shard_info=step_ctx.optimizer_state.shard_info,
            gather_moe_metrics_fn=gather_moe_metrics, apply_optimizer_step_fn=apply_step, sync_plugin=None,
            zero_grad_fn=lambda _: self.optimizer_runtime.zero_grad(step_ctx.optimizer_state),
            refresh_persistent_params_fn=refresh_persistent_lowbit_params, precision_controller=ctrl,
            precision_config=step_ctx.runtime_context.run_config.precision_config)
        return StepOutput(task_loss=t, aux_loss=a, total_loss=t + args.aux_loss_coef * a, drop_fraction=d,
                          counters={"objective_count": oc, "drop_count": dc})


@dataclass
class Train4PScheduleSelector:
    optimizer_runtime: Train4POptimizerRuntime

    def __post_init__(self) -> None:
        self._selector = DefaultScheduleSelector(
            non_pipeline_schedule=NonPipelineSchedule(step_fn=Train4PNonPipelineSchedule(self.optimizer_runtime).run_step),
            pipeline_schedule=Pipeline1F1BSchedule(step_fn=Train4PPipelineSchedule(self.optimizer_runtime).run_step))

    def select(self, ctx: RuntimeContext):
        return self._selector.select(ctx)


class Train4PCheckpointManager(NoOpCheckpointManager):
    """No-op unless --checkpoint-dir is given (then a DirectoryCheckpointManager)."""

    def __init__(self):
        self._impl = None

    def _get(self, ctx):
        args = ctx.run_config.args
        d = getattr(args, "checkpoint_dir", None)
        if d and self._impl is None:
            self._impl = DirectoryCheckpointManager(d, save_every=int(getattr(args, "save_every", 0)))
        return self._impl

    def load(self, *, model, optimizer_state, ctx) -> ResumeState:
        impl = self._get(ctx)
        return impl.load(model=model, optimizer_state=optimizer_state, ctx=ctx) if impl else ResumeState()

    def on_step_end(self, *, model, optimizer_state, state, ctx) -> None:
        impl = self._get(ctx)
        if impl:
            impl.on_step_end(model=model, optimizer_state=optimizer_state, state=state, ctx=ctx)

    def on_run_end(self, *, model, optimizer_state, state, ctx) -> None:
        impl = self._get(ctx)
        if impl:
            impl.on_run_end(model=model, optimizer_state=optimizer_state, state=state, ctx=ctx)


def build_train_4d_components() -> RuntimeComponents:
    ort = Train4POptimizerRuntime()
    return RuntimeComponents(bootstrap=Train4PBootstrap(), model_provider=Train4PModelProvider(),
                             data_provider=Train4PDataProvider(), optimizer_runtime=ort,
                             schedule_selector=Train4PScheduleSelector(optimizer_runtime=ort),
                             checkpoint_manager=Train4PCheckpointManager())


def setup_process_logging(rank: int) -> None:
    setup_logging(level="INFO" if rank == 0 else "WARNING", use_colors=False)


def main(argv=None) -> None:
    args = parse_args(argv)
    setup_process_logging(int(os.environ.get("RANK", "0")))
    RuntimeEngine().run(components=build_train_4d_components(), args=args)
