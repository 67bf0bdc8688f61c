"""Non-interleaved 1F1B pipeline parallelism over NCCL (or gloo) point-to-point.

Schedule, tags and loss handling follow the reference
(src/runtime/pipeline.py:26-487): warm-up of ``min(pp - rank - 1, M)``
forwards, steady one-forward-one-backward, cool-down backwards; activations
[B_mb, S, H] and their gradients travel between neighbouring stages with tags
10000+mb / 20000+mb, labels go from the first to the last stage (tag
30000+mb); the last stage computes CE / M (+ aux * coef / M) and non-last
stages back-propagate ``[output, aux]`` with ``[dY, coef / M * loss_scale]``.

Issue order. NCCL ignores tags: between one pair of ranks it matches sends
and receives of one direction in the order they were issued. With PP = 2 the
first stage is also the last stage's previous stage, so the label and the
activation of a micro-batch travel the same pair in the same direction. Every
sender therefore issues, per micro-batch, the label first and the activation
second, and every receiver posts its receives of a micro-batch through
``_post_stage_inputs`` in that same order (label, then activation), early
posting (``NTB_PP_PREFETCH=1``) included. Gradients travel the other
direction and are matched on their own.

Receives are posted as non-blocking requests. Posting the next micro-batch's
receives early (``NTB_PP_PREFETCH=1``) lets the transfer run under the current
micro-batch's compute, but an early receive can sit in front of a send the
peer is waiting for; it is therefore off by default.

Losses and MoE statistics stay on the device during the step (no ``.item()``
per micro-batch); ``train_step_pipeline`` reads them once, after the schedule.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

import os

from ..precision.mixed_precision import dtype_alias_to_torch

PREFETCH = os.environ.get("NTB_PP_PREFETCH", "0") == "1"


def activation_tag(mb: int) -> int:
    return 10_000 + mb


def grad_tag(mb: int) -> int:
    return 20_000 + mb


def label_tag(mb: int) -> int:
    return 30_000 + mb


@dataclass
class PipelinePeers:
    prev_rank: Optional[int]
    next_rank: Optional[int]
    first_stage_rank: int
    last_stage_rank: int


@dataclass
class PipelineStepState:
    stage_inputs: list = field(default_factory=list)
    stage_outputs: list = field(default_factory=list)
    stage_aux_losses: list = field(default_factory=list)
    stage_labels: list = field(default_factory=list)
    label_send_reqs: list = field(default_factory=list)
    activation_send_reqs: list = field(default_factory=list)
    activation_send_buffers: list = field(default_factory=list)
    grad_send_reqs: list = field(default_factory=list)
    grad_send_buffers: list = field(default_factory=list)
    pending_act_recv: dict = field(default_factory=dict)
    pending_label_recv: dict = field(default_factory=dict)
    pending_grad_recv: dict = field(default_factory=dict)
    task_loss_sum: object = 0.0  # device scalars during the step, floats after finalize_pipeline_metrics
    aux_loss_sum: object = 0.0
    drop_sum: object = 0.0
    drop_count: int = 0


def resolve_pipeline_peers(parallel) -> PipelinePeers:
    def at(pp):
        return parallel.rank_from_coords(data_parallel_rank=parallel.data_parallel_rank,
                                         pipeline_model_parallel_rank=pp,
                                         tensor_model_parallel_rank=parallel.tensor_model_parallel_rank,
                                         expert_model_parallel_rank=parallel.expert_model_parallel_rank,
                                         context_parallel_rank=parallel.context_parallel_rank)

    r, n = parallel.pipeline_model_parallel_rank, parallel.pipeline_model_parallel_size
    return PipelinePeers(prev_rank=at(r - 1) if r > 0 else None, next_rank=at(r + 1) if r + 1 < n else None,
                         first_stage_rank=at(0), last_stage_rank=at(n - 1))


def prepare_microbatches(batch, model, expected_local_batch: int, num_microbatches: int, device):
    if not model.is_first_pp_stage:
        return [None] * num_microbatches
    if batch is None:
        raise ValueError("batch is required on first PP stage")
    ids = batch["input_ids"].to(device, non_blocking=True)
    if ids.size(0) != expected_local_batch:
        raise ValueError("Observed local batch size differs from expected fixed pipeline shape. "
                         "Adjust num_samples/batch_size to keep full batches.")
    return list(torch.chunk(ids, num_microbatches, dim=0))


def _post_stage_inputs(state, mb, model, peers, shape, dtype, device):
    """Post this stage's receives of micro-batch ``mb``: the label (last stage only) before the
    activation (non-first stages), the order in which the senders issue them."""
    if model.is_last_pp_stage and not model.is_first_pp_stage and mb not in state.pending_label_recv:
        lab = torch.empty(shape[:2], dtype=torch.long, device=device)
        state.pending_label_recv[mb] = (lab, dist.irecv(lab, src=peers.first_stage_rank, tag=label_tag(mb)))
    if not model.is_first_pp_stage and mb not in state.pending_act_recv:
        if peers.prev_rank is None:
            raise RuntimeError("Missing previous PP rank")
        buf = torch.empty(shape, device=device, dtype=dtype)
        state.pending_act_recv[mb] = (buf, dist.irecv(buf, src=peers.prev_rank, tag=activation_tag(mb)))


def _post_grad_recv(state, mb, shape, dtype, device, src):
    if mb in state.pending_grad_recv:
        return
    buf = torch.empty(shape, device=device, dtype=dtype)
    state.pending_grad_recv[mb] = (buf, dist.irecv(buf, src=src, tag=grad_tag(mb)))


def pipeline_forward_microbatch(microbatch_idx: int, model, microbatches, peers: PipelinePeers,
                                state: PipelineStepState, microbatch_batch_size: int, seq_len: int, hidden_size: int,
                                activation_dtype, device, gather_moe_metrics_fn, precision_controller=None,
                                num_microbatches: Optional[int] = None) -> None:
    label = None
    stage_input = None
    ctx = precision_controller.autocast_context() if precision_controller is not None else _null()
    shape = (microbatch_batch_size, seq_len, hidden_size)
    if model.is_first_pp_stage:
        ids = microbatches[microbatch_idx]
        if ids is None:
            raise RuntimeError("Missing first-stage microbatch")
        if not model.is_last_pp_stage:
            # Label before activation: the receiver posts them in this order (module docstring).
            state.label_send_reqs.append(dist.isend(ids.contiguous(), dst=peers.last_stage_rank,
                                                    tag=label_tag(microbatch_idx)))
        with ctx:
            out = model.forward_stage(input_ids=ids, hidden_states=None, attention_mask=None)
        if model.is_last_pp_stage:
            label = ids
    else:
        _post_stage_inputs(state, microbatch_idx, model, peers, shape, activation_dtype, device)
        if model.is_last_pp_stage:
            label, label_req = state.pending_label_recv.pop(microbatch_idx)
        buf, req = state.pending_act_recv.pop(microbatch_idx)
        req.wait()
        if PREFETCH and num_microbatches is not None and microbatch_idx + 1 < num_microbatches:
            _post_stage_inputs(state, microbatch_idx + 1, model, peers, shape, activation_dtype, device)
        stage_input = buf.requires_grad_(True)
        with ctx:
            out = model.forward_stage(input_ids=None, hidden_states=stage_input, attention_mask=None)
        if model.is_last_pp_stage:
            label_req.wait()
    aux, drop = gather_moe_metrics_fn(model, device=device)
    state.aux_loss_sum = state.aux_loss_sum + aux.detach().float().reshape(())
    state.drop_sum = state.drop_sum + drop
    state.drop_count += 1
    if not model.is_last_pp_stage:
        if peers.next_rank is None:
            raise RuntimeError("Missing next PP rank")
        payload = out.contiguous()
        state.activation_send_buffers.append(payload)
        state.activation_send_reqs.append(dist.isend(payload, dst=peers.next_rank, tag=activation_tag(microbatch_idx)))
    state.stage_inputs.append(stage_input)
    state.stage_outputs.append(out)
    state.stage_aux_losses.append(aux)
    state.stage_labels.append(label)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def pipeline_backward_microbatch(microbatch_idx: int, model, peers: PipelinePeers, state: PipelineStepState,
                                 num_microbatches: int, aux_loss_coef: float, microbatch_batch_size: int,
                                 seq_len: int, hidden_size: int, activation_dtype, device,
                                 precision_controller=None) -> None:
    stage_input = state.stage_inputs.pop(0)
    out = state.stage_outputs.pop(0)
    aux = state.stage_aux_losses.pop(0)
    labels = state.stage_labels.pop(0)
    if model.is_last_pp_stage:
        if labels is None:
            raise RuntimeError("Missing labels on last PP stage")
        if labels.size(0) == 0 or labels.size(1) < 2:
            task = out.sum() * 0.0
        else:
            task = F.cross_entropy(out[:, :-1, :].reshape(-1, out.size(-1)).float(), labels[:, 1:].reshape(-1))
        state.task_loss_sum = state.task_loss_sum + task.detach().float()
        scale = 1.0 / float(num_microbatches)
        total = task * scale + aux_loss_coef * scale * aux
        if precision_controller is None:
            total.backward()
        else:
            precision_controller.backward(total)
    else:
        if peers.next_rank is None:
            raise RuntimeError("Missing next PP rank")
        shape = (microbatch_batch_size, seq_len, hidden_size)
        _post_grad_recv(state, microbatch_idx, shape, activation_dtype, device, peers.next_rank)
        g, req = state.pending_grad_recv.pop(microbatch_idx)
        req.wait()
        if PREFETCH and microbatch_idx + 1 < num_microbatches:
            _post_grad_recv(state, microbatch_idx + 1, shape, activation_dtype, device, peers.next_rank)
        if aux.requires_grad:
            ls = 1.0
            if precision_controller is not None and precision_controller.uses_loss_scaling:
                ls = float(precision_controller.runtime_state.loss_scale)
            aux_scale = torch.tensor((aux_loss_coef / float(num_microbatches)) * ls, dtype=aux.dtype, device=device)
            torch.autograd.backward([out, aux], [g, aux_scale])
        else:
            torch.autograd.backward(out, g)
    if not model.is_first_pp_stage:
        if stage_input is None or stage_input.grad is None:
            raise RuntimeError("Expected stage input gradient on non-first PP stage")
        if peers.prev_rank is None:
            raise RuntimeError("Missing previous PP rank")
        payload = stage_input.grad.contiguous()
        state.grad_send_buffers.append(payload)
        state.grad_send_reqs.append(dist.isend(payload, dst=peers.prev_rank, tag=grad_tag(microbatch_idx)))


def execute_1f1b_schedule(parallel, num_microbatches: int, run_forward: Callable[[int], None],
                          run_backward: Callable[[int], None]) -> None:
    """Run this stage's forwards and backwards in 1F1B order (runtime/schedules/pipeline_1f1b.py)."""
    from ..runtime.schedules.pipeline_1f1b import one_f_one_b

    for kind, mb in one_f_one_b(parallel.pipeline_model_parallel_size, parallel.pipeline_model_parallel_rank,
                                num_microbatches):
        (run_forward if kind == "F" else run_backward)(mb)


def finalize_pipeline_sends(state: PipelineStepState) -> None:
    for r in state.activation_send_reqs + state.grad_send_reqs + state.label_send_reqs:
        r.wait()
    pending = (list(state.pending_label_recv.items()) + list(state.pending_act_recv.items())
               + list(state.pending_grad_recv.items()))
    for _, (_, r) in pending:
        r.wait()
    state.pending_label_recv.clear()
    state.pending_act_recv.clear()
    state.pending_grad_recv.clear()
    state.activation_send_buffers.clear()
    state.grad_send_buffers.clear()


def finalize_pipeline_metrics(state: PipelineStepState) -> None:
    """Turn the step's device-side sums into floats with one host read."""
    vals = [state.task_loss_sum, state.aux_loss_sum, state.drop_sum]
    dev = next((v for v in vals if isinstance(v, torch.Tensor)), None)
    if dev is None:
        return
    out = torch.stack([v.detach().float().reshape(()) if isinstance(v, torch.Tensor)
                       else torch.tensor(float(v), device=dev.device) for v in vals]).tolist()
    state.task_loss_sum, state.aux_loss_sum, state.drop_sum = out


def train_step_pipeline(model, optimizer, use_distributed_optimizer: bool, batch, parallel, num_microbatches: int,
                        expected_local_batch: int, seq_len: int, aux_loss_coef: float, shard_info,
                        gather_moe_metrics_fn, apply_optimizer_step_fn, sync_plugin, zero_grad_fn=None,
                        refresh_persistent_params_fn=None, precision_controller=None, precision_config=None):
    """One 1F1B step; returns (task_sum, aux_sum, drop_sum, objective_count, drop_count)."""
    if parallel.pipeline_model_parallel_size <= 1:
        raise ValueError("train_step_pipeline requires pipeline_model_parallel_size > 1")
    device = parallel.device
    act_dtype = (next(model.parameters()).dtype if precision_config is None
                 else dtype_alias_to_torch(precision_config.activation_dtype))
    hidden = model.config.hidden_size
    mbs = expected_local_batch // num_microbatches
    peers = resolve_pipeline_peers(parallel)
    state = PipelineStepState()
    if zero_grad_fn is None:
        optimizer.zero_grad(set_to_none=True)
    else:
        zero_grad_fn(optimizer)
    # The helpers are called by keyword: scripts and tests may substitute any of them.
    mbatches = prepare_microbatches(batch=batch, model=model, expected_local_batch=expected_local_batch,
                                    num_microbatches=num_microbatches, device=device)
    execute_1f1b_schedule(
        parallel=parallel, num_microbatches=num_microbatches,
        run_forward=lambda i: pipeline_forward_microbatch(
            microbatch_idx=i, model=model, microbatches=mbatches, peers=peers, state=state,
            microbatch_batch_size=mbs, seq_len=seq_len, hidden_size=hidden, activation_dtype=act_dtype,
            device=device, gather_moe_metrics_fn=gather_moe_metrics_fn, precision_controller=precision_controller,
            num_microbatches=num_microbatches),
        run_backward=lambda i: pipeline_backward_microbatch(
            microbatch_idx=i, model=model, peers=peers, state=state, num_microbatches=num_microbatches,
            aux_loss_coef=aux_loss_coef, microbatch_batch_size=mbs, seq_len=seq_len, hidden_size=hidden,
            activation_dtype=act_dtype, device=device, precision_controller=precision_controller))
    finalize_pipeline_sends(state)
    finalize_pipeline_metrics(state)
    should_step = True
    if precision_controller is not None:
        should_step = precision_controller.prepare_optimizer_step(model)
    if should_step:
        apply_optimizer_step_fn(model=model, optimizer=optimizer, use_distributed_optimizer=use_distributed_optimizer,
                                shard_info=shard_info, data_parallel_size=parallel.data_parallel_size,
                                expert_data_parallel_size=parallel.expert_data_parallel_size,
                                data_parallel_group=parallel.data_parallel_group,
                                expert_data_parallel_group=parallel.expert_data_parallel_group,
                                sync_plugin=sync_plugin)
        if refresh_persistent_params_fn is not None:
            refresh_persistent_params_fn(model)
    if precision_controller is not None:
        precision_controller.update_after_step(step_applied=should_step)
    return (state.task_loss_sum, state.aux_loss_sum, state.drop_sum,
            num_microbatches if model.is_last_pp_stage else 0, state.drop_count)
