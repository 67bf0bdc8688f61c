"""Flat-buffer mixed-precision AdamW with optional ZeRO-1/2 sharding.

Layout: the parameters of one group (same sharding domain, same weight-decay
class) are re-pointed into one contiguous bf16/fp32 buffer; each parameter
gets a ``main_grad`` fp32 view into a matching gradient buffer. The linear
layers' weight-gradient GEMMs accumulate into ``main_grad`` in their
epilogue; other parameters add their ``.grad`` through a post-accumulate
hook. A step is then, per buffer:

  no_shard     : all-reduce(grad)            -> fused AdamW on the whole buffer
  optim        : all-reduce(grad)            -> fused AdamW on this rank's shard -> all-gather(params)
  optim_grads  : reduce-scatter(grad)        -> fused AdamW on this rank's shard -> all-gather(params)

Gradient clipping and the data-parallel average are folded into a device
scalar that the AdamW kernel multiplies into the gradient, so a step has no
host synchronisation. fp32 master weights and moments exist only for the
local shard.

Tensor parallelism: groups flagged ``tp_replicated`` hold parameters that
every TP rank keeps whole (norm weights, row-parallel biases, positions).
Under sequence parallelism each TP rank only sees its sequence shard, so
their gradients are partial and are summed over ``tp_group`` before the
update. For the clipping norm, the squared sums of TP-sharded groups are
summed over ``tp_group`` while replicated groups count once.

Reference parity: src/runtime/optimizer_runtime.py:15-162 (PrecisionAdamW,
full-size master), src/distributed/zero.py:119-503 (per-parameter ZeRO-1/2
with one collective per parameter); here one collective and one kernel per
buffer.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Iterable, Optional

import torch
import torch.distributed as dist

from .. import ops
from . import comm

_ALIGN = 64  # elements; keeps every parameter view 128-byte aligned in bf16 and 256 in fp32


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class _Slot:
    param: torch.nn.Parameter
    offset: int
    numel: int


class FlatParamBuffer:
    """Contiguous storage of a parameter group and its fp32 gradient."""

    @staticmethod
    def padded_numel(params: list[torch.nn.Parameter], dp_size: int = 1) -> int:
        """Elements of the buffer FlatParamBuffer(params, dp_size=...) allocates."""
        seen, off = set(), 0
        for p in params:
            if id(p) not in seen:
                seen.add(id(p))
                off = _round_up(off + p.numel(), _ALIGN)
        return _round_up(max(off, 1), _ALIGN * dp_size)

    def __init__(self, params: list[torch.nn.Parameter], *, dp_size: int = 1, grad_dtype=torch.float32,
                 name: str = "buffer", storage: Optional[tuple] = None):
        """``storage``: optional caller-owned (param_data, grad_data) 1-D tensors of the padded size
        (e.g. views of peer-visible memory); zeroed here."""
        self.name = name
        seen = set()
        uniq = []
        for p in params:
            if id(p) not in seen:
                seen.add(id(p))
                uniq.append(p)
        self.params = uniq
        dtype = uniq[0].dtype if uniq else torch.float32
        device = uniq[0].device if uniq else torch.device("cpu")
        self.slots: list[_Slot] = []
        off = 0
        for p in uniq:
            if p.dtype != dtype:
                raise ValueError(f"{name}: mixed parameter dtypes {p.dtype} vs {dtype}")
            self.slots.append(_Slot(p, off, p.numel()))
            off = _round_up(off + p.numel(), _ALIGN)
        total = _round_up(max(off, 1), _ALIGN * dp_size)
        self.numel = total
        self.dtype = dtype
        if storage is None:
            self.param_data = torch.zeros(total, dtype=dtype, device=device)
            self.grad_data = torch.zeros(total, dtype=grad_dtype, device=device)
        else:
            self.param_data, self.grad_data = storage
            if (self.param_data.numel() != total or self.grad_data.numel() != total or self.param_data.dtype != dtype
                    or self.grad_data.dtype != grad_dtype):
                raise ValueError(f"{name}: storage must be ({total} x {dtype}, {total} x {grad_dtype})")
            self.param_data.zero_()
            self.grad_data.zero_()
        for s in self.slots:
            view = self.param_data[s.offset: s.offset + s.numel].view_as(s.param)
            view.copy_(s.param.data)
            s.param.data = view
            s.param.main_grad = self.grad_data[s.offset: s.offset + s.numel].view_as(s.param)

    def zero_grad(self) -> None:
        self.grad_data.zero_()


def _install_grad_hooks(params: Iterable[torch.nn.Parameter], on_ready=None) -> list:
    """``.grad`` -> ``main_grad`` after autograd accumulated it; ``on_ready(param)`` then runs, as it does
    when a native kernel accumulated straight into ``main_grad`` (``param._ntb_grad_ready_hook``)."""
    handles = []
    for p in params:
        if not p.requires_grad:
            continue

        def hook(param):
            if param.grad is not None:
                param.main_grad.add_(param.grad.to(param.main_grad.dtype))
                param.grad = None
                if on_ready is not None:
                    on_ready(param)

        handles.append(p.register_post_accumulate_grad_hook(hook))
        if on_ready is not None:
            p._ntb_grad_ready_hook = on_ready
    return handles


def _buckets(params: list, bucket_elems: int) -> list[list]:
    """Consecutive runs of ``params`` in reverse order (the backward produces the last parameters'
    gradients first), each about ``bucket_elems`` elements; bucket 0 holds the last parameters."""
    out, cur, n = [], [], 0
    for p in reversed(params):
        cur.append(p)
        n += p.numel()
        if n >= bucket_elems:
            out.append(list(reversed(cur)))
            cur, n = [], 0
    if cur:
        out.append(list(reversed(cur)))
    return out


class FlatAdamW:
    """AdamW over flat buffers; see the module docstring for the sharding strategies."""

    def __init__(self, param_groups: list[dict], *, lr: float = 1e-3, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.0, dp_group=None, strategy: str = "no_shard",
                 max_grad_norm: Optional[float] = None, grad_norm_group=None, tp_group=None,
                 sequence_parallel: bool = False, fused_dp: Optional[bool] = None,
                 bucket_mb: Optional[float] = None):
        """``fused_dp``: run the sharded step as the peer-memory kernels of parallel/zero_fused.py
        (None: whenever the group allows it; NTB_FUSED_ZERO=0 turns it off).

        ``bucket_mb`` (default NTB_ZERO_BUCKET_MB, else one buffer per group): with the peer-memory
        step, cut every group into buffers of about this many MB of fp32 gradient, last parameters
        first, so that ``overlap_next_backward`` can reduce-scatter each bucket as soon as the
        backward has produced it."""
        if strategy not in ("no_shard", "optim", "optim_grads"):
            raise ValueError(f"unknown sharding strategy {strategy}")
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.dp_group = dp_group
        self.dp_size = comm.group_size(dp_group)
        self.dp_rank = comm.group_rank(dp_group)
        # One rank has nothing to shard, except when a one-rank group runs the peer-memory step
        # (comm.min_fused_ranks) so that its kernels can be checked on one GPU.
        self.strategy = strategy if self.dp_size >= comm.min_fused_ranks() else "no_shard"
        self.max_grad_norm = max_grad_norm
        self.grad_norm_group = grad_norm_group if grad_norm_group is not None else tp_group
        self.tp_group = tp_group
        self.sequence_parallel = bool(sequence_parallel) and comm.group_size(tp_group) > 1
        self.step_count = 0
        self.buffers: list[FlatParamBuffer] = []
        self.group_wd: list[float] = []
        self.group_replicated: list[bool] = []
        self.shards: list[dict] = []
        dp_for_pad = self.dp_size if self.strategy != "no_shard" else 1
        all_params = []
        groups = [(i, g, [p for p in g["params"] if p.requires_grad]) for i, g in enumerate(param_groups)]
        groups = [(i, g, ps) for i, g, ps in groups if ps]
        self._zsym = None
        fused = False
        if self.strategy != "no_shard" and fused_dp is not False and groups:
            from .zero_fused import fused_zero_available

            dts = [p.dtype for _, _, ps in groups for p in ps]
            fused = fused_zero_available(dp_group, dts, grad_norm_group=self.grad_norm_group) \
                and all(p.is_cuda for _, _, ps in groups for p in ps)
        if bucket_mb is None:
            bucket_mb = float(os.environ.get("NTB_ZERO_BUCKET_MB", "0") or 0)
        if fused and bucket_mb > 0:
            from .zero_fused import MAX_BUFFERS

            total = sum(p.numel() for _, _, ps in groups for p in ps)
            elems = max(int(bucket_mb * 2 ** 20 / 4), -(-total // max(1, MAX_BUFFERS - 2 * len(groups))))
            pos = {id(p): k for k, p in enumerate(p for _, _, ps in groups for p in ps)}
            groups = [(i, g, b) for i, g, ps in groups for b in _buckets(ps, elems)]
            # bucket order = expected readiness order: the backward finishes the last layers first
            groups.sort(key=lambda t: -max(pos[id(p)] for p in t[2]))
        if fused and len(groups) > 32:
            raise ValueError(f"the peer-memory ZeRO step takes at most 32 buffers, got {len(groups)} parameter groups")
        if fused:
            from .zero_fused import ZeroSymm

            self._zsym = ZeroSymm(dp_group, [FlatParamBuffer.padded_numel(ps, dp_for_pad) for _, _, ps in groups],
                                  groups[0][2][0].device)
        for bi, (i, g, params) in enumerate(groups):
            storage = self._zsym.views(bi) if self._zsym is not None else None
            name = g.get("name", f"group{i}") + (f".b{bi}" if fused and bucket_mb > 0 else "")
            buf = FlatParamBuffer(params, dp_size=dp_for_pad, name=name, storage=storage)
            self.buffers.append(buf)
            self.group_wd.append(g.get("weight_decay", weight_decay))
            self.group_replicated.append(bool(g.get("tp_replicated", False)))
            all_params.extend(params)
            if self.strategy == "no_shard":
                lo, hi = 0, buf.numel
            else:
                chunk = buf.numel // self.dp_size
                lo, hi = self.dp_rank * chunk, (self.dp_rank + 1) * chunk
            master = buf.param_data[lo:hi].float().clone()
            self.shards.append(dict(lo=lo, hi=hi, master=master, exp_avg=torch.zeros_like(master),
                                    exp_avg_sq=torch.zeros_like(master)))
        self._hooks = _install_grad_hooks(all_params, self._on_grad_ready if self._zsym is not None else None)
        # Overlap of the peer-memory reduce-scatter with the backward (overlap_next_backward).
        self._bucket_of = {id(p): bi for bi, buf in enumerate(self.buffers) for p in buf.params}
        self._armed = False
        self._calls: dict = {}        # notifications per parameter in the armed backward
        self._expected: Optional[dict] = None  # the same, learned from the previous armed backward
        self._bucket_done = [0] * len(self.buffers)
        self._side: Optional[torch.cuda.Stream] = None
        # torch-optimizer-style groups (one per buffer): schedulers set "lr" here.
        self.param_groups = [dict(params=buf.params, lr=float(lr), weight_decay=float(wd), betas=tuple(betas),
                                  eps=float(eps), name=buf.name) for buf, wd in zip(self.buffers, self.group_wd)]
        dev = self.buffers[0].param_data.device if self.buffers else torch.device("cpu")
        self._stats = torch.zeros(2, dtype=torch.float32, device=dev)
        self._stats_rep = torch.zeros(2, dtype=torch.float32, device=dev)
        self._scale = torch.ones(1, dtype=torch.float32, device=dev)
        self.last_grad_norm: Optional[torch.Tensor] = None

    # ------------------------------------------------------------------ overlap with the backward
    def overlap_next_backward(self) -> bool:
        """Reduce-scatter each bucket while the next backward still runs (the last micro-batch's
        backward before ``step``). A bucket is launched - in bucket order, on a side stream, after
        the gradients enqueued so far - once each of its parameters has been notified as many times
        as in the previous armed backward (so the first armed step only learns those counts and
        reduces everything in ``step``, as without overlap). Returns whether overlap is possible
        (the peer-memory step is in use)."""
        if self._zsym is None or os.environ.get("NTB_ZERO_OVERLAP", "0") != "1":
            return False
        self._armed = True
        self._calls = {}
        self._bucket_done = [0] * len(self.buffers)
        return True

    def _on_grad_ready(self, param) -> None:
        if not self._armed:
            return
        key = id(param)
        c = self._calls.get(key, 0) + 1
        self._calls[key] = c
        if self._expected is None or c != self._expected.get(key, -1):
            return
        bi = self._bucket_of.get(key)
        if bi is None:
            return
        self._bucket_done[bi] += 1
        # launch every complete bucket from the next one on, in order
        k = self._zsym.next_bucket
        while k < len(self.buffers) and self._bucket_done[k] == len(self.buffers[k].params):
            k += 1
        if k > self._zsym.next_bucket:
            if self._side is None:
                self._side = torch.cuda.Stream(device=self.buffers[0].param_data.device)
            self._side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._side):
                self._zsym.reduce_through(k - 1, self.shards, self.group_replicated, grid=32)

    def _finish_overlap(self) -> None:
        """Before the step: the side stream's reductions precede the update; learn or check counts."""
        if not self._armed:
            return
        self._armed = False
        if self._side is not None:
            torch.cuda.current_stream().wait_stream(self._side)
        if self._expected is None:
            self._expected = dict(self._calls)
            return
        early = [k for k, c in self._calls.items() if c > self._expected.get(k, c)]
        if early:
            # a bucket may have been reduced before all of its gradient arrived
            raise RuntimeError(f"{len(early)} parameters received more gradient contributions than in the "
                               "previous overlapped backward; overlap_next_backward needs the same graph every step")

    # ------------------------------------------------------------------ API
    def zero_grad(self, set_to_none: bool = True) -> None:
        for b in self.buffers:
            b.zero_grad()
        for b in self.buffers:
            for s in b.slots:
                s.param.grad = None

    def _reduce_grads(self) -> list[torch.Tensor]:
        """Returns, per buffer, the (summed over DP) gradient of this rank's shard."""
        out = []
        for buf, sh, rep in zip(self.buffers, self.shards, self.group_replicated):
            g = buf.grad_data
            if rep and self.sequence_parallel:
                dist.all_reduce(g, group=self.tp_group)
            if self.dp_size > 1:
                if self.strategy == "optim_grads":
                    shard = torch.empty(sh["hi"] - sh["lo"], dtype=g.dtype, device=g.device)
                    dist.reduce_scatter_tensor(shard, g, group=self.dp_group)
                    out.append(shard)
                    continue
                dist.all_reduce(g, group=self.dp_group)
            out.append(g[sh["lo"]: sh["hi"]])
        return out

    @property
    def fused_dp(self) -> bool:
        """True when the sharded step runs as the peer-memory kernels (no NCCL)."""
        return self._zsym is not None

    @torch.no_grad()
    def step(self, lr: Optional[float] = None) -> None:
        """One update. ``lr`` overrides the groups' learning rates for this step."""
        self.step_count += 1
        self._finish_overlap()
        if self._zsym is not None:
            for buf, rep in zip(self.buffers, self.group_replicated):
                if rep and self.sequence_parallel:
                    dist.all_reduce(buf.grad_data, group=self.tp_group)
            lrs = [float(pg["lr"]) if lr is None else float(lr) for pg in self.param_groups]
            self._zsym.step(self.shards, lrs, [float(pg["weight_decay"]) for pg in self.param_groups],
                            self.group_replicated, step=self.step_count, betas=self.betas, eps=self.eps,
                            inv_dp=1.0 / self.dp_size, max_norm=float(self.max_grad_norm or 0.0))
            self.last_grad_norm = self._zsym.grad_norm
            self._scale = self._zsym.scale
            return
        grads = self._reduce_grads()
        inv_dp = 1.0 / self.dp_size
        if self.max_grad_norm is not None and self.max_grad_norm > 0:
            self._stats.zero_()
            self._stats_rep.zero_()
            for g, rep in zip(grads, self.group_replicated):
                ops.grad_stats_(g.contiguous() if not g.is_contiguous() else g,
                                self._stats_rep if rep else self._stats)
            if self.strategy != "no_shard" and self.dp_size > 1:
                both = torch.cat([self._stats, self._stats_rep])
                dist.all_reduce(both, group=self.dp_group)
                self._stats.copy_(both[:2])
                self._stats_rep.copy_(both[2:])
            if self.grad_norm_group is not None and comm.group_size(self.grad_norm_group) > 1:
                dist.all_reduce(self._stats, group=self.grad_norm_group)
            self._stats.add_(self._stats_rep)
            norm = torch.sqrt(self._stats[0:1]) * inv_dp
            self.last_grad_norm = norm
            coef = torch.clamp(self.max_grad_norm / (norm + 1e-6), max=1.0)
            torch.mul(coef, inv_dp, out=self._scale)
        else:
            self._scale.fill_(inv_dp)
        for buf, sh, g, wd, pg in zip(self.buffers, self.shards, grads, self.group_wd, self.param_groups):
            pb = buf.param_data[sh["lo"]: sh["hi"]]
            bf16_out = pb if pb.dtype == torch.bfloat16 else None
            glr = float(pg["lr"]) if lr is None else float(lr)
            ops.adamw_flat_(sh["master"], sh["exp_avg"], sh["exp_avg_sq"], g, lr=glr, beta1=self.betas[0],
                            beta2=self.betas[1], eps=self.eps, weight_decay=float(pg["weight_decay"]), step=self.step_count,
                            param_bf16=bf16_out, grad_scale=self._scale)
            if bf16_out is None:
                pb.copy_(sh["master"])
            if self.strategy != "no_shard" and self.dp_size > 1:
                dist.all_gather_into_tensor(buf.param_data, pb.clone(), group=self.dp_group)

    @torch.no_grad()
    def grad_norm(self) -> torch.Tensor:
        """L2 norm of this rank's accumulated gradients (all buffers, before any clipping or DP
        reduction), as a device scalar: nothing is read back to the host."""
        sq = torch.zeros((), dtype=torch.float32, device=self._stats.device)
        for buf in self.buffers:
            sq += buf.grad_data.float().pow(2).sum()
        return sq.sqrt()

    def state_tensors(self) -> list[dict]:
        return self.shards

    # ------------------------------------------------------------------ checkpoint state
    def state_dict(self) -> dict:
        """This rank's optimizer state: fp32 master shard and moments per buffer, step, group LRs."""
        return {"format": "flat_adamw_v1", "step_count": self.step_count, "strategy": self.strategy,
                "dp_size": self.dp_size, "dp_rank": self.dp_rank,
                "buffers": [{"name": b.name, "numel": b.numel, "lo": sh["lo"], "hi": sh["hi"],
                             "master": sh["master"].detach().cpu().clone(),
                             "exp_avg": sh["exp_avg"].detach().cpu().clone(),
                             "exp_avg_sq": sh["exp_avg_sq"].detach().cpu().clone()}
                            for b, sh in zip(self.buffers, self.shards)],
                "param_groups": [{"lr": g["lr"], "weight_decay": g["weight_decay"]} for g in self.param_groups]}

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        if state.get("format") != "flat_adamw_v1":
            raise ValueError("not a FlatAdamW state dict")
        if len(state["buffers"]) != len(self.buffers):
            raise ValueError("optimizer state has a different number of buffers")
        for b, sh, st in zip(self.buffers, self.shards, state["buffers"]):
            if st["numel"] != b.numel or (st["lo"], st["hi"]) != (sh["lo"], sh["hi"]):
                raise ValueError(f"buffer {b.name}: layout or sharding differs from the checkpoint")
            sh["master"].copy_(st["master"])
            sh["exp_avg"].copy_(st["exp_avg"])
            sh["exp_avg_sq"].copy_(st["exp_avg_sq"])
            b.param_data[sh["lo"]: sh["hi"]].copy_(sh["master"])
            if self.strategy != "no_shard" and self.dp_size > 1:
                dist.all_gather_into_tensor(b.param_data, b.param_data[sh["lo"]: sh["hi"]].clone(),
                                            group=self.dp_group)
        self.step_count = int(state["step_count"])
        for g, st in zip(self.param_groups, state["param_groups"]):
            g["lr"] = float(st["lr"])
            g["weight_decay"] = float(st["weight_decay"])


def split_decay_groups(model: torch.nn.Module, weight_decay: float, *, split_tp_replicated: bool = False) -> list[dict]:
    """Matrices decay; biases, norm weights and 1-D params do not (reference: src/optimizer.py:12-55).

    With ``split_tp_replicated`` the groups are further split into TP-sharded
    parameters (marked ``tensor_model_parallel``) and TP-replicated ones
    (flagged ``tp_replicated`` for the optimizer).
    """
    groups: dict[tuple[bool, bool], list] = {}
    seen = set()
    for name, p in model.named_parameters():
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        nd = p.dim() < 2 or name.endswith(".bias") or "norm" in name or ".ln" in name or name.startswith("ln")
        rep = split_tp_replicated and not getattr(p, "tensor_model_parallel", False)
        groups.setdefault((nd, rep), []).append(p)
    out = []
    for (nd, rep), params in sorted(groups.items()):
        out.append(dict(params=params, weight_decay=0.0 if nd else weight_decay, tp_replicated=rep,
                        name=("no_decay" if nd else "decay") + ("_tp_replicated" if rep else "")))
    return out
