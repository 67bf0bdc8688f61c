"""Optimizer runtime: dtype-configurable AdamW and the ZeRO-aware step policy.

``PrecisionAdamW`` keeps a full-size main copy of every parameter plus both
moments in configurable dtypes (reference: src/runtime/optimizer_runtime.py:15-116).
Here the main params and moments of all parameters live in flat buffers and
the update is one fused AdamW launch per buffer (fp32 state) instead of a
Python loop over parameters.

``step_with_sync_policy``: the distributed optimizer's
``step_with_ready_grads`` when it is enabled, else DP/EDP gradient
synchronisation followed by ``step`` (reference :127-162).
"""
from __future__ import annotations

from typing import Callable

import torch

from .. import ops
from ..precision.mixed_precision import dtype_alias_to_torch
from .contracts import OptimizerState


class PrecisionAdamW:
    def __init__(self, params, *, lr: float, weight_decay: float, betas: tuple[float, float], eps: float,
                 main_params_dtype: str, main_grads_dtype: str, exp_avg_dtype: str, exp_avg_sq_dtype: str) -> None:
        self._params = [p for p in params if p.requires_grad]
        self.param_groups = [{"params": self._params, "lr": float(lr), "weight_decay": float(weight_decay),
                              "betas": tuple(betas), "eps": float(eps)}]
        self._mp = dtype_alias_to_torch(main_params_dtype)
        self._mg = dtype_alias_to_torch(main_grads_dtype)
        self._ea = dtype_alias_to_torch(exp_avg_dtype)
        self._es = dtype_alias_to_torch(exp_avg_sq_dtype)
        self._global_step = 0
        self.state: dict = {}
        # Flat storage per device (parameters may live on several devices only in unusual setups).
        self._flat: dict = {}
        by_dev: dict = {}
        for p in self._params:
            by_dev.setdefault(p.device, []).append(p)
        for dev, ps in by_dev.items():
            n = sum(p.numel() for p in ps)
            master = torch.empty(n, dtype=self._mp, device=dev)
            ea = torch.zeros(n, dtype=self._ea, device=dev)
            es = torch.zeros(n, dtype=self._es, device=dev)
            off = 0
            for p in ps:
                k = p.numel()
                master[off: off + k].copy_(p.detach().reshape(-1).to(self._mp))
                self.state[p] = {"step": 0, "main_param": master[off: off + k].view_as(p),
                                 "exp_avg": ea[off: off + k].view_as(p), "exp_avg_sq": es[off: off + k].view_as(p)}
                off += k
            self._flat[dev] = (ps, master, ea, es)

    # ------------------------------------------------------------------ checkpoint state
    def state_dict(self) -> dict:
        """Main params, moments and per-parameter step counts (flat, in parameter order)."""
        flat = []
        for dev, (ps, master, ea, es) in self._flat.items():
            flat.append({"main_param": master.detach().cpu().clone(), "exp_avg": ea.detach().cpu().clone(),
                         "exp_avg_sq": es.detach().cpu().clone(),
                         "steps": [int(self.state[p]["step"]) for p in ps], "numel": [p.numel() for p in ps]})
        g0 = self.param_groups[0]
        return {"format": "precision_adamw_v1", "global_step": self._global_step, "flat": flat,
                "param_groups": [{k: v for k, v in g0.items() if k != "params"}]}

    def load_state_dict(self, state: dict) -> None:
        if state.get("format") != "precision_adamw_v1":
            raise ValueError("not a PrecisionAdamW state dict")
        if len(state["flat"]) != len(self._flat):
            raise ValueError("optimizer state has a different number of device buffers")
        for (dev, (ps, master, ea, es)), st in zip(self._flat.items(), state["flat"]):
            if st["numel"] != [p.numel() for p in ps]:
                raise ValueError("optimizer state does not match the parameter layout")
            master.copy_(st["main_param"].to(master.dtype))
            ea.copy_(st["exp_avg"].to(ea.dtype))
            es.copy_(st["exp_avg_sq"].to(es.dtype))
            for p, n in zip(ps, st["steps"]):
                self.state[p]["step"] = int(n)
        self._global_step = int(state["global_step"])
        for k, v in state["param_groups"][0].items():
            self.param_groups[0][k] = v

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self._params:
            if p.grad is not None:
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.zero_()
            mg = getattr(p, "main_grad", None)
            if mg is not None:
                mg.zero_()

    @torch.no_grad()
    def step(self) -> bool:
        g0 = self.param_groups[0]
        lr, wd, eps = float(g0["lr"]), float(g0["weight_decay"]), float(g0["eps"])
        b1, b2 = (float(x) for x in g0["betas"])
        self._global_step += 1
        for dev, (ps, master, ea, es) in self._flat.items():
            grads = []
            have = False
            for p in ps:
                g = getattr(p, "main_grad", None)
                if g is None:
                    g = p.grad
                if g is None:
                    grads.append(torch.zeros(p.numel(), dtype=torch.float32, device=dev))
                else:
                    have = True
                    grads.append(g.detach().reshape(-1).to(self._mg).float())
            if not have:
                continue
            # Parameters without a gradient keep their state (the reference skips them).
            mask_none = [getattr(p, "main_grad", None) is None and p.grad is None for p in ps]
            step = None
            for p, skip in zip(ps, mask_none):
                if not skip:
                    self.state[p]["step"] = int(self.state[p]["step"]) + 1
                    step = self.state[p]["step"]
            flat_g = torch.cat(grads)
            if any(mask_none):
                keep = torch.cat([torch.full((p.numel(),), not s, dtype=torch.bool, device=dev)
                                  for p, s in zip(ps, mask_none)])
            else:
                keep = None
            if self._mp == self._ea == self._es == torch.float32 and keep is None:
                ops.adamw_flat_(master, ea, es, flat_g, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd,
                                step=step)
            else:
                w, m, v = master.float(), ea.float(), es.float()
                w0, m0, v0 = w.clone(), m.clone(), v.clone()
                ops.adamw_flat_(w, m, v, flat_g, lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=step)
                if keep is not None:
                    w = torch.where(keep, w, w0)
                    m = torch.where(keep, m, m0)
                    v = torch.where(keep, v, v0)
                master.copy_(w)
                ea.copy_(m)
                es.copy_(v)
            off = 0
            for p in ps:
                k = p.numel()
                p.data.copy_(master[off: off + k].view_as(p).to(p.dtype))
                off += k
        return True


def zero_grad_optimizer(state: OptimizerState) -> None:
    fn = getattr(state.optimizer, "zero_grad", None)
    if not callable(fn):
        raise TypeError("optimizer in OptimizerState does not implement zero_grad")
    fn(set_to_none=True)


def step_with_sync_policy(*, model: torch.nn.Module, state: OptimizerState, ctx,
                          synchronize_gradients_fn: Callable[..., None]) -> None:
    args = ctx.run_config.args
    if args.use_distributed_optimizer:
        fn = getattr(state.optimizer, "step_with_ready_grads", None)
        if not callable(fn):
            raise TypeError("Expected optimizer with step_with_ready_grads when use_distributed_optimizer=True")
        fn()
        return
    synchronize_gradients_fn(model=model, shard_info=state.shard_info,
                             data_parallel_size=ctx.parallel.data_parallel_size,
                             expert_data_parallel_size=ctx.parallel.expert_data_parallel_size,
                             data_parallel_group=ctx.parallel.data_parallel_group,
                             expert_data_parallel_group=ctx.parallel.expert_data_parallel_group)
    fn = getattr(state.optimizer, "step", None)
    if not callable(fn):
        raise TypeError("optimizer in OptimizerState does not implement step")
    fn()
