"""Checkpoint hooks for the runtime engine.

``NoOpCheckpointManager`` is the reference's default (src/runtime/checkpoint.py:13-44).
``DirectoryCheckpointManager`` actually saves and restores: model state,
optimizer state (ZeRO format v2 shards when the optimizer is sharded),
train cursors and RNG states, every ``save_every`` steps and at the end of
the run, and resumes from the newest complete checkpoint on ``load``.
"""
from __future__ import annotations

import json
import os
import random
from typing import Optional

import torch

from ..distributed.failure import fault_point
from .context import RuntimeContext, TrainState
from .contracts import OptimizerState, ResumeState


class NoOpCheckpointManager:
    def load(self, *, model, optimizer_state: OptimizerState, ctx: RuntimeContext) -> ResumeState:
        del model, optimizer_state, ctx
        return ResumeState()

    def on_step_end(self, *, model, optimizer_state, state: TrainState, ctx) -> None:
        del model, optimizer_state, state, ctx

    def on_run_end(self, *, model, optimizer_state, state: TrainState, ctx) -> None:
        del model, optimizer_state, state, ctx


def _rng_state() -> dict:
    st = {"torch": torch.get_rng_state(), "python": random.getstate()}
    if torch.cuda.is_available():
        st["cuda"] = torch.cuda.get_rng_state_all()
    return st


def _set_rng_state(st: dict) -> None:
    torch.set_rng_state(st["torch"])
    random.setstate(st["python"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(st["cuda"])


class DirectoryCheckpointManager:
    """Save/restore to ``root/step_{N}/`` (one model + optimizer file per rank).

    A checkpoint directory is complete when its ``COMPLETE`` marker exists;
    incomplete directories (a rank died mid-save) are ignored on load. A
    checkpoint records ``next_step``, the number of completed steps, which is
    where a resumed run starts.
    """

    def __init__(self, root: str, save_every: int = 0, keep_last: int = 2):
        self.root = root
        self.save_every = save_every
        self.keep_last = keep_last

    def _dir(self, step: int) -> str:
        return os.path.join(self.root, f"step_{step:08d}")

    def latest(self) -> Optional[str]:
        if not os.path.isdir(self.root):
            return None
        cands = sorted(d for d in os.listdir(self.root) if d.startswith("step_")
                       and os.path.exists(os.path.join(self.root, d, "COMPLETE")))
        return os.path.join(self.root, cands[-1]) if cands else None

    def save(self, *, model, optimizer_state: OptimizerState, state: TrainState, ctx: RuntimeContext,
             next_step: Optional[int] = None) -> str:
        """Save after ``next_step`` completed steps (default: the step ``state.global_step`` just finished)."""
        rank = ctx.parallel.rank
        world = ctx.parallel.world_size
        next_step = state.global_step + 1 if next_step is None else next_step
        d = self._dir(next_step)
        if os.path.exists(os.path.join(d, "COMPLETE")):
            return d  # already saved at this point (step-end save followed by the run-end save)
        os.makedirs(d, exist_ok=True)
        torch.save(model.state_dict(), os.path.join(d, f"model_rank{rank}.pt"))
        opt = optimizer_state.optimizer
        if hasattr(opt, "save_checkpoint_files"):
            opt.save_checkpoint_files(d)
        elif hasattr(opt, "state_dict"):
            torch.save(opt.state_dict(), os.path.join(d, f"optimizer_rank{rank}.pt"))
        torch.save({"train_state": vars(state).copy(), "next_step": next_step, "rng": _rng_state()},
                   os.path.join(d, f"meta_rank{rank}.pt"))
        fault_point("checkpoint_save", next_step, rank)
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.barrier()
        if rank == 0:
            with open(os.path.join(d, "COMPLETE"), "w") as f:
                json.dump({"next_step": next_step, "world_size": world}, f)
            self._prune()
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.barrier()
        return d

    def _prune(self) -> None:
        if self.keep_last <= 0:
            return
        cands = sorted(d for d in os.listdir(self.root) if d.startswith("step_"))
        import shutil

        for d in cands[:-self.keep_last]:
            shutil.rmtree(os.path.join(self.root, d), ignore_errors=True)

    def load(self, *, model, optimizer_state: OptimizerState, ctx: RuntimeContext) -> ResumeState:
        d = self.latest()
        if d is None:
            return ResumeState()
        rank = ctx.parallel.rank
        model.load_state_dict(torch.load(os.path.join(d, f"model_rank{rank}.pt"), map_location="cpu"))
        opt = optimizer_state.optimizer
        if hasattr(opt, "load_checkpoint_files"):
            opt.load_checkpoint_files(d)
        elif hasattr(opt, "load_state_dict") and os.path.exists(os.path.join(d, f"optimizer_rank{rank}.pt")):
            opt.load_state_dict(torch.load(os.path.join(d, f"optimizer_rank{rank}.pt"), map_location="cpu",
                                           weights_only=False))
        meta = torch.load(os.path.join(d, f"meta_rank{rank}.pt"), map_location="cpu", weights_only=False)
        _set_rng_state(meta["rng"])
        ts = meta["train_state"]
        return ResumeState(start_global_step=int(meta["next_step"]), start_epoch=int(ts["epoch"]),
                           pipeline_epoch=int(ts["pipeline_epoch"]), data_seed=ts.get("data_seed"))

    def on_step_end(self, *, model, optimizer_state, state: TrainState, ctx) -> None:
        if self.save_every > 0 and (state.global_step + 1) % self.save_every == 0:
            self.save(model=model, optimizer_state=optimizer_state, state=state, ctx=ctx)

    def on_run_end(self, *, model, optimizer_state, state: TrainState, ctx) -> None:
        # At run end ``state.global_step`` counts the completed steps.
        if self.save_every > 0:
            self.save(model=model, optimizer_state=optimizer_state, state=state, ctx=ctx,
                      next_step=state.global_step)
