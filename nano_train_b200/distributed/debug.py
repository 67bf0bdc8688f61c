"""Debug checks for distributed runs (off by default).

Collective order check: every rank must issue the same collectives in the same
order with the same shapes (the reference relies on this rule without
checking it: zero-filled gradients, identical hook order). With the check on,
each collective first compares a signature of (sequence number in its group,
operation, tensor shapes and dtypes) across the group with two tiny
reductions (MIN and MAX of the signature); a mismatch raises
``CollectiveOrderError`` on every rank, naming the sequence number and the
local operation, instead of letting the mismatched collective hang or
silently combine unrelated tensors. Point-to-point send/recv is not checked
(peers differ by design).

    from nano_train_b200.distributed.debug import collective_order_check
    with collective_order_check():
        ...   # or NTB_CHECK_COLLECTIVES=1 with enable_from_env()
"""
from __future__ import annotations

import contextlib
import hashlib
import os
import threading

import torch
import torch.distributed as dist

_CHECKED = ("all_reduce", "all_gather", "all_gather_into_tensor", "reduce_scatter_tensor", "broadcast",
            "all_to_all_single", "barrier", "reduce_scatter", "all_gather_object", "broadcast_object_list")


class CollectiveOrderError(RuntimeError):
    pass


class _State:
    def __init__(self):
        self.orig = {}
        self.seq: dict = {}
        self.local = threading.local()
        self.log: list = []


_STATE: _State | None = None


def _describe(args, kwargs) -> str:
    parts = []
    for a in list(args) + [v for k, v in sorted(kwargs.items()) if k not in ("group", "async_op")]:
        if isinstance(a, torch.Tensor):
            parts.append(f"T{tuple(a.shape)}{str(a.dtype)[6:]}")
        elif isinstance(a, (list, tuple)) and a and isinstance(a[0], torch.Tensor):
            parts.append("L[" + ",".join(f"{tuple(t.shape)}" for t in a) + "]")
        elif isinstance(a, (int, float, str, bool)) or a is None:
            parts.append(repr(a))
        elif isinstance(a, (list, tuple)):
            parts.append(f"list{len(a)}")
        else:
            parts.append(type(a).__name__)
    return ",".join(parts)


def _group_key(group):
    g = group if group is not None else dist.group.WORLD
    try:
        return tuple(dist.get_process_group_ranks(g))
    except Exception:  # pragma: no cover - non-standard groups
        return (id(g),)


def _check(name: str, args, kwargs):
    st = _STATE
    group = kwargs.get("group")
    if group is None and name in ("all_reduce", "broadcast", "reduce_scatter_tensor", "all_gather_into_tensor",
                                  "all_to_all_single", "reduce_scatter", "all_gather"):
        # positional group argument of the torch signatures
        pos = {"all_reduce": 2, "broadcast": 2, "reduce_scatter_tensor": 3, "all_gather_into_tensor": 2,
               "all_to_all_single": 4, "reduce_scatter": 3, "all_gather": 2}[name]
        if len(args) > pos and not isinstance(args[pos], (torch.Tensor, list, int)):
            group = args[pos]
    key = _group_key(group)
    seq = st.seq.get(key, 0) + 1
    st.seq[key] = seq
    desc = f"{name}({_describe(args, kwargs)})"
    h = int.from_bytes(hashlib.sha256(f"{seq}:{desc}".encode()).digest()[:7], "little")
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    lo = torch.tensor([h], dtype=torch.int64, device=dev)
    hi = lo.clone()
    st.orig["all_reduce"](lo, op=dist.ReduceOp.MIN, group=group)
    st.orig["all_reduce"](hi, op=dist.ReduceOp.MAX, group=group)
    st.log.append((key, seq, desc))
    if int(lo.item()) != int(hi.item()):
        raise CollectiveOrderError(
            f"rank {dist.get_rank()}: collective #{seq} in group {key} differs across ranks; "
            f"this rank called {desc}")


def _wrap(name):
    orig = _STATE.orig[name]

    def wrapper(*args, **kwargs):
        st = _STATE
        if st is not None and not getattr(st.local, "busy", False):
            st.local.busy = True
            try:
                _check(name, args, kwargs)
            finally:
                st.local.busy = False
        return orig(*args, **kwargs)

    wrapper.__wrapped__ = orig
    return wrapper


def enable() -> None:
    """Wrap the torch.distributed collectives with the order check (idempotent)."""
    global _STATE
    if _STATE is not None:
        return
    _STATE = _State()
    for name in _CHECKED:
        if hasattr(dist, name):
            _STATE.orig[name] = getattr(dist, name)
    for name in list(_STATE.orig):
        setattr(dist, name, _wrap(name))


def disable() -> None:
    global _STATE
    if _STATE is None:
        return
    for name, fn in _STATE.orig.items():
        setattr(dist, name, fn)
    _STATE = None


def enable_from_env() -> bool:
    if os.environ.get("NTB_CHECK_COLLECTIVES", "0") == "1":
        enable()
        return True
    return False


def checked_log() -> list:
    """(group ranks, sequence number, description) of every checked collective so far."""
    return list(_STATE.log) if _STATE is not None else []


@contextlib.contextmanager
def collective_order_check():
    enable()
    try:
        yield
    finally:
        disable()
