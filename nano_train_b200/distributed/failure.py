"""Failure detection: host-side heartbeats, process-group timeouts, device wait status.

Three layers, none of which needs a GPU fault to be exercised:

* ``HeartbeatMonitor`` - every rank writes a timestamp into the process
  group's key-value store from a daemon thread; ``dead_ranks()`` lists peers
  whose heartbeat is older than ``timeout_s``. A training loop calls
  ``raise_if_peer_dead()`` between steps (never with a kernel or collective
  in flight), so a crashed or wedged peer becomes a ``PeerFailureError`` on
  the host before the next launch instead of a hang inside a collective.
* Process-group timeouts - ``init_process_group(timeout=...)`` (the runtime's
  ``--dist-timeout-s``) bounds every collective on the host side.
* Device waits - every spin in the fused kernels (peer flags, arrival
  counters, mbarriers) is bounded by a %globaltimer budget; on expiry the
  kernel writes a code into a device status word and returns.
  ``check_device(device)`` reads and clears it and raises
  ``CommTimeoutError`` for communication waits.

Plus ``assert_finite`` (fail fast on non-finite loss / norms, reference:
src/trainer.py:1301-1304, 1371-1375), and ``HostFaultInjector``: faults made on
the host (a rank that exits like a crashed process, or raises) at named points
of the training loop, for recovery tests. The reference has no fault injection.
"""
from __future__ import annotations

import math
import os
import sys
import threading
import time
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


class PeerFailureError(RuntimeError):
    """A peer rank stopped heartbeating (crashed, killed or wedged)."""


class CommTimeoutError(RuntimeError):
    """A device-side communication wait ran out of its time budget."""


class NonFiniteError(RuntimeError):
    """A monitored scalar (loss, gradient norm, ...) is NaN or infinite."""


_COMM_CODES = {5: "peer wait timed out", 7: "flag wait timed out"}


def check_device(device: int = 0) -> None:
    """Read and clear the device status word; raise on a failed bounded wait."""
    from ..ops._ext import KernelStatusError, ext

    code = int(ext().read_and_clear_status(device))
    if code == 0:
        return
    if code in _COMM_CODES:
        raise CommTimeoutError(f"device {device}: {_COMM_CODES[code]} (status {code})")
    raise KernelStatusError(code)


def assert_finite(name: str, value) -> float:
    """Return ``value`` as a float; raise ``NonFiniteError`` if it is NaN/inf."""
    v = float(value.detach().float().item()) if torch.is_tensor(value) else float(value)
    if not math.isfinite(v):
        raise NonFiniteError(f"{name} is not finite: {v}")
    return v


def _default_store():
    from torch.distributed import distributed_c10d as c10d

    return c10d._get_default_store()


_active_monitor: Optional["HeartbeatMonitor"] = None


class HeartbeatMonitor:
    """Store-based liveness of the ranks of the default process group.

    ``start()`` launches a daemon thread that writes ``hb/<rank>`` every
    ``interval_s``. ``dead_ranks()`` lists peers whose beat has not changed for
    ``timeout_s`` seconds of this process's clock. ``on_failure`` (optional) is called from the
    thread with the list of dead ranks the first time one is seen (once armed).
    """

    def __init__(self, *, interval_s: float = 1.0, timeout_s: float = 10.0, store=None, rank: Optional[int] = None,
                 world_size: Optional[int] = None, prefix: str = "ntb_hb",
                 on_failure: Optional[Callable[[list[int]], None]] = None):
        self.interval_s = interval_s
        self.timeout_s = timeout_s
        self.store = store if store is not None else _default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world_size = dist.get_world_size() if world_size is None else world_size
        self.prefix = prefix
        self.on_failure = on_failure
        self._stop = threading.Event()
        self._armed = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._reported = False
        self._seen: dict[int, tuple[Optional[str], float]] = {}  # peer -> (last stored beat, local time seen)

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.beat()
                if self.on_failure is not None and not self._reported and self._armed.is_set():
                    dead = self.dead_ranks()
                    if dead:
                        self._reported = True
                        self.on_failure(dead)
            except Exception:  # the store itself went away: nothing more to report from here
                return
            self._stop.wait(self.interval_s)

    def start(self, arm: bool = True) -> "HeartbeatMonitor":
        """Beat now and from a daemon thread. With ``arm=False`` the thread does not call ``on_failure``
        until ``arm()`` (so ranks that start at different times can first meet at a barrier)."""
        global _active_monitor
        _active_monitor = self
        self.beat()
        if arm:
            self.arm()
        self._thread = threading.Thread(target=self._run, name="ntb-heartbeat", daemon=True)
        self._thread.start()
        return self

    def stop(self, done: bool = False) -> None:
        """Stop beating. ``done=True`` (a clean end of this rank's run) also records that in the store,
        so peers still finishing do not take the silence for a failure."""
        global _active_monitor
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval_s + 1)
        if done:
            try:
                self.store.set(self._key(self.rank), "done")
            except Exception:  # the store may already be gone at teardown
                pass
        if _active_monitor is self:
            _active_monitor = None

    def arm(self) -> None:
        """Start judging peers from now on: each peer's silence is counted from this moment at the earliest."""
        self._seen.clear()
        self._armed.set()

    def _raw(self, r: int) -> Optional[str]:
        try:
            key = self._key(r)
            return self.store.get(key).decode() if self.store.check([key]) else None
        except Exception:
            return None

    def last_beat(self, r: int) -> Optional[float]:
        key = self._key(r)
        try:
            if not self.store.check([key]):
                return None
            v = self.store.get(key).decode()
            return math.inf if v == "done" else float(v)
        except Exception:
            return None

    def dead_ranks(self) -> list[int]:
        """Peers whose stored beat has not changed for more than ``timeout_s`` by this process's clock
        (a peer's clock is never compared with ours, so hosts need not agree on the time); a peer that
        recorded a clean end is never dead, and a peer is first judged one call after it was first seen."""
        now = time.monotonic()
        dead = []
        for r in range(self.world_size):
            if r == self.rank:
                continue
            v = self._raw(r)
            if v == "done":
                continue
            seen = self._seen.get(r)
            if seen is None or seen[0] != v:
                self._seen[r] = (v, now)
            elif now - seen[1] > self.timeout_s:
                dead.append(r)
        return dead

    def raise_if_peer_dead(self) -> None:
        dead = self.dead_ranks()
        if dead:
            raise PeerFailureError(f"rank {self.rank}: no heartbeat from ranks {dead} for > {self.timeout_s}s")


EXIT_PEER_DEAD = 43


def fail_fast_monitor(timeout_s: float, *, interval_s: Optional[float] = None, exit_code: int = EXIT_PEER_DEAD,
                      **kw) -> HeartbeatMonitor:
    """A started ``HeartbeatMonitor`` that ends this process (``os._exit(exit_code)``, after a message on
    stderr) as soon as a peer has been silent for ``timeout_s``. A rank blocked in a collective with a dead
    or wedged peer then leaves after about ``timeout_s`` instead of the process-group timeout, and the
    launcher ends the job with a named culprit."""

    def _exit(dead: list[int]) -> None:
        print(f"heartbeat: rank {mon.rank}: no heartbeat from ranks {dead} for > {timeout_s}s; ending this process",
              file=sys.stderr, flush=True)
        os._exit(exit_code)

    mon = HeartbeatMonitor(interval_s=interval_s if interval_s is not None else max(0.05, min(1.0, timeout_s / 4)),
                           timeout_s=timeout_s, on_failure=_exit, **kw)
    mon.start(arm=False)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()  # every rank has beaten once before any rank starts judging
    mon.arm()
    return mon


# --------------------------------------------------------------------------- host fault injection
class InjectedFault(RuntimeError):
    """Raised by a ``HostFaultInjector`` in mode ``"raise"``."""


FAULT_POINTS = ("step_end", "checkpoint_save")


@dataclass
class HostFaultInjector:
    """Host-side fault at a named point of the training loop; nothing on the GPU is touched.

    Points: ``"step_end"`` - step ``step`` finished and its checkpoint hook ran, with no kernel or
    collective in flight; ``"checkpoint_save"`` - this rank's files of the checkpoint taken after
    ``step`` completed steps are written and the completion barrier is not yet reached (the directory
    stays without its ``COMPLETE`` marker). At the point, rank ``rank`` either leaves the process the way a
    crashed one does (``mode="exit"``: output flushed, then ``os._exit(exit_code)``, no teardown, so the
    peers see a dead rank), raises ``InjectedFault`` (``mode="raise"``), or wedges (``mode="stall"``: its
    heartbeat stops and it sleeps for ``stall_s`` seconds, then exits like ``"exit"``)."""

    point: str
    step: int
    rank: int = 0
    mode: str = "exit"
    exit_code: int = 17
    stall_s: float = 60.0

    def __post_init__(self) -> None:
        if self.point not in FAULT_POINTS:
            raise ValueError(f"fault point must be one of {FAULT_POINTS}, got {self.point!r}")
        if self.mode not in ("exit", "raise", "stall"):
            raise ValueError(f"fault mode must be 'exit', 'raise' or 'stall', got {self.mode!r}")

    @classmethod
    def from_env(cls, env=None) -> Optional["HostFaultInjector"]:
        """NTB_FAULT_STEP (required to enable), NTB_FAULT_POINT (default step_end), NTB_FAULT_RANK
        (default 0), NTB_FAULT_MODE (default exit), NTB_FAULT_STALL_S (default 60): an unmodified launch
        line can be failed from outside."""
        env = os.environ if env is None else env
        if not env.get("NTB_FAULT_STEP"):
            return None
        return cls(point=env.get("NTB_FAULT_POINT", "step_end"), step=int(env["NTB_FAULT_STEP"]),
                   rank=int(env.get("NTB_FAULT_RANK", "0")), mode=env.get("NTB_FAULT_MODE", "exit"),
                   stall_s=float(env.get("NTB_FAULT_STALL_S", "60")))

    def maybe_fail(self, point: str, step: int, rank: int) -> None:
        if (point, step, rank) != (self.point, self.step, self.rank):
            return
        msg = f"injected fault: rank {rank} at {point} of step {step}"
        if self.mode == "raise":
            raise InjectedFault(msg)
        import logging

        print(msg, file=sys.stderr)
        if self.mode == "stall":
            if _active_monitor is not None:
                _active_monitor.stop()
            sys.stderr.flush()
            time.sleep(self.stall_s)
        for h in logging.getLogger().handlers:
            h.flush()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(self.exit_code)


_injector: Optional[HostFaultInjector] = None
_injector_read = False


def set_fault_injector(injector: Optional[HostFaultInjector]) -> None:
    """Install (or with None remove) the process's injector; overrides the environment."""
    global _injector, _injector_read
    _injector, _injector_read = injector, True


def fault_point(point: str, step: int, rank: int) -> None:
    """Hook the runtime calls at each fault point; a no-op unless an injector names this point."""
    global _injector, _injector_read
    if not _injector_read:
        _injector, _injector_read = HostFaultInjector.from_env(), True
    if _injector is not None:
        _injector.maybe_fail(point, step, rank)
