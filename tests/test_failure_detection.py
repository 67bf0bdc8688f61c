"""Failure detection without a GPU fault.

Host side (gloo ranks on CPU): a rank that raises before a collective, a rank
that never joins one (short process-group timeout), a rank that stops
heartbeating, non-finite loss, the host fault injector's configuration
(the kill-and-resume run is in test_train4d_cpu.py). Device side (GPU test): a bounded wait on a
flag that nothing sets returns with a status the host turns into
CommTimeoutError, and the context stays usable.
"""
import datetime
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port
from nano_train_b200.distributed.failure import (CommTimeoutError, HeartbeatMonitor, NonFiniteError,
                                                 PeerFailureError, assert_finite)


def _spawn(fn, world, *args, timeout=120, report=(0,)):
    """Run ``fn`` on ``world`` gloo ranks; collect the results of the ranks in ``report``
    (ranks that leave with os._exit may lose queued messages)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + timeout
    while any(r not in res for r in report):
        r, v = q.get(timeout=max(1, deadline - time.time()))
        res[r] = v
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def _init(rank, world, port, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _raise_worker(rank, world, port, q):
    _init(rank, world, port, 10)
    if rank == 1:
        os._exit(3)  # dies between steps, no collective in flight
    t0 = time.time()
    try:
        x = torch.ones(4)
        dist.all_reduce(x)
        q.put((rank, ("no error", time.time() - t0)))
    except Exception as e:  # noqa: BLE001 - any backend error is the detection
        q.put((rank, (type(e).__name__, time.time() - t0)))


def test_dead_rank_turns_into_error_not_hang():
    res = _spawn(_raise_worker, 2)
    kind, dt = res[0]
    assert kind != "no error"
    assert dt < 30


def _nojoin_worker(rank, world, port, q):
    _init(rank, world, port, 3)
    if rank == 1:
        time.sleep(12)  # never joins the collective within the timeout
        os._exit(0)
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((rank, ("no error", time.time() - t0)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, (type(e).__name__, time.time() - t0)))


def test_collective_timeout_bounds_a_missing_peer():
    res = _spawn(_nojoin_worker, 2)
    kind, dt = res[0]
    assert kind != "no error"
    assert dt < 11, dt


def _hb_worker(rank, world, port, q):
    _init(rank, world, port, 30)
    seen = []
    mon = HeartbeatMonitor(interval_s=0.2, timeout_s=1.5, on_failure=lambda d: seen.extend(d)).start()
    dist.barrier()
    if rank == 1:
        mon.stop()  # stops heartbeating (wedged), stays alive
        time.sleep(4)
        os._exit(0)
    time.sleep(3)
    try:
        mon.raise_if_peer_dead()
        q.put((rank, ("alive", seen)))
    except PeerFailureError as e:
        q.put((rank, (str(e), seen)))
    mon.stop()
    time.sleep(0.5)  # let the queue feeder flush before the hard exit
    os._exit(0)


def test_heartbeat_reports_silent_peer():
    res = _spawn(_hb_worker, 2)
    msg, seen = res[0]
    assert "ranks [1]" in msg
    assert seen == [1]


def test_assert_finite():
    assert assert_finite("loss", torch.tensor(1.5)) == 1.5
    with pytest.raises(NonFiniteError):
        assert_finite("loss", torch.tensor(float("nan")))
    with pytest.raises(NonFiniteError):
        assert_finite("grad_norm", float("inf"))


def test_host_fault_injector_configuration_and_raise_mode():
    from nano_train_b200.distributed.failure import (HostFaultInjector, InjectedFault, fault_point,
                                                     set_fault_injector)
    assert HostFaultInjector.from_env({}) is None
    inj = HostFaultInjector.from_env({"NTB_FAULT_STEP": "2", "NTB_FAULT_RANK": "1", "NTB_FAULT_MODE": "raise",
                                      "NTB_FAULT_POINT": "checkpoint_save"})
    assert (inj.point, inj.step, inj.rank, inj.mode) == ("checkpoint_save", 2, 1, "raise")
    with pytest.raises(ValueError):
        HostFaultInjector.from_env({"NTB_FAULT_STEP": "2", "NTB_FAULT_POINT": "forward"})
    with pytest.raises(ValueError):
        HostFaultInjector(point="step_end", step=1, mode="segfault")
    set_fault_injector(HostFaultInjector(point="step_end", step=3, rank=0, mode="raise"))
    try:
        fault_point("step_end", 2, 0)        # other step
        fault_point("step_end", 3, 1)        # other rank
        fault_point("checkpoint_save", 3, 0)  # other point
        with pytest.raises(InjectedFault, match="rank 0 at step_end of step 3"):
            fault_point("step_end", 3, 0)
    finally:
        set_fault_injector(None)
    fault_point("step_end", 3, 0)  # removed: no-op


@pytest.mark.gpu
def test_device_wait_on_unset_flag_returns_timeout_status():
    from nano_train_b200.distributed.failure import check_device
    from nano_train_b200.ops._ext import ext

    dev = torch.device("cuda", 0)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.time()
    ext().wait_flag(flag, 1, 200_000_000)  # 0.2 s budget, nothing ever sets the flag
    torch.cuda.synchronize(dev)
    assert time.time() - t0 < 5
    with pytest.raises(CommTimeoutError):
        check_device(0)
    # the context is still usable and the status was cleared
    flag.fill_(1)
    ext().wait_flag(flag, 1, 200_000_000)
    torch.cuda.synchronize(dev)
    check_device(0)
    assert float((torch.ones(8, device=dev) * 2).sum()) == 16.0
