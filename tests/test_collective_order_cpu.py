"""Debug collective-order check on gloo ranks (no GPU): matching sequences pass, a rank that issues a
different collective (or the same one with another shape) is reported on every rank before the
mismatched collective runs."""
import datetime
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from nano_train_b200.distributed.debug import CollectiveOrderError, checked_log, collective_order_check

    out = None
    orig = dist.all_reduce
    try:
        with collective_order_check():
            x = torch.ones(4)
            dist.all_reduce(x)
            dist.broadcast(x, 0)
            full = torch.empty(4 * world)
            dist.all_gather_into_tensor(full, x)
            if mode == "shape":
                dist.all_reduce(torch.ones(4 + rank))
            elif mode == "op":
                if rank == 0:
                    dist.all_reduce(torch.ones(4))
                else:
                    dist.broadcast(torch.ones(4), 0)
            dist.barrier()
            out = ("ok", len(checked_log()), float(x[0]))
    except CollectiveOrderError as e:
        out = ("order_error", str(e))
    assert dist.all_reduce is orig  # the check is removed on exit
    dist.destroy_process_group()
    q.put((rank, out))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    return res


def test_matching_sequence_passes():
    res = _run("same")
    for r in (0, 1):
        assert res[r][0] == "ok", res
        assert res[r][1] == 4  # all_reduce, broadcast, all_gather_into_tensor, barrier
        assert res[r][2] == 2.0


def test_shape_mismatch_is_reported_on_every_rank():
    res = _run("shape")
    for r in (0, 1):
        assert res[r][0] == "order_error", res
        assert "#4" in res[r][1] and "all_reduce" in res[r][1]


def test_operation_mismatch_is_reported_on_every_rank():
    res = _run("op")
    for r in (0, 1):
        assert res[r][0] == "order_error", res
    assert "all_reduce" in res[0][1] and "broadcast" in res[1][1]
