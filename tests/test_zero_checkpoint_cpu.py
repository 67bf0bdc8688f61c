"""ZeRO optimizer checkpoint format v2 on CPU: shard save/load round trip, signature / version /
recipe / world-size checks, and a 2-rank gloo ZeRO-2 run that matches plain AdamW on the averaged
gradient and resumes bit-identically from its checkpoint files.

Covers the behaviour of the reference's tests/test_zero_checkpoint_io.py (shard round trip and the
"signature mismatch" error) and the v2 file set (optimizer_nonparam.pt, optimizer_shard_rank{r}.pt,
optimizer_manifest.json)."""
import datetime
import json
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from conftest import free_port
from nano_train_b200.distributed.zero import (ZERO_CHECKPOINT_FORMAT_VERSION, DistributedOptimizerConfig,
                                              MegatronZeroOptimizer)


class _Tiny(nn.Module):
    def __init__(self, hidden=8):
        super().__init__()
        self.fc1 = nn.Linear(6, hidden)
        self.fc2 = nn.Linear(hidden, 4)
        self.expert = nn.Linear(hidden, hidden, bias=False)  # stands in for an expert weight (EDP domain)

    def forward(self, x):
        h = torch.tanh(self.fc1(x))
        return self.fc2(h + self.expert(h))


def _config(strategy="optim_grads", **kw):
    return DistributedOptimizerConfig(use_distributed_optimizer=True, data_parallel_sharding_strategy=strategy,
                                      learning_rate=1e-2, weight_decay=0.01, **kw)


def _opt(model, group=None, strategy="optim_grads", **kw):
    return MegatronZeroOptimizer(model, _config(strategy, **kw), group, group, {id(model.expert.weight)})


def _train(model, opt, steps, seed):
    g = torch.Generator().manual_seed(seed)
    for _ in range(steps):
        x, y = torch.randn(4, 6, generator=g), torch.randn(4, 4, generator=g)
        opt.zero_grad(set_to_none=True)
        nn.functional.mse_loss(model(x), y).backward()
        opt.step_with_ready_grads()


def _save(opt, path, rank=0, world=1):
    os.makedirs(path, exist_ok=True)
    torch.save(opt.state_dict(), os.path.join(path, "optimizer_nonparam.pt"))
    opt.save_parameter_state(str(path), rank=rank, world_size=world)
    with open(os.path.join(path, "optimizer_manifest.json"), "w") as f:
        json.dump(opt.build_checkpoint_manifest(rank=rank, world_size=world), f)


def test_shard_roundtrip_restores_identical_state_and_continues_identically(tmp_path):
    torch.manual_seed(11)
    model = _Tiny()
    opt = _opt(model)
    _train(model, opt, 3, seed=1)
    ckpt = tmp_path / "ckpt"
    _save(opt, ckpt)
    assert sorted(os.listdir(ckpt)) == ["optimizer_manifest.json", "optimizer_nonparam.pt",
                                        "optimizer_shard_rank0.pt"]
    man = json.loads((ckpt / "optimizer_manifest.json").read_text())
    assert man["format_version"] == ZERO_CHECKPOINT_FORMAT_VERSION == 2
    assert man["parameter_signature_hash"] == opt.parameter_signature_hash()
    assert man["files"] == {"nonparam": "optimizer_nonparam.pt", "shard": "optimizer_shard_rank0.pt"}

    torch.manual_seed(99)  # different initial weights: everything must come from the checkpoint
    model2 = _Tiny()
    opt2 = _opt(model2)
    opt2.load_state_dict(torch.load(ckpt / "optimizer_nonparam.pt", weights_only=False))
    opt2.load_parameter_state(str(ckpt), rank=0, world_size=1)
    a = opt.get_parameter_state_dp_zero(include_tensors=True)
    b = opt2.get_parameter_state_dp_zero(include_tensors=True)
    assert a["global_step"] == b["global_step"] == 3
    for name, rec in a["parameters"].items():
        got = b["parameters"][name]
        assert got["step"] == rec["step"] == 3
        assert got["is_expert_param"] == (name == "expert.weight")
        for k in ("master_param", "exp_avg", "exp_avg_sq"):
            assert torch.equal(rec[k], got[k]), (name, k)

    # the module weights follow the master copy once the restored optimizer steps
    model2.load_state_dict(model.state_dict())
    _train(model, opt, 2, seed=5)
    _train(model2, opt2, 2, seed=5)
    for (n, p), (_, q) in zip(model.named_parameters(), model2.named_parameters()):
        assert torch.equal(p, q), n


def test_signature_mismatch_raises(tmp_path):
    opt = _opt(_Tiny(hidden=8))
    opt.save_parameter_state(str(tmp_path), rank=0, world_size=1)
    other = _opt(_Tiny(hidden=10))
    with pytest.raises(ValueError, match="signature mismatch"):
        other.load_parameter_state(str(tmp_path), rank=0, world_size=1)


def test_version_recipe_world_size_and_missing_file_checks(tmp_path):
    opt = _opt(_Tiny())
    state = opt.state_dict()
    with pytest.raises(ValueError, match="format version"):
        _opt(_Tiny()).load_state_dict({**state, "format_version": 1})
    with pytest.raises(ValueError, match="recipe"):
        _opt(_Tiny(), precision_recipe_name="fp8_deepseek").load_state_dict(state)
    opt.save_parameter_state(str(tmp_path), rank=0, world_size=1)
    with pytest.raises(ValueError, match="world_size mismatch"):
        _opt(_Tiny()).load_parameter_state(str(tmp_path), rank=0, world_size=2)
    with pytest.raises(FileNotFoundError):
        _opt(_Tiny()).load_parameter_state(str(tmp_path), rank=1, world_size=1)
    with pytest.raises(ValueError, match="sharded strategies"):
        _opt(_Tiny(), strategy="no_shard")


def test_nonparam_state_restores_hyperparameters():
    opt = _opt(_Tiny())
    opt.param_groups[0]["lr"] = 3e-4
    opt._global_step = 17
    opt2 = _opt(_Tiny())
    opt2.load_state_dict(opt.state_dict())
    assert opt2.param_groups[0]["lr"] == 3e-4 and opt2._global_step == 17


def _zero_worker(rank, world, port, path, strategy, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    rs_calls = []
    if strategy == "optim_grads_rs_fault":
        # the reduce-scatter fails (host-side fault): the optimizer falls back to all-reduce + slice for good
        strategy = "optim_grads"

        def failing_reduce_scatter(*a, **k):
            rs_calls.append(1)
            raise RuntimeError("injected reduce-scatter failure")

        dist.reduce_scatter_tensor = failing_reduce_scatter
    try:
        torch.manual_seed(3)
        model = _Tiny(hidden=7)  # odd sizes: the last shard of every parameter is ragged
        ref = _Tiny(hidden=7)
        ref.load_state_dict(model.state_dict())
        opt = _opt(model, dist.group.WORLD, strategy)
        ref_opt = torch.optim.AdamW(ref.parameters(), lr=1e-2, weight_decay=0.01)
        shard_sizes = {n: (m.shard_start, m.shard_end) for n, m in opt._meta_by_name.items()}
        g = torch.Generator().manual_seed(7)
        for _ in range(3):
            xs = [torch.randn(4, 6, generator=g) for _ in range(world)]
            ys = [torch.randn(4, 4, generator=g) for _ in range(world)]
            opt.zero_grad()
            nn.functional.mse_loss(model(xs[rank]), ys[rank]).backward()
            opt.step_with_ready_grads()
            ref_opt.zero_grad()
            (sum(nn.functional.mse_loss(ref(x), y) for x, y in zip(xs, ys)) / world).backward()
            ref_opt.step()
        err = max(float((p - r).abs().max()) for p, r in zip(model.parameters(), ref.parameters()))
        n_rs = len(rs_calls)  # reduce-scatter attempts of the first optimizer over its three steps

        opt.save_checkpoint_files(path)
        dist.barrier()
        torch.manual_seed(100 + rank)
        model2 = _Tiny(hidden=7)
        opt2 = _opt(model2, dist.group.WORLD, strategy)
        opt2.load_checkpoint_files(path)  # also re-materialises the parameters from the shards
        same_params = all(torch.equal(p, r) for p, r in zip(model.parameters(), model2.parameters()))
        x, y = torch.randn(4, 6, generator=g), torch.randn(4, 4, generator=g)
        for m, o in ((model, opt), (model2, opt2)):
            o.zero_grad()
            nn.functional.mse_loss(m(x), y).backward()
            o.step_with_ready_grads()
        same_after = all(torch.equal(p, r) for p, r in zip(model.parameters(), model2.parameters()))
        q.put((rank, ("ok", err, same_params, same_after, shard_sizes, n_rs, opt._reduce_scatter_fallback)))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, ("error", repr(e))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("strategy", ["optim", "optim_grads", "optim_grads_rs_fault"])
def test_two_rank_zero_matches_adamw_and_resumes_from_files(tmp_path, strategy):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_zero_worker, args=(r, world, port, str(tmp_path), strategy, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    for r in range(world):
        assert res[r][0] == "ok", res[r]
        _, err, same_params, same_after, shards, rs_calls, fallback = res[r]
        assert err < 1e-5, err
        assert same_params and same_after
        if strategy == "optim_grads_rs_fault":
            assert fallback and rs_calls == 1, (fallback, rs_calls)  # sticky: never retried
    # the two ranks own disjoint halves (ceil-sized chunks, ragged last) of every parameter
    for name, (s0, e0) in res[0][4].items():
        s1, e1 = res[1][4][name]
        assert s0 == 0 and e0 == s1 and e1 >= e0
    files = sorted(os.listdir(tmp_path))
    assert files == ["optimizer_manifest.json", "optimizer_manifest_rank1.json", "optimizer_nonparam.pt",
                     "optimizer_shard_rank0.pt", "optimizer_shard_rank1.pt"]


def test_corrupted_shard_file_fails_the_load_and_leaves_the_state_alone(tmp_path):
    """A truncated shard file (a host-side corruption) makes the load raise; the optimizer that tried to
    load keeps its own state instead of a partly restored one."""
    torch.manual_seed(5)
    model = _Tiny()
    opt = _opt(model)
    _train(model, opt, 2, seed=3)
    _save(opt, tmp_path)
    shard = tmp_path / "optimizer_shard_rank0.pt"
    data = shard.read_bytes()
    shard.write_bytes(data[: len(data) // 2])
    other = _opt(_Tiny())
    before = other.get_parameter_state_dp_zero(include_tensors=True)
    with pytest.raises(Exception):
        other.load_parameter_state(str(tmp_path), rank=0, world_size=1)
    after = other.get_parameter_state_dp_zero(include_tensors=True)
    for name, rec in before["parameters"].items():
        for k in ("master_param", "exp_avg", "exp_avg_sq"):
            assert torch.equal(rec[k], after["parameters"][name][k]), (name, k)
