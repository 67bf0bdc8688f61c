"""Topology tables, rank layout and argument validation (CPU, no process group).

Mirrors the reference's topology/validation unit tests: group tables are
computed for a virtual world with ``dist.new_group`` replaced by a recorder,
so no process group is needed.
"""
import argparse

import pytest

from nano_train_b200.distributed import topology as topo
from nano_train_b200.runtime.validation import parse_pp_layer_splits, validate_args


def _make(monkeypatch, world, rank, **sizes):
    created = []
    monkeypatch.setenv("RANK", str(rank))
    monkeypatch.setenv("WORLD_SIZE", str(world))
    monkeypatch.setenv("LOCAL_RANK", "0")
    monkeypatch.setattr(topo.dist, "is_initialized", lambda: True)
    monkeypatch.setattr(topo.dist, "new_group", lambda ranks, **kw: ("group", tuple(ranks)))
    monkeypatch.setattr(topo, "get_backend", lambda *a, **k: "gloo")
    t = topo.initialize_model_parallel(**sizes)
    return t


def test_rank_layout_ep_fastest_roundtrip():
    PP, TP, EP, CP = 2, 2, 2, 1
    seen = set()
    for dp in range(2):
        for pp in range(PP):
            for tp in range(TP):
                for ep in range(EP):
                    r = topo.rank_from_coords(dp, pp, tp, ep, PP, TP, EP)
                    assert topo.coords_from_rank(r, PP, TP, EP, CP) == (dp, pp, tp, ep, 0)
                    seen.add(r)
    assert seen == set(range(16))
    # EP is the fastest axis, then TP, then PP, then DP
    assert topo.rank_from_coords(0, 0, 0, 1, PP, TP, EP) == 1
    assert topo.rank_from_coords(0, 0, 1, 0, PP, TP, EP) == 2
    assert topo.rank_from_coords(0, 1, 0, 0, PP, TP, EP) == 4
    assert topo.rank_from_coords(1, 0, 0, 0, PP, TP, EP) == 8


def test_group_tables_world16(monkeypatch):
    t = _make(monkeypatch, 16, 5, tensor_model_parallel_size=2, pipeline_model_parallel_size=2,
              expert_model_parallel_size=2)
    # rank 5 = dp0 pp1 tp0 ep1
    assert (t.dp_rank, t.pp_rank, t.tp_rank, t.ep_rank) == (0, 1, 0, 1)
    assert t.data_parallel_size == 2 and t.expert_data_parallel_size == 4
    assert [0, 2] in t.tp_group_table and [5, 7] in t.tp_group_table
    assert [4, 5] in t.ep_group_table
    assert [1, 5] in t.pp_group_table
    assert [5, 13] in t.dp_group_table
    assert sorted([5, 7, 13, 15]) in [sorted(g) for g in t.expert_data_parallel_group_table]
    assert t.tp_group == ("group", (5, 7))
    assert t.pp_group == ("group", (1, 5))
    # every table partitions the world
    for table in (t.tp_group_table, t.ep_group_table, t.pp_group_table, t.dp_group_table,
                  t.expert_data_parallel_group_table):
        flat = sorted(r for g in table for r in g)
        assert flat == list(range(16))
    assert not t.is_first_pipeline_stage and t.is_last_pipeline_stage


def test_fold_dp_layout(monkeypatch):
    t = _make(monkeypatch, 8, 3, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
              expert_model_parallel_size=4, expert_layout="fold_dp")
    assert t.data_parallel_size == 8 and t.expert_model_parallel_size == 4
    assert t.ep_rank == 3
    assert [0, 1, 2, 3] in t.ep_group_table and [4, 5, 6, 7] in t.ep_group_table
    assert [3, 7] in t.expert_data_parallel_group_table


def test_fold_dp_rank_from_coords_round_trips_with_tp_and_pp(monkeypatch):
    """With EP inside DP the rank grid has no EP axis: every rank's own coordinates map back to it, and
    the broadcast sources of its replica groups (dp = 0) and its pipeline peers are members of them."""
    for r in range(8):
        t = _make(monkeypatch, 8, r, tensor_model_parallel_size=2, pipeline_model_parallel_size=2,
                  expert_model_parallel_size=2, expert_layout="fold_dp")
        me = t.rank_from_coords(t.data_parallel_rank, t.pipeline_model_parallel_rank, t.tensor_model_parallel_rank,
                                t.expert_model_parallel_rank, t.context_parallel_rank)
        assert me == r
        assert t.expert_model_parallel_rank == t.data_parallel_rank % 2
        src = t.rank_from_coords(0, t.pipeline_model_parallel_rank, t.tensor_model_parallel_rank, 0)
        assert any(src in g and r in g for g in t.data_parallel_group_table)
        other = t.rank_from_coords(t.data_parallel_rank, 1 - t.pipeline_model_parallel_rank,
                                   t.tensor_model_parallel_rank, t.expert_model_parallel_rank)
        assert any(other in g and r in g for g in t.pipeline_model_parallel_group_table)


def test_world_not_divisible(monkeypatch):
    with pytest.raises(ValueError, match="divisible"):
        _make(monkeypatch, 6, 0, tensor_model_parallel_size=4, pipeline_model_parallel_size=1,
              expert_model_parallel_size=1)


def _args(**kw):
    base = dict(tensor_model_parallel_size=1, pipeline_model_parallel_size=1, expert_model_parallel_size=1,
                context_parallel_size=1, expert_tensor_parallel_size=1, intermediate_size=256, num_heads=8,
                num_experts=8, seq_len=32, dropout=0.0, data_parallel_sharding_strategy="no_shard",
                use_distributed_optimizer=False, num_distributed_optimizer_instances=1, num_microbatches=1,
                batch_size=16, num_layers=5, expert_layout="separate")
    base.update(kw)
    return argparse.Namespace(**base)


@pytest.mark.parametrize("kw,world,msg", [
    (dict(tensor_model_parallel_size=3), 4, "divisible"),
    (dict(tensor_model_parallel_size=8), 4, "cannot exceed"),
    (dict(tensor_model_parallel_size=2, num_heads=7), 2, "num_heads"),
    (dict(num_experts=6, expert_model_parallel_size=4), 4, "num_experts"),
    (dict(context_parallel_size=2), 2, "context_parallel_size"),
    (dict(tensor_model_parallel_size=2, expert_model_parallel_size=2), 4, "disallows"),
    (dict(tensor_model_parallel_size=2, dropout=0.1), 2, "dropout"),
    (dict(data_parallel_sharding_strategy="optim_grads_params", use_distributed_optimizer=True), 1, "ZeRO-3"),
    (dict(data_parallel_sharding_strategy="optim"), 1, "use_distributed_optimizer"),
    (dict(use_distributed_optimizer=True), 1, "select sharding strategy"),
    (dict(batch_size=10, num_microbatches=4), 1, "divisible by num_microbatches"),
    (dict(seq_len=1), 1, "seq_len"),
])
def test_validation_messages(kw, world, msg):
    with pytest.raises(ValueError, match=msg):
        validate_args(_args(**kw), world, None)


def test_validation_accepts_and_fold_relaxes():
    validate_args(_args(tensor_model_parallel_size=2, pipeline_model_parallel_size=2), 8, None)
    validate_args(_args(tensor_model_parallel_size=2, expert_model_parallel_size=2, expert_layout="fold_dp"), 4,
                  None)


def test_pp_layer_splits():
    assert parse_pp_layer_splits(None) is None
    assert parse_pp_layer_splits(" ") is None
    assert parse_pp_layer_splits("0,2,5") == (0, 2, 5)
    with pytest.raises(ValueError):
        parse_pp_layer_splits("0,a")
    validate_args(_args(pipeline_model_parallel_size=2), 2, (0, 2, 5))
    for bad, msg in [((0, 5), "length"), ((1, 2, 5), "start with 0"), ((0, 2, 4), "end at"),
                     ((0, 5, 5), "strictly")]:
        with pytest.raises(ValueError, match=msg):
            validate_args(_args(pipeline_model_parallel_size=2), 2, bad)


def test_train_4d_parser_requires_the_canonical_parallel_flags():
    from nano_train_b200.runtime.train4d import parse_args

    with pytest.raises(SystemExit):
        parse_args([])
    a = parse_args(["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "2",
                    "--expert-model-parallel-size", "4", "--use-distributed-optimizer",
                    "--data-parallel-sharding-strategy", "optim"])
    assert (a.tensor_model_parallel_size, a.pipeline_model_parallel_size, a.expert_model_parallel_size) == (1, 2, 4)
    assert a.use_distributed_optimizer and a.data_parallel_sharding_strategy == "optim"


def test_train_4d_parser_takes_the_shared_precision_flags():
    import torch

    from nano_train_b200.precision.mixed_precision import resolve_precision_config
    from nano_train_b200.runtime.train4d import parse_args

    canon = ["--tensor-model-parallel-size", "1", "--pipeline-model-parallel-size", "1",
             "--expert-model-parallel-size", "1"]
    a = parse_args(canon + ["--fp8", "--fp8-backend", "emulated", "--fp8-format", "hybrid",
                            "--fp8-amax-history-len", "32", "--fp8-amax-compute-algo", "max"])
    cfg = resolve_precision_config(a, torch.device("cpu"))
    assert (cfg.mode, cfg.fp8_backend, cfg.fp8_format, cfg.fp8_amax_history_len, cfg.fp8_amax_compute_algo) == \
        ("fp8", "emulated", "hybrid", 32, "max")
    with pytest.raises(ValueError, match="At most one"):
        resolve_precision_config(parse_args(canon + ["--fp8", "--fp16"]), torch.device("cpu"))
    bad = parse_args(canon + ["--fp8"])
    bad.fp8_backend = "cublas"
    with pytest.raises(ValueError, match="--fp8-backend"):
        resolve_precision_config(bad, torch.device("cpu"))
