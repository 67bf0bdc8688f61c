"""The multi-rank logic of bench.py's DeepSeek-V2-Lite fp8 and GPT-1.3B fp4 configurations on CPU
(gloo, 2 ranks, tiny dimensions). DeepSeek: EP folded inside DP (every rank its own batch), dense
parameters replicated and sharded by ZeRO-1 over the world, expert parameters local to their rank.
GPT: DP replicas kept identical by the ZeRO-1 step while each rank trains on its own batch. 4-D: the
train_4d runtime components stepped by bench.py on 8 ranks (TP2 x PP2 x DP2, EP2 inside DP, ZeRO-2, 1F1B)."""
import os
import sys

import torch
import torch.multiprocessing as mp

from conftest import ROOT, free_port

DIMS = dict(vocab_size=128, hidden_size=64, num_attention_heads=4, num_key_value_heads=4, intermediate_size=128,
            q_lora_rank=32, kv_lora_rank=16, qk_nope_head_dim=8, qk_rope_head_dim=8, v_head_dim=8,
            moe_intermediate_size=32, n_routed_experts=4, num_experts_per_tok=2, n_shared_experts=1,
            max_position_embeddings=64)


def _worker(rank, world, port, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port))
        sys.path.insert(0, ROOT)
        import argparse

        import torch.distributed as dist

        import bench

        dist.init_process_group("gloo", rank=rank, world_size=world)
        args = argparse.Namespace(layers=2)
        trainer, _ = bench.build_dsv2lite(args, rank, world, device="cpu", dims=DIMS)
        g = torch.Generator().manual_seed(rank)
        losses = []
        for _ in range(2):
            ids = torch.randint(0, 128, (2, 17), generator=g)
            losses.append(float(trainer.train_step(ids[:, :-1], ids[:, 1:])))
        model = trainer.model
        dense = [p.detach().clone() for p in model.parameters() if not getattr(p, "expert_model_parallel", False)]
        expert = [p.detach().clone() for p in model.parameters() if getattr(p, "expert_model_parallel", False)]
        same = True
        for t in dense:
            other = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(other, t)
            same = same and all(torch.equal(other[0], o) for o in other)
        ex = [torch.zeros_like(expert[0]) for _ in range(world)]
        dist.all_gather(ex, expert[0])
        q.put((rank, losses, same, not torch.equal(ex[0], ex[1]), len(expert) > 0, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, None, None, None, traceback.format_exc()))


def test_dsv2lite_ep_inside_dp_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for rank, losses, same, experts_differ, has_experts, err in res:
        assert err is None, f"rank {rank}:\n{err}"
        assert all(l == l and 0 < l < 20 for l in losses)
        assert same, "dense parameters diverged across ranks"
        assert has_experts and experts_differ, "expert parameters should be local to each rank"
    assert res[0][1] != res[1][1]  # each rank trains on its own batch


def _gpt_worker(rank, world, port, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port))
        sys.path.insert(0, ROOT)
        import argparse

        import torch.distributed as dist

        import bench

        dist.init_process_group("gloo", rank=rank, world_size=world)
        trainer, _ = bench.build_gpt_fp4(argparse.Namespace(layers=2), rank, world, device="cpu",
                                         dims=dict(hidden_size=64, num_attention_heads=4, intermediate_size=128,
                                                   vocab_size=128, max_position_embeddings=32))
        g = torch.Generator().manual_seed(rank)
        losses = []
        for _ in range(2):
            ids = torch.randint(0, 128, (2, 17), generator=g)
            losses.append(float(trainer.train_step(ids[:, :-1], ids[:, 1:])))
        same = True
        for p in trainer.model.parameters():
            other = [torch.zeros_like(p) for _ in range(world)]
            dist.all_gather(other, p.detach().contiguous())
            same = same and torch.equal(other[0], other[1])
        q.put((rank, losses, same, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def test_gpt_fp4_dp_zero1_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_gpt_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for rank, losses, same, err in res:
        assert err is None, f"rank {rank}:\n{err}"
        assert all(l == l and 0 < l < 20 for l in losses)
        assert same, "DP replicas diverged"
    assert res[0][1] != res[1][1]


def _4d_worker(rank, world, port, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port), OMP_NUM_THREADS="1")
        sys.path.insert(0, ROOT)
        import argparse

        import torch.distributed as dist

        import bench

        stepper, _ = bench.build_4d(argparse.Namespace(layers=4, seq=16), rank, world,
                                    dims=dict(hidden_size=64, num_heads=4, num_kv_heads=4, intermediate_size=128,
                                              moe_intermediate_size=64, vocab_size=128, q_lora_rank=32,
                                              kv_lora_rank=16, qk_nope_head_dim=8, qk_rope_head_dim=8,
                                              v_head_dim=8))
        g = torch.Generator().manual_seed(stepper.dp_rank)
        losses = []
        for _ in range(2):
            ids = torch.randint(0, 128, (8, 17), generator=g)
            losses.append(float(stepper.train_step(ids[:, :-1], ids[:, 1:])))
        q.put((rank, losses, stepper.dp_size, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def test_deepseek_4d_config_eight_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_4d_worker, args=(r, 8, port, q)) for r in range(8)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for rank, losses, dp, err in res:
        assert err is None, f"rank {rank}:\n{err}"
        assert dp == 2 and all(l == l and abs(l) < 100 for l in losses)


def _bench_line(monkeypatch, capsys, argv, world=1, ms=500.0):
    """Run bench.main() with the GPU parts stubbed: returns the JSON line rank 0 prints."""
    import json

    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    monkeypatch.setattr(bench, "init_dist", lambda n: (0, 0, world))
    clocks = {"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 5}
    e2e = {"value": 1.0, "unit": "tokens/s", "ms_per_step": ms, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4}
    monkeypatch.setattr(bench, "run_ours", lambda args, rank, local, w: (ms, 8, 1234, clocks, e2e, None))
    bench.main()
    out = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(out) == 1
    return json.loads(out[0])


def test_bench_json_line_contract(monkeypatch, capsys):
    """The default run's line carries every key the driver reads, with value = whole-job tokens / s."""
    line = _bench_line(monkeypatch, capsys, ["--steps", "3", "--warmup", "3"])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "clocks", "e2e", "gpu_launches"):
        assert k in line, k
    assert line["n_gpus"] == 1 and line["steps"] == 3 and line["warmup"] == 3 and line["higher_is_better"] is True
    assert line["value"] == 8 * 4096 / 0.5 and line["dtype"] == "bf16" and line["gpu_launches"] == 1234
    assert line["config"]["global_batch"] == 8 and line["config"]["seq_len"] == 4096
    assert line["config"]["parallelism"] == "tp1" and line["scaling"] == "strong"
    assert "flush" in line["config"]["l2"] or "L2" in line["config"]["l2"]
    line8 = _bench_line(monkeypatch, capsys, ["--gpus", "8"], world=8)
    assert line8["config"]["parallelism"] == "tp8+sp" and line8["value"] == 8 * 4096 / 0.5


def test_bench_json_line_other_configs(monkeypatch, capsys):
    gpt = _bench_line(monkeypatch, capsys, ["--config", "gpt1.3b-fp4-dp", "--gpus", "4"], world=4)
    assert gpt["scaling"] == "weak" and gpt["config"]["seq_len"] == 2048 and gpt["config"]["global_batch"] == 32
    assert gpt["value"] == 8 * 4 * 2048 / 0.5 and gpt["config"]["parallelism"] == "dp4+zero1"
    ds = _bench_line(monkeypatch, capsys, ["--config", "dsv2lite-fp8-ep", "--gpus", "8"], world=8)
    assert ds["config"]["parallelism"] == "ep8+dp8" and ds["value"] == 2 * 8 * 4096 / 0.5
    d4 = _bench_line(monkeypatch, capsys, ["--config", "deepseek-4d", "--gpus", "8"], world=8)
    assert d4["config"]["global_batch"] == 16 and d4["value"] == 16 * 2048 / 0.5


def test_bench_reference_arm_lines(monkeypatch, capsys):
    import json

    sys.path.insert(0, ROOT)
    import bench

    clocks = {"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 5}
    monkeypatch.setattr(bench, "run_reference", lambda args, rank, local, w: (1000.0, 8, 0, clocks, None))
    line = _bench_line(monkeypatch, capsys, ["--impl", "reference"])
    assert line["impl"] == "reference" and line["value"] == 8 * 4096 / 1.0 and line["metric"] == bench.METRIC
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--config", "deepseek-4d", "--gpus", "8"])
    monkeypatch.setattr(bench, "init_dist", lambda n: (0, 0, 8))
    bench.main()
    out = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(out) == 1 and out[0]["impl"] == "reference" and "unavailable" in out[0]


def test_clock_sampler_reads_nvidia_smi_and_summarises(tmp_path, monkeypatch):
    """The sampler polls nvidia-smi during the timed region; the summary keeps the median SM clock, the
    maximum clock and every throttle reason that was Active in any sample ("Not Active" is not a reason)."""
    sys.path.insert(0, ROOT)
    import bench

    rows = ["0, 1800, 1965, 950.1, 0x4, Not Active, Not Active, Not Active, Active",
            "0, 1900, 1965, 990.0, 0x0, Not Active, Not Active, Not Active, Not Active",
            "0, 1850, 1965, 999.9, 0x4, Not Active, Not Active, Not Active, Active"]
    fake = tmp_path / "nvidia-smi"
    counter = tmp_path / "n"
    counter.write_text("0")
    # a stand-in for nvidia-smi that answers the query with the next canned row
    fake.write_text("#!/bin/sh\n"
                    f"n=$(cat {counter}); echo $((n + 1)) > {counter}\n"
                    "case $((n % 3)) in\n" +
                    "".join(f"  {i}) echo '{r}';;\n" for i, r in enumerate(rows)) +
                    "esac\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ['PATH']}")
    s = bench.ClockSampler(0)
    s.start()
    import time

    deadline = time.time() + 20
    while len(s.samples) < 3 and time.time() < deadline:
        time.sleep(0.05)
    s.stop()
    got = s.summary()
    assert got["samples"] >= 3 and got["sm_max_mhz"] == 1965.0
    assert got["sm_mhz"] in (1800.0, 1850.0, 1900.0)
    assert got["reasons"] == ["sw_power_cap"]

    s = bench.ClockSampler(0)
    s.samples = [[x.strip() for x in rows[1].replace("Not Active, Not Active, Not Active, Not Active",
                                                         "Active, Not Active, Active, Not Active").split(",")]]
    assert s.summary()["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert bench.ClockSampler(0).summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
