"""Scheduler, loss module, optimizer factory, dataset, monitoring math, model report and Trainer (CPU)."""
import math
import os

import pytest
import torch
import torch.nn.functional as F

from nano_train_b200 import monitoring as mon
from nano_train_b200.config import Config, ModelConfig, TrainingConfig, _NoOpPrecisionResolver
from nano_train_b200.dataset import SyntheticTokenDataset, TextDataset, create_dataloader
from nano_train_b200.losses import CrossEntropyLoss
from nano_train_b200.models.transformer import TransformerModel, llama3_8b_config
from nano_train_b200.optimizer import create_optimizer
from nano_train_b200.scheduler import CosineAnnealingScheduler
from nano_train_b200.trainer import Trainer
from nano_train_b200.utils.model_info import ParallelismAssumptions, dump_model_info, estimate


def _tiny_cfg(**kw):
    d = dict(param_dtype=torch.float32, param_device=torch.device("cpu"), precision_resolver=_NoOpPrecisionResolver(),
             hidden_size=32, num_layers=2, num_attention_heads=4, intermediate_size=64, vocab_size=64,
             max_position_embeddings=64, dropout=0.0)
    d.update(kw)
    return ModelConfig(**d)


def test_cosine_schedule():
    p = torch.nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1.0)
    s = CosineAnnealingScheduler(opt, warmup_steps=4, max_steps=12, min_lr=0.1)
    lrs = [s.step() for _ in range(14)]
    assert lrs[:4] == [0.25, 0.5, 0.75, 1.0]
    assert abs(lrs[7] - (0.1 + 0.45 * (1 + math.cos(math.pi * 0.5)))) < 1e-12
    assert abs(lrs[11] - 0.1) < 1e-12 and abs(lrs[13] - 0.1) < 1e-12
    st = s.state_dict()
    s2 = CosineAnnealingScheduler(opt, 4, 12, 0.1)
    s2.load_state_dict(st)
    assert s2.get_lr() == s.get_lr() and opt.param_groups[0]["lr"] == s.get_lr()
    with pytest.raises(ValueError):
        CosineAnnealingScheduler(opt, 12, 12)


def test_cross_entropy_module():
    torch.manual_seed(0)
    logits, t = torch.randn(2, 3, 9), torch.randint(0, 9, (2, 3))
    t[1, 1] = -100
    torch.testing.assert_close(CrossEntropyLoss()(logits, t), F.cross_entropy(logits.reshape(-1, 9), t.reshape(-1)))
    assert CrossEntropyLoss(reduction="none")(logits, t).shape == (2, 3)
    with pytest.raises(ValueError):
        CrossEntropyLoss()(logits, t[:, :2])


def test_create_optimizer_groups_and_step():
    torch.manual_seed(1)
    model = TransformerModel(_tiny_cfg())
    opt = create_optimizer(model, 1e-2, 0.1)
    names = {n for n, _ in model.named_parameters()}
    nd = {id(p) for g in opt.param_groups if g["weight_decay"] == 0.0 for p in g["params"]}
    for n, p in model.named_parameters():
        expect_nd = "bias" in n.lower() or "ln_" in n.lower()
        assert (id(p) in nd) == expect_nd, n
    ids = torch.randint(0, 64, (2, 8))
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    model.forward_loss(ids, ids).backward()
    opt.step()
    assert any(not torch.equal(before[n], p) for n, p in model.named_parameters())
    st = opt.state_dict()
    opt2 = create_optimizer(TransformerModel(_tiny_cfg()), 1e-2, 0.1)
    opt2.load_state_dict(st)
    assert opt2.step_count == 1
    assert names


def test_text_dataset(tmp_path):
    p = tmp_path / "t.txt"
    p.write_text("hello world, hello b200!" * 3)
    ds = TextDataset(str(p), max_seq_length=9)
    assert ds.pad_id == 0 and ds.chars[0] == "<pad>"
    item = ds[1]
    assert item["input_ids"].shape == (8,) and item["labels"].shape == (8,)
    assert torch.equal(item["input_ids"][1:], item["labels"][:-1])
    assert len(ds) == (len("hello world, hello b200!" * 3) - 9) // 4 + 1
    short = tmp_path / "s.txt"
    short.write_text("abc")
    it = TextDataset(str(short), max_seq_length=8)[0]
    assert (it["labels"] == -100).sum() == 5
    dl = create_dataloader(ds, 4)
    assert next(iter(dl))["input_ids"].shape == (4, 8)


def test_monitoring_math():
    assert mon.resolve_sentinel_blocks(12) == (0, 6, 11)
    assert mon.resolve_sentinel_blocks(1) == (0,)
    assert mon.resolve_sentinel_blocks(4, [5, 1, 1]) == (1,)
    assert mon.clip_coef(10.0, 1.0) == pytest.approx(1.0 / (10.0 + 1e-6))
    assert mon.clip_coef(0.5, 1.0) == 1.0 and mon.clip_coef(3.0, 0.0) == 1.0
    assert mon.global_update_ratio(0.1, grad_norm_pre_clip=2.0, clip_coef_value=0.5, param_norm=4.0) == \
        pytest.approx(0.025)
    assert mon.achieved_tflops(1e3, 8_000_000_000) == pytest.approx(48.0)
    assert mon.mfu(500.0, 2000.0) == 0.25
    h1 = mon.eval_artifact_hash(input_ids_bytes=b"ab", labels_bytes=b"cd", input_dtype="torch.int64",
                                labels_dtype="torch.int64", input_shape=(1, 2), labels_shape=(1, 2), vocab_size=10,
                                max_seq_length=3, seed=1)
    h2 = mon.eval_artifact_hash(input_ids_bytes=b"ab", labels_bytes=b"ce", input_dtype="torch.int64",
                                labels_dtype="torch.int64", input_shape=(1, 2), labels_shape=(1, 2), vocab_size=10,
                                max_seq_length=3, seed=1)
    assert h1 != h2 and len(h1) == 64


def test_model_report_llama8b(tmp_path):
    model = TransformerModel(llama3_8b_config(param_device=torch.device("meta"), sequence_parallel=False))
    info = dump_model_info(model, str(tmp_path / "r.md"), batch=8, seq_len=4096,
                           parallel=ParallelismAssumptions(tp=8))
    assert 8.0e9 < info.total_params < 8.1e9
    train = next(m for m in info.modes if m.mode == "train")
    assert train.flops == pytest.approx(6 * 32768 * (info.total_params - 128256 * 4096), rel=0.08)
    assert train.net_bytes > 0
    assert os.path.exists(tmp_path / "r.md") and os.path.exists(tmp_path / "r.json")
    for name in ("r_roofline.svg", "r_decode_sweep.svg"):  # dependency-free SVG charts beside the report
        svg = (tmp_path / name).read_text()
        assert svg.startswith("<svg") and svg.rstrip().endswith("</svg>") and "<polyline" in svg
    assert "r_roofline.svg" in (tmp_path / "r.md").read_text()


def test_trainer_runs_and_checkpoints(tmp_path):
    torch.manual_seed(0)
    mcfg = _tiny_cfg()
    cfg = Config(model=mcfg, training=TrainingConfig(batch_size=4, micro_batch_size=2, learning_rate=3e-3,
                                                     max_steps=12, warmup_steps=2, log_steps=4, eval_steps=6,
                                                     save_steps=6, clip_grad=1.0),
                 output_dir=str(tmp_path / "out"), log_dir=str(tmp_path / "logs"))
    cfg.monitoring.probe_steps = 6
    cfg.monitoring.update_ratio_steps = 4
    cfg.monitoring.opt_state_check_steps = 4
    ds = SyntheticTokenDataset(32, 16, 64, seed=0)
    tr = Trainer(TransformerModel(mcfg), cfg, create_dataloader(ds, 4), "cpu",
                 val_loader=create_dataloader(ds, 4, shuffle=False))
    out = tr.train()
    assert out["step"] == 12 and math.isfinite(out["loss"]) and "eval" in out
    ck = tmp_path / "out" / "checkpoint-step-12"
    for f in ("model.pt", "optimizer.pt", "scheduler.pt", "config.json", "trainer_state.json"):
        assert (ck / f).exists(), f
    tr2 = Trainer(TransformerModel(mcfg), cfg, create_dataloader(ds, 4), "cpu")
    assert tr2.load_checkpoint(str(ck)) == 12
    for (n, a), (_, b) in zip(tr.model.state_dict().items(), tr2.model.state_dict().items()):
        torch.testing.assert_close(a, b, msg=n)
    assert tr2.scheduler.current_step == 12


@pytest.mark.parametrize("script,args,expect", [
    ("examples/train_tp.py", ["--max_steps", "12", "--log_every", "5"], "step 10"),
    ("examples/train_ddp.py", ["--epochs", "1", "--num_samples", "128"], "mean loss"),
    ("examples/train_tp.py", ["--max_steps", "12", "--log_every", "5", "--fp8", "--fp8-backend", "emulated"],
     "step 10"),
    ("examples/train_ddp.py", ["--epochs", "1", "--num_samples", "128", "--fp4", "--fp4-backend", "emulated"],
     "mean loss"),
])
def test_examples_via_launcher(script, args, expect):
    import subprocess
    import sys

    from conftest import ROOT

    cmd = [sys.executable, "examples/launch.py", "--world-size", "2", "--backend", "gloo", "--script", script,
           "--script-args"] + args
    env = dict(os.environ, OMP_NUM_THREADS="1", MASTER_ADDR="127.0.0.1")
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert expect in p.stdout


def test_example_scripts_share_the_precision_flags(tmp_path):
    """Every training entry point takes the same precision flags (the reference's shared builder)."""
    import subprocess
    import sys

    from conftest import ROOT

    for script in ("train_mvp.py", "train_tp.py", "train_ddp.py", "train_4d.py"):
        out = subprocess.run([sys.executable, f"examples/{script}", "--help"], capture_output=True, text=True,
                             cwd=ROOT, timeout=120).stdout
        for flag in ("--fp8", "--fp4", "--fp8-backend", "--fp4-backend", "--precision-recipe", "--params-dtype"):
            assert flag in out, (script, flag)
    p = subprocess.run([sys.executable, "examples/train_mvp.py", "--max_steps", "2", "--seq_len", "64",
                        "--hidden_size", "64", "--num_layers", "1", "--batch_size", "2", "--fp4", "--fp4-backend",
                        "native", "--output_dir", str(tmp_path / "mvp")], capture_output=True, text=True, cwd=ROOT,
                       timeout=300, env=dict(os.environ, OMP_NUM_THREADS="1"))
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert "'step': 2" in p.stdout


def test_model_report_sweeps_and_sensitivity(tmp_path):
    from nano_train_b200.utils.model_info import (DecodeEPExplorationConfig, decode_ep_exploration, decode_sweep,
                                                  default_roofline_targets, sensitivity_grid)

    model = TransformerModel(llama3_8b_config(param_device=torch.device("meta"), sequence_parallel=False))
    pts = sensitivity_grid(model)
    assert len(pts) == 2 * 3 * 3 * 3 * 4 * 2  # kv dtype x top-k x kv rank x hidden x context x exec model
    # longer contexts never make decode faster; fp8 KV never slower than bf16
    for p in pts:
        if p.cache_len == 2048:
            q = next(o for o in pts if (o.exec_model, o.kv_dtype_bytes, o.top_k, o.kv_rank_scale, o.hidden_scale,
                                        o.cache_len) == (p.exec_model, p.kv_dtype_bytes, p.top_k, p.kv_rank_scale,
                                                         p.hidden_scale, 16384))
            assert q.t_est_ms >= p.t_est_ms
    rows = decode_sweep(model, targets=default_roofline_targets()[:2])
    assert rows[0]["bound"]["B200 fp8"] == "hbm"      # batch 1 decode streams the weights
    bc = rows[0]["b_crit"]["B200 fp8"]
    assert bc is None or bc > 8
    info = dump_model_info(model, str(tmp_path / "full.md"), batch=8, seq_len=4096)
    text = (tmp_path / "full.md").read_text()
    for sec in ("Parameters by category", "Mode estimates", "Decode batch sweep", "Prefill batch sweep",
                "Sensitivity grid (432 points"):
        assert sec in text, sec
    assert {k.exec_model for k in info.kpis} == {"naive", "efficient"}
    naive = next(k for k in info.kpis if k.mode == "prefill" and k.exec_model == "naive")
    eff = next(k for k in info.kpis if k.mode == "prefill" and k.exec_model == "efficient"
               and k.target == naive.target)
    assert naive.bytes_temporary > 0 and eff.bytes_temporary == 0 and eff.bytes_hbm < naive.bytes_hbm
    # routed-expert model: EP exploration rows and partial expert coverage at small decode batches
    from nano_train_b200.config import _NoOpPrecisionResolver
    from nano_train_b200.models.deepseek import DeepSeekModel, DeepSeekModelConfig

    cfg = DeepSeekModelConfig(param_dtype=torch.bfloat16, param_device=torch.device("meta"),
                              precision_resolver=_NoOpPrecisionResolver(), vocab_size=1024, hidden_size=256,
                              num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4,
                              n_routed_experts=16, num_experts_per_tok=2, moe_intermediate_size=128,
                              intermediate_size=512, first_k_dense_replace=1, kv_lora_rank=64, q_lora_rank=96,
                              qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32, n_shared_experts=1,
                              max_position_embeddings=1024)
    ds = DeepSeekModel(cfg)
    ex = decode_ep_exploration(ds, DecodeEPExplorationConfig(ep_sizes=[1, 2, 4], cache_lengths=[1024]))
    assert [r["ep"] for r in ex] == [1, 2, 4]
    e1 = estimate(ds, batch=1, decode_ctx=1024)
    e64 = estimate(ds, batch=64, decode_ctx=1024)
    w1 = next(k for k in e1.kpis if k.mode == "decode").bytes_weights
    w64 = next(k for k in e64.kpis if k.mode == "decode").bytes_weights
    assert w1 < w64  # one token touches top_k of the experts, 64 tokens nearly all of them


def test_view_logs_renders_jsonl_metrics(tmp_path):
    """The offline log viewer turns metrics.jsonl runs into one HTML page of SVG charts, including
    flat series at large magnitude (tick generation is bounded)."""
    import json

    from nano_train_b200.utils.svg_plot import _lin_ticks
    from nano_train_b200.utils.view_logs import main

    for run, off in (("a", 0.0), ("b", 0.1)):
        d = tmp_path / "logs" / run
        d.mkdir(parents=True)
        with open(d / "metrics.jsonl", "w") as f:
            for s in range(5):
                f.write(json.dumps({"tag": "Loss/train", "value": 5.0 - s * 0.3 + off, "step": s}) + "\n")
                f.write(json.dumps({"tag": "Throughput/tokens", "value": 1e9 + s * 1e-7, "step": s}) + "\n")
            f.write('{"tag": "Loss/train", "val')  # a partly written last line is skipped
    out = tmp_path / "m.html"
    assert main(["--logdir", str(tmp_path / "logs"), "--html", str(out)]) == 0
    html = out.read_text()
    assert html.count("<svg") == 2 and "Loss/train" in html and html.count("<polyline") == 4
    for lo, hi in ((1e9, 1e9 + 1e-7), (0.0, 0.0), (-1.0, 1.0), (1e-12, 2e-12)):
        assert 1 <= len(_lin_ticks(lo, hi)) <= 8


def test_gpt_1p3b_config_shape():
    from nano_train_b200.models.transformer import gpt_1p3b_config

    m = TransformerModel(gpt_1p3b_config(param_device=torch.device("meta")))
    n = sum(p.numel() for p in m.parameters())  # tied head: the embedding is counted once
    assert 1.30e9 < n < 1.33e9, n
    assert m.config.hidden_size == 2048 and len(m.blocks) == 24 and m.config.vocab_size == 50304


def test_logged_gradient_norm_is_the_norm_of_the_steps_gradient(tmp_path):
    """The pre-clip gradient norm the Trainer logs is taken from the step's gradients before they are
    cleared: it equals the norm of the same batch's gradient computed independently."""
    import copy

    torch.manual_seed(0)
    mcfg = _tiny_cfg()
    model = TransformerModel(mcfg)
    twin = copy.deepcopy(model)
    cfg = Config(model=mcfg, training=TrainingConfig(batch_size=4, micro_batch_size=4, learning_rate=1e-3,
                                                     max_steps=1, warmup_steps=0, log_steps=1, eval_steps=100,
                                                     save_steps=100, clip_grad=0.05),
                 output_dir=str(tmp_path / "out"), log_dir=str(tmp_path / "logs"))
    ds = SyntheticTokenDataset(16, 16, 64, seed=0)
    loader = create_dataloader(ds, 4, shuffle=False)
    tr = Trainer(model, cfg, loader, "cpu")
    logged = {}
    tr.writer = type("W", (), {"add_scalar": lambda self, tag, v, step: logged.setdefault((tag, step), float(v)),
                               "flush": lambda self: None, "close": lambda self: None})()
    tr.train()
    batch = next(iter(create_dataloader(ds, 4, shuffle=False)))
    logits = twin(batch["input_ids"])
    torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), batch["labels"].reshape(-1),
                                      ignore_index=-100).backward()
    expect = float(torch.sqrt(sum(p.grad.float().pow(2).sum() for p in twin.parameters() if p.grad is not None)))
    got = logged[("Gradients/global_norm_pre_clip", 1)]
    assert got == pytest.approx(expect, rel=1e-4)
    assert got > 0.05 and logged[("Gradients/clip_coef", 1)] == pytest.approx(0.05 / (expect + 1e-6), rel=1e-4)
