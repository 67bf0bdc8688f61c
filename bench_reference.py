"""Reference arm of bench.py: the unmodified reference (installed into
``baseline/_ref`` as its ``src`` package) on the same Llama-3-8B-shape config.

The reference's ``TransformerModel`` is GPT-2 only (LayerNorm, learned
positions, MHA, GELU, no vocab-parallel loss), so the Llama block is
composed here from the reference's own public primitives, each on its stock
code path: ``src.layers.Embedding`` / ``ColumnParallelLinear`` /
``RowParallelLinear`` (all-reduce tensor parallelism, no sequence
parallelism), ``src.models.deepseek.RMSNorm``, ``GatedMLP`` and its RoPE
helpers, materialised causal softmax attention as the reference computes it
(fp32 softmax over [B, h, S, S] scores), GQA by repeating k/v heads, full
logits gathered across TP for the loss, and ``src.runtime.optimizer_runtime
.PrecisionAdamW`` (fp32 main params and moments). None of this framework's
kernels, models or engine are imported on this path.
"""
from __future__ import annotations

import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(ROOT, "baseline", "_ref")
WHEELHOUSE = "/opt/wheelhouse"
_UNAVAILABLE_WHY = ""


def _reference_sources():
    """Source trees the reference can be installed from, in the order they are tried:
    ``$NTB_REFERENCE_PATH``, then ``reference_path`` of ``BASELINE.json`` next to this file."""
    out = []
    env = os.environ.get("NTB_REFERENCE_PATH")
    if env:
        out.append(env)
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            p = json.load(f).get("reference_path")
        if p:
            out.append(p)
    except (OSError, ValueError):
        pass
    return out


def _install_reference(tried):
    """``pip install --no-deps`` of the unmodified reference into ``baseline/_ref`` (offline, from the
    image's wheelhouse; the image's torch is used, which is why dependency resolution is skipped). The
    source tree may be read-only, so the build runs from a copy in a temporary directory. One process
    per host installs; the others wait on the same file lock and then find the installed copy."""
    import fcntl
    import shutil
    import subprocess
    import tempfile

    os.makedirs(os.path.dirname(REF), exist_ok=True)
    with open(os.path.join(os.path.dirname(REF), ".install.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if os.path.isdir(os.path.join(REF, "src")):
            return True
        for srcdir in _reference_sources():
            if not os.path.isfile(os.path.join(srcdir, "setup.py")):
                tried.append(f"{srcdir}: no setup.py")
                continue
            with tempfile.TemporaryDirectory(prefix="ntb_ref_") as tmp:
                copy = os.path.join(tmp, "reference")
                shutil.copytree(srcdir, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
                cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                       "--find-links", WHEELHOUSE, "--target", REF, copy]
                r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode == 0 and os.path.isdir(os.path.join(REF, "src")):
                return True
            err = (r.stderr or r.stdout).strip().splitlines()
            tried.append(f"pip install {srcdir}: rc={r.returncode} {err[-1] if err else ''}")
    return False


def _import_reference():
    """Import the reference's ``src`` package from ``baseline/_ref`` (or ``$NTB_REFERENCE_SRC``, a
    directory holding an installed ``src``), installing it first when it is absent. Returns None
    and records every path tried and the pip error when no copy can be had."""
    global _UNAVAILABLE_WHY
    tried = []
    roots = [r for r in (os.environ.get("NTB_REFERENCE_SRC"), REF) if r]
    root = next((r for r in roots if os.path.isdir(os.path.join(r, "src"))), None)
    if root is None:
        tried += [f"{r}/src: absent" for r in roots]
        if _install_reference(tried):
            root = REF
    if root is None:
        _UNAVAILABLE_WHY = "reference not installed; tried " + "; ".join(tried)
        return None
    sys.path.insert(0, root)
    for k in [m for m in sys.modules if m == "src" or m.startswith("src.")]:
        del sys.modules[k]
    import src  # noqa: F401
    from src import layers as L
    from src.config import _default_precision_resolver
    from src.models import deepseek as DS
    from src.runtime.optimizer_runtime import PrecisionAdamW

    return L, DS, PrecisionAdamW, _default_precision_resolver


def _print_unavailable(rank, config=None):
    if rank == 0:
        line = {"impl": "reference", "unavailable": _UNAVAILABLE_WHY or "reference not installed"}
        if config:
            line["config"] = config
        print(json.dumps(line), flush=True)


def build_model(ref, layers, rank, world, group, seq):
    L, DS, _, resolver_fn = ref
    H, NQ, NKV, D, I, V = 4096, 32, 8, 128, 14336, 128256
    dt, dev = torch.bfloat16, torch.device("cuda")
    res = resolver_fn()
    kw = dict(param_dtype=dt, param_device=dev, precision_resolver=res)
    tp = world
    pc = DS.DeepSeekParallelContext(tensor_model_parallel_rank=rank, tensor_model_parallel_size=tp,
                                    tensor_model_parallel_group=group)

    def col(i, o, path):
        if tp > 1:
            return L.ColumnParallelLinear(i, o, tp_rank=rank, tp_size=tp, tp_group=group, bias=False,
                                          module_path=path, **kw)
        return L.Linear(i, o, bias=False, module_path=path, **kw)

    def row(i, o, path):
        if tp > 1:
            return L.RowParallelLinear(i, o, tp_rank=rank, tp_size=tp, tp_group=group, bias=False,
                                       module_path=path, **kw)
        return L.Linear(i, o, bias=False, module_path=path, **kw)

    class Block(nn.Module):
        def __init__(self, i):
            super().__init__()
            p = f"layers.{i}"
            self.norm1 = DS.RMSNorm(H, eps=1e-5, module_path=f"{p}.norm1", **kw)
            self.q = col(H, NQ * D, f"{p}.q")
            self.k = col(H, NKV * D, f"{p}.k")
            self.v = col(H, NKV * D, f"{p}.v")
            self.o = row(NQ * D, H, f"{p}.o")
            self.norm2 = DS.RMSNorm(H, eps=1e-5, module_path=f"{p}.norm2", **kw)
            self.mlp = DS.GatedMLP(H, I, 0.0, dt, dev, res, f"{p}.mlp", parallel_context=pc)
            self.nq, self.nkv = NQ // tp, NKV // tp

        def forward(self, x, cos, sin, mask):
            B, S, _ = x.shape
            h = self.norm1(x)
            q = self.q(h).view(B, S, self.nq, D).transpose(1, 2)
            k = self.k(h).view(B, S, self.nkv, D).transpose(1, 2)
            v = self.v(h).view(B, S, self.nkv, D).transpose(1, 2)
            q = DS._apply_rope(q, cos, sin)
            k = DS._apply_rope(k, cos, sin)
            rep = self.nq // self.nkv
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
            scores = torch.matmul(q, k.transpose(-1, -2)) * (1.0 / math.sqrt(D)) + mask
            probs = torch.softmax(scores.float(), dim=-1).to(v.dtype)
            a = torch.matmul(probs, v).transpose(1, 2).reshape(B, S, self.nq * D)
            x = x + self.o(a)
            return x + self.mlp(self.norm2(x))

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.emb = L.Embedding(V, H, module_path="emb", **kw)
            self.blocks = nn.ModuleList([Block(i) for i in range(layers)])
            self.norm = DS.RMSNorm(H, eps=1e-5, module_path="norm", **kw)
            self.head = col(H, V, "lm_head")

        def forward(self, ids, labels):
            B, S = ids.shape
            cos, sin = DS._build_rope_cache(S, D, ids.device, 500000.0)
            cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
            mask = torch.full((S, S), float("-inf"), device=ids.device, dtype=torch.bfloat16).triu(1)
            x = self.emb(ids)
            for b in self.blocks:
                x = b(x, cos, sin, mask)
            logits = self.head(self.norm(x))
            if tp > 1:
                import torch.distributed.nn.functional as dnn

                logits = torch.cat(dnn.all_gather(logits.contiguous(), group=group), dim=-1)
            return F.cross_entropy(logits.float().view(-1, V), labels.reshape(-1))

    return Model()


def run(args, rank, local, world, global_batch, micro_batch, make_batches, barrier, max_over_ranks, ClockSampler):
    ref = _import_reference()
    if ref is None:
        _print_unavailable(rank)
        return None
    _, _, PrecisionAdamW, _ = ref
    layers = args.layers or (8 if world == 1 else 32)
    group = dist.group.WORLD if world > 1 else None
    torch.manual_seed(1234 + rank)
    model = build_model(ref, layers, rank, world, group, args.seq)
    opt = PrecisionAdamW(model.parameters(), lr=3e-4, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8,
                         main_params_dtype="fp32", main_grads_dtype="fp32", exp_avg_dtype="fp32",
                         exp_avg_sq_dtype="fp32")
    n_mb = global_batch // micro_batch

    def step(ids_h, lab_h):
        ids = ids_h.to("cuda", non_blocking=True)
        lab = lab_h.to("cuda", non_blocking=True)
        opt.zero_grad()
        tot = torch.zeros((), device="cuda")
        for i in range(n_mb):
            loss = model(ids[i * micro_batch:(i + 1) * micro_batch], lab[i * micro_batch:(i + 1) * micro_batch])
            (loss / n_mb).backward()
            tot += loss.detach()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        return tot / n_mb

    batches = make_batches(4, args.seq, 128256)
    for i in range(args.warmup):
        step(*batches[i % len(batches)])
    barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier(world)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(*batches[i % len(batches)])
    e.record()
    barrier(world)
    sampler.stop()
    ms = max_over_ranks(s.elapsed_time(e) / args.steps, world)
    e2e = None
    if not args.no_e2e:
        barrier(world)
        t0 = time.perf_counter()
        for i in range(args.steps):
            float(step(*batches[i % len(batches)]))
        barrier(world)
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps, world)
        e2e = {"value": global_batch * args.seq / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": 2 * global_batch * args.seq * 8, "d2h_bytes_per_step": 4,
               "api": "reference primitives (src.layers / src.models.deepseek) + PrecisionAdamW"}
    return ms, layers, 0, sampler.summary(), e2e


def run_deepseek(args, rank, local, world, make_batches, barrier, max_over_ranks, ClockSampler, batch, dims=None):
    """The DeepSeek-V2-Lite-shape fp8 configuration through the reference's own public API:
    ``src.models.deepseek.DeepSeekModel`` built from its config under the reference's
    ``resolve_precision_config`` with the deepseek_v3 recipe on its stock (emulated) fp8 backend,
    its router aux losses, ``PrecisionAdamW`` with fp32 main weights and moments. With N ranks it runs
    EP = N and DP = 1 (the reference cannot fold EP into DP): every rank trains on the same batch, so the
    tokens of a step are one batch. ``dims`` shrinks the model for a CPU check of this code."""
    ref = _import_reference()
    if ref is None:
        _print_unavailable(rank)
        return None
    import argparse as _ap

    from src.models.deepseek import DeepSeekModel, DeepSeekModelConfig, DeepSeekParallelContext
    from src.models.moe import ExpertParallelMoE, LocalRoutedMoE
    from src.runtime.mixed_precision import build_module_precision_resolver, resolve_precision_config
    from src.runtime.optimizer_runtime import PrecisionAdamW

    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    pargs = _ap.Namespace(precision_recipe="deepseek_v3", bf16=False, fp16=False, fp8=True, fp4=False,
                          fp8_backend="emulated", params_dtype="bf16" if dev.type == "cuda" else "fp32")
    pc = resolve_precision_config(pargs, dev)
    res = build_module_precision_resolver(pc)
    d = dict(vocab_size=102400, hidden_size=2048, num_hidden_layers=args.layers or 8, num_attention_heads=16,
             num_key_value_heads=16, intermediate_size=10944, max_position_embeddings=4096, q_lora_rank=1536,
             kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
             moe_intermediate_size=1408, n_routed_experts=64, n_shared_experts=2, num_experts_per_tok=6,
             first_k_dense_replace=1, scoring_func="softmax", n_group=1, topk_group=1, norm_topk_prob=False,
             routed_scaling_factor=1.0)
    d.update(dims or {})
    pctx = None
    if world > 1:
        # The reference cannot fold EP into DP: EP = N forces DP = 1, so every rank runs the same batch
        # (the caller counts its tokens once) and dense gradients need no reduction.
        from src.distributed.topology import initialize_model_parallel

        par = initialize_model_parallel(tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                                        expert_model_parallel_size=world)
        pctx = DeepSeekParallelContext(expert_model_parallel_rank=par.expert_model_parallel_rank,
                                       expert_model_parallel_size=world,
                                       expert_model_parallel_group=par.expert_model_parallel_group)
    torch.manual_seed(1234)  # the same on every rank: identical dense weights
    dt = torch.bfloat16 if dev.type == "cuda" else torch.float32
    model = DeepSeekModel(DeepSeekModelConfig(param_dtype=dt, param_device=dev, precision_resolver=res, **d),
                          parallel_context=pctx)
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() >= 2:
                p.normal_(0.0, 0.006)
    moes = [m for m in model.modules() if isinstance(m, (LocalRoutedMoE, ExpertParallelMoE))]
    opt = PrecisionAdamW(model.parameters(), lr=3e-4, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8,
                         main_params_dtype="fp32", main_grads_dtype="fp32", exp_avg_dtype="fp32",
                         exp_avg_sq_dtype="fp32")

    def step(ids_h, lab_h):
        ids, lab = ids_h.to(dev, non_blocking=True), lab_h.to(dev, non_blocking=True)
        opt.zero_grad()
        logits = model(ids)
        loss = F.cross_entropy(logits.float().view(-1, logits.size(-1)), lab.reshape(-1))
        aux = torch.stack([m.last_aux_loss.float().reshape(()) for m in moes]).sum()
        (loss + 0.01 * aux).backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        return loss.detach()

    batches = make_batches(2, args.seq, d["vocab_size"], batch=batch)  # same seed on every rank: one batch
    for i in range(args.warmup):
        step(*batches[i % len(batches)])
    if dev.type != "cuda":
        return float(step(*batches[0]))
    barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(*batches[i % len(batches)])
    e.record()
    barrier(world)
    sampler.stop()
    ms = max_over_ranks(s.elapsed_time(e) / args.steps, world)
    e2e = None
    if not args.no_e2e:
        barrier(world)
        t0 = time.perf_counter()
        for i in range(args.steps):
            float(step(*batches[i % len(batches)]))
        barrier(world)
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps, world)
        e2e = {"value": batch * args.seq / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": 2 * batch * args.seq * 8, "d2h_bytes_per_step": 4,
               "api": "src.models.deepseek.DeepSeekModel + PrecisionAdamW (deepseek_v3 recipe, emulated fp8)"}
    return ms, d["num_hidden_layers"], 0, sampler.summary(), e2e


def run_gpt_fp4(args, rank, local, world, make_batches, barrier, ClockSampler, batch, dims=None):
    """The GPT-1.3B-shape fp4 configuration through the reference's own ``TransformerModel`` (GPT-2
    block, materialised attention, tied head) under its ``resolve_precision_config`` with ``--fp4`` on
    its stock (emulated, integer-grid) fp4 backend, ``PrecisionAdamW`` with fp32 main weights and
    moments. One GPU: the reference wires ZeRO only for its DeepSeekModel."""
    ref = _import_reference()
    if ref is None:
        _print_unavailable(rank)
        return None
    if world > 1:
        if rank == 0:
            print(json.dumps({"impl": "reference", "config": args.config, "unavailable":
                              "the reference wires ZeRO-1 only for DeepSeekModel; measured at N = 1"}), flush=True)
        return None
    import argparse as _ap

    from src.config import ModelConfig
    from src.models.transformer import TransformerModel
    from src.runtime.mixed_precision import build_module_precision_resolver, resolve_precision_config
    from src.runtime.optimizer_runtime import PrecisionAdamW

    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    pargs = _ap.Namespace(precision_recipe="default", bf16=False, fp16=False, fp8=False, fp4=True,
                          fp4_backend="emulated", params_dtype="bf16" if dev.type == "cuda" else "fp32")
    res = build_module_precision_resolver(resolve_precision_config(pargs, dev))
    d = dict(hidden_size=2048, num_layers=args.layers or 24, num_attention_heads=16, intermediate_size=8192,
             max_position_embeddings=2048, vocab_size=50304, dropout=0.0)
    d.update(dims or {})
    torch.manual_seed(1234)
    dt = torch.bfloat16 if dev.type == "cuda" else torch.float32
    model = TransformerModel(ModelConfig(param_dtype=dt, param_device=dev, precision_resolver=res, **d))
    opt = PrecisionAdamW(model.parameters(), lr=3e-4, weight_decay=0.1, betas=(0.9, 0.95), eps=1e-8,
                         main_params_dtype="fp32", main_grads_dtype="fp32", exp_avg_dtype="fp32",
                         exp_avg_sq_dtype="fp32")

    def step(ids_h, lab_h):
        ids, lab = ids_h.to(dev, non_blocking=True), lab_h.to(dev, non_blocking=True)
        opt.zero_grad()
        logits = model(ids)
        loss = F.cross_entropy(logits.float().view(-1, logits.size(-1)), lab.reshape(-1))
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        return loss.detach()

    batches = make_batches(2, args.seq, d["vocab_size"], batch=batch)
    for i in range(args.warmup):
        step(*batches[i % len(batches)])
    if dev.type != "cuda":
        return float(step(*batches[0]))
    barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(*batches[i % len(batches)])
    e.record()
    barrier(world)
    sampler.stop()
    ms = s.elapsed_time(e) / args.steps
    e2e = None
    if not args.no_e2e:
        t0 = time.perf_counter()
        for i in range(args.steps):
            float(step(*batches[i % len(batches)]))
        torch.cuda.synchronize()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        e2e = {"value": batch * args.seq / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": 2 * batch * args.seq * 8, "d2h_bytes_per_step": 4,
               "api": "src.models.transformer.TransformerModel + PrecisionAdamW (--fp4, emulated backend)"}
    return ms, d["num_layers"], 0, sampler.summary(), e2e
