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


def _import_reference():
    if not os.path.isdir(os.path.join(REF, "src")):
        return None
    sys.path.insert(0, REF)
    for k in [m for m in sys.modules if m == "src" or m.startswith("src.")]:
        del sys.modules[k]
    import src  # noqa: F401
    from src import layers as L
    from src.config import _default_precision_resolver
    from src.models import deepseek as DS
    from src.runtime.optimizer_runtime import PrecisionAdamW

    return L, DS, PrecisionAdamW, _default_precision_resolver


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
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}), flush=True)
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
