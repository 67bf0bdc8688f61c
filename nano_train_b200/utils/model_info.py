"""Static model analytics: parameters, FLOPs, bytes and a roofline time estimate.

A compact analytic model in the spirit of the reference's report generator
(src/utils/model_info.py: ``RooflineConfig`` 114-132, ``dump_model_info``
5076-): it inspects a ``TransformerModel`` or ``DeepSeekModel`` (works on the
``meta`` device, so full-size configs need no memory) and estimates, per
token and per step,

* FLOPs: 2 * in * out per linear (MoE experts weighted by top_k / E),
  attention 4 * S_ctx * d per head (halved for causal prefill/training),
  training = 3 x forward;
* HBM bytes: weights once per step (active experts only), activations
  read/written per layer, KV cache for decode;
* network bytes for tensor parallelism (sequence-parallel all-gather +
  reduce-scatter per linear pair) and expert parallelism (dispatch +
  combine all-to-all);
* time = max(FLOPs / peak, HBM bytes / bandwidth, network bytes / link)
  and the bound that sets it, for every ``RooflineConfig``.

Roofline targets: the public H200 / B200 spec constants, plus the measured
copy bandwidth and bf16 GEMM rate of this pool when ``MEASURED_PEAKS.json``
is next to the package.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Optional

import torch.nn as nn


@dataclass
class RooflineConfig:
    name: str
    peak_tflops: float
    hbm_gbs: float
    link_gbs: float = 900.0  # per direction per GPU (NVLink 5)


def default_roofline_targets() -> list[RooflineConfig]:
    targets = [RooflineConfig("H200 SXM fp8", 1979.0, 4800.0, 450.0),
               RooflineConfig("B200 fp8", 4500.0, 8000.0, 900.0),
               RooflineConfig("B200 bf16", 2250.0, 7700.0, 900.0)]
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        try:
            m = json.load(open(p))
            targets.append(RooflineConfig("B200 bf16 (measured)", float(m["bf16_tflops"]), float(m["hbm_gbs"]), 770.0))
        except Exception:
            pass
    return targets


@dataclass
class ParallelismAssumptions:
    tp: int = 1
    ep: int = 1
    dp: int = 1
    pp: int = 1


@dataclass
class LayerInfo:
    name: str
    kind: str
    params: int
    in_features: int = 0
    out_features: int = 0
    active_fraction: float = 1.0


@dataclass
class ModeEstimate:
    mode: str
    tokens: int
    flops: float
    hbm_bytes: float
    net_bytes: float
    per_target: dict = field(default_factory=dict)


@dataclass
class ModelInfo:
    architecture: dict
    total_params: int
    active_params_per_token: float
    layers: list
    kv_cache_bytes_per_token: float
    modes: list


def _arch(model: nn.Module) -> dict:
    cfg = getattr(model, "config", None)
    def get(*names, d=None):
        for n in names:
            v = getattr(cfg, n, None) if cfg is not None else None
            if v is not None:
                return v
        return d

    hidden = get("hidden_size", d=0)
    heads = get("num_attention_heads", d=1)
    kv_heads = get("num_key_value_heads", d=None) or heads
    arch = dict(kind=type(model).__name__, hidden=hidden, layers=get("num_layers", "num_hidden_layers", d=0),
                heads=heads, kv_heads=kv_heads, vocab=get("vocab_size", d=0),
                head_dim=get("head_dim", d=None) or (hidden // max(heads, 1)),
                num_experts=get("n_routed_experts", "num_experts", d=0), top_k=get("num_experts_per_tok", "top_k", d=0),
                kv_lora_rank=get("kv_lora_rank", d=0), qk_rope_head_dim=get("qk_rope_head_dim", d=0),
                qk_nope_head_dim=get("qk_nope_head_dim", d=0), v_head_dim=get("v_head_dim", d=0))
    arch["mla"] = bool(arch["kv_lora_rank"])
    return arch


def _collect_layers(model: nn.Module, arch: dict) -> list[LayerInfo]:
    out = []
    E, K = arch["num_experts"], arch["top_k"]
    for name, mod in model.named_modules():
        w = getattr(mod, "weight", None)
        if w is None or not isinstance(w, nn.Parameter) or w.dim() != 2 or any(True for _ in mod.children()):
            continue
        kind = "embedding" if "embed" in name else ("expert" if ".experts." in name else
                                                    ("router" if "router" in name else "linear"))
        frac = (K / E) if kind == "expert" and E else 1.0
        if kind == "embedding":
            out.append(LayerInfo(name, kind, w.numel()))
        else:
            # torch layout [out, in] for the linears of this framework (row-parallel shards included)
            out.append(LayerInfo(name, kind, w.numel(), w.shape[1], w.shape[0], frac))
    return out


def _kv_bytes_per_token(arch: dict, dtype_bytes: int = 2) -> float:
    L = arch["layers"]
    if arch["mla"]:
        return L * (arch["kv_lora_rank"] + arch["qk_rope_head_dim"]) * dtype_bytes
    return L * 2 * arch["kv_heads"] * arch["head_dim"] * dtype_bytes


def _attn_flops_per_token(arch: dict, ctx: int, causal: bool) -> float:
    d_qk = (arch["qk_nope_head_dim"] + arch["qk_rope_head_dim"]) if arch["mla"] else arch["head_dim"]
    d_v = arch["v_head_dim"] if arch["mla"] else arch["head_dim"]
    f = 2 * arch["heads"] * ctx * (d_qk + d_v) * arch["layers"]
    return f * (0.5 if causal else 1.0)


def estimate(model: nn.Module, *, batch: int = 1, seq_len: int = 4096, decode_ctx: int = 4096,
             parallel: Optional[ParallelismAssumptions] = None, targets: Optional[list] = None,
             weight_bytes: float = 2.0) -> ModelInfo:
    parallel = parallel or ParallelismAssumptions()
    targets = targets or default_roofline_targets()
    arch = _arch(model)
    layers = _collect_layers(model, arch)
    total = sum(p.numel() for p in model.parameters())
    lin = [l for l in layers if l.kind != "embedding"]
    active = sum(l.params * l.active_fraction for l in lin)
    flops_linear_tok = sum(2.0 * l.in_features * l.out_features * l.active_fraction for l in lin)
    H, L = arch["hidden"], arch["layers"]
    modes = []
    for mode, tokens, ctx, causal, mult in (("train", batch * seq_len, seq_len, True, 3.0),
                                           ("prefill", batch * seq_len, seq_len, True, 1.0),
                                           ("decode", batch, decode_ctx, False, 1.0)):
        flops = mult * tokens * (flops_linear_tok + _attn_flops_per_token(arch, ctx, causal))
        w_bytes = active * weight_bytes if mode != "train" else active * (weight_bytes + 4 + 4 + 12)  # + grads/master/moments
        act_bytes = tokens * H * 2 * L * (8 if mode == "train" else 4)
        kv = _kv_bytes_per_token(arch) * (decode_ctx * batch if mode == "decode" else tokens)
        hbm = w_bytes + act_bytes + kv
        net = 0.0
        if parallel.tp > 1:  # AG + RS of [tokens, H] twice per layer (fwd), doubled for backward
            net += (2 if mode == "train" else 1) * 4 * tokens * H * 2 * L * (parallel.tp - 1) / parallel.tp
        if parallel.ep > 1 and arch["num_experts"]:
            net += (2 if mode == "train" else 1) * 2 * tokens * arch["top_k"] * H * 2 * L * (parallel.ep - 1) / parallel.ep
        gpus = parallel.tp * parallel.ep * parallel.dp * parallel.pp
        per = {}
        for t in targets:
            tc = flops / gpus / (t.peak_tflops * 1e12)
            th = hbm / max(parallel.tp * parallel.ep * parallel.pp, 1) / (t.hbm_gbs * 1e9)
            tn = net / max(gpus, 1) / (t.link_gbs * 1e9) if net else 0.0
            T = max(tc, th, tn)
            bound = "compute" if T == tc else ("hbm" if T == th else "network")
            per[t.name] = dict(time_ms=T * 1e3, bound=bound, tokens_per_s=tokens / T if T > 0 else 0.0,
                               tokens_per_s_per_gpu=tokens / T / gpus if T > 0 else 0.0,
                               arithmetic_intensity=flops / hbm if hbm else 0.0)
        modes.append(ModeEstimate(mode, tokens, flops, hbm, net, per))
    return ModelInfo(arch, total, active, layers, _kv_bytes_per_token(arch), modes)


def _fmt(x: float, unit: str = "") -> str:
    for s, k in (("P", 1e15), ("T", 1e12), ("G", 1e9), ("M", 1e6), ("K", 1e3)):
        if abs(x) >= k:
            return f"{x / k:.2f} {s}{unit}"
    return f"{x:.2f} {unit}"


def render_markdown(info: ModelInfo) -> str:
    a = info.architecture
    lines = ["# Model report", "", "## Architecture", "", "| field | value |", "|---|---|"]
    lines += [f"| {k} | {v} |" for k, v in a.items()]
    lines += ["", f"Total parameters: {_fmt(info.total_params)}; active per token (MoE weighted): "
              f"{_fmt(info.active_params_per_token)}; KV cache: {_fmt(info.kv_cache_bytes_per_token, 'B')}/token", "",
              "## Largest modules", "", "| module | kind | params | active |", "|---|---|---|---|"]
    for l in sorted(info.layers, key=lambda l: -l.params)[:15]:
        lines.append(f"| {l.name} | {l.kind} | {_fmt(l.params)} | {l.active_fraction:.3f} |")
    lines += ["", "## Roofline estimates", ""]
    for m in info.modes:
        lines += [f"### {m.mode} ({m.tokens} tokens)", "",
                  f"FLOPs {_fmt(m.flops, 'FLOP')}, HBM {_fmt(m.hbm_bytes, 'B')}, network {_fmt(m.net_bytes, 'B')}", "",
                  "| target | time | bound | tokens/s | tokens/s/GPU | FLOP/byte |", "|---|---|---|---|---|---|"]
        for name, r in m.per_target.items():
            lines.append(f"| {name} | {r['time_ms']:.3f} ms | {r['bound']} | {r['tokens_per_s']:.1f} | "
                         f"{r['tokens_per_s_per_gpu']:.1f} | {r['arithmetic_intensity']:.1f} |")
        lines.append("")
    return "\n".join(lines)


def dump_model_info(model: nn.Module, output_path: str, **kw) -> ModelInfo:
    """Write the Markdown report (and a JSON twin) for ``model``; returns the estimate."""
    info = estimate(model, **kw)
    os.makedirs(os.path.dirname(os.path.abspath(output_path)), exist_ok=True)
    with open(output_path, "w") as f:
        f.write(render_markdown(info))
    with open(os.path.splitext(output_path)[0] + ".json", "w") as f:
        json.dump({"architecture": info.architecture, "total_params": info.total_params,
                   "active_params_per_token": info.active_params_per_token,
                   "kv_cache_bytes_per_token": info.kv_cache_bytes_per_token,
                   "layers": [asdict(l) for l in info.layers], "modes": [asdict(m) for m in info.modes]}, f, indent=1)
    return info


def decode_sweep(model: nn.Module, batch_sizes=(1, 8, 32, 128, 512), ctx: int = 4096, **kw) -> list[dict]:
    """Decode throughput estimate across batch sizes (where HBM turns into compute bound)."""
    rows = []
    for b in batch_sizes:
        info = estimate(model, batch=b, decode_ctx=ctx, **kw)
        d = next(m for m in info.modes if m.mode == "decode")
        rows.append({"batch": b, **{k: v["tokens_per_s"] for k, v in d.per_target.items()},
                     "bound": {k: v["bound"] for k, v in d.per_target.items()}})
    return rows


__all__ = ["RooflineConfig", "default_roofline_targets", "ParallelismAssumptions", "ModelInfo", "estimate",
           "dump_model_info", "render_markdown", "decode_sweep"]
