"""Static model analytics: parameters, FLOPs, bytes, network traffic and roofline estimates.

The capabilities of the reference's report generator (src/utils/model_info.py:
``RooflineConfig`` 113-132, execution models 135-162 and 284-305, tensor-core
model 165-191, sweeps 308-389, sensitivity 220-246, ``dump_model_info``),
built on an analytic model of this file's own:

* The model is inspected module by module (``meta`` device works, so
  full-size configs need no memory); every 2-D weight is classified as
  embedding / attention projection / dense FFN / shared expert / routed
  expert / router / lm_head.
* FLOPs per token: 2 * in * out per linear (a routed expert weighted by
  top_k / E), attention 2 * heads * ctx * (d_qk + d_v) per layer (halved for
  causal prefill / training); training = 3 x forward.
* Realizable FLOPs (what the tensor cores actually spend): per class, the
  tensor-core eligible part costs theory / eta(M) with eta(M) = min(1, M / b_sat)
  for an M-row GEMM (a routed expert sees M = tokens * K / E rows), the rest
  costs theory / eta_scalar.
* HBM bytes, split into weights (each touched weight read once per step,
  divided by the execution model's reuse factor; a decode batch of B tokens
  touches the expected fraction 1 - (1 - K/E)^B of the routed experts),
  activations, KV cache and temporaries (the S x ctx score matrix of
  non-fused attention), plus optimizer traffic for training.
* Network bytes per GPU: sequence-parallel all-gather + reduce-scatter per
  linear pair (TP), dispatch + combine (EP, bf16 or fp8 payload), gradient
  reduce-scatter + parameter all-gather (DP, training).
* Per GPU: t_comp = realizable / peak, t_hbm = bytes / bandwidth (dense weights
  split over TP x PP, experts over EP x TP x PP, the rest over all GPUs),
  t_net = bytes / link; t_est = max; the regime names the bound.

Sweeps: decode over batch (with the critical batch where decode turns compute
bound), prefill over batch, decode expert-parallel exploration (smallest
per-GPU batch that is within ``alpha`` of compute bound, per EP size and
context), and a sensitivity grid over KV dtype, top-k, KV rank, hidden size,
context and execution model (2 x 3 x 3 x 3 x 4 x 2 = 432 points by default).
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Optional

import torch.nn as nn


# ----------------------------------------------------------------------------- hardware and execution models
@dataclass
class RooflineConfig:
    name: str
    peak_tflops: float
    hbm_gbs: float
    link_gbs: float = 900.0  # per direction per GPU (NVLink 5)

    @property
    def mem_bw_gbps(self) -> float:  # the reference's field name
        return self.hbm_gbs

    @property
    def knee(self) -> float:
        """Arithmetic intensity (FLOP/byte) where HBM and compute time meet."""
        return self.peak_tflops * 1e12 / (self.hbm_gbs * 1e9)


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
class ExecutionModel:
    """How well an implementation reuses data (knobs of the byte model, not measured claims)."""
    name: str
    attention: str = "naive"           # "naive": S x ctx scores go through HBM; "flash": they do not
    weight_reuse: float = 1.0          # weight bytes are divided by this (tiles reused across M)
    expert_weight_reuse: float = 1.0
    activation_factor: float = 1.0     # activation bytes multiplier (fusion < 1)
    elementwise_factor: float = 1.0    # norm / activation / residual passes multiplier

    def validate(self) -> None:
        if self.attention not in ("naive", "flash"):
            raise ValueError("attention must be 'naive' or 'flash'")
        for k in ("weight_reuse", "expert_weight_reuse", "activation_factor", "elementwise_factor"):
            if getattr(self, k) <= 0:
                raise ValueError(f"{k} must be > 0")


def default_execution_models() -> list[ExecutionModel]:
    return [ExecutionModel("naive"),
            ExecutionModel("efficient", attention="flash", weight_reuse=4.0, expert_weight_reuse=2.0,
                           activation_factor=0.5, elementwise_factor=0.7)]


@dataclass
class TensorCoreModel:
    enabled: bool = True
    b_sat: int = 64            # GEMM rows at which the tensor cores are fully fed
    eta_scalar: float = 0.35   # efficiency of the non tensor-core remainder
    eligible: dict = field(default_factory=lambda: {"attention": 0.95, "linear": 0.98, "embedding": 0.70})

    def validate(self) -> None:
        if self.b_sat <= 0 or not (0.0 < self.eta_scalar <= 1.0):
            raise ValueError("b_sat must be > 0 and eta_scalar in (0, 1]")
        for k, v in self.eligible.items():
            if not (0.0 <= v <= 1.0):
                raise ValueError(f"eligible[{k}] must be in [0, 1]")

    def eta(self, rows: float) -> float:
        """Tensor-core saturation at GEMM height ``rows`` (tokens per GEMM, or per active expert)."""
        return 1.0 if not self.enabled else min(1.0, max(rows, 1e-9) / self.b_sat)

    def realizable(self, flops: float, rows: float, kind: str) -> float:
        """Peak-equivalent FLOPs: eligible work at the tensor cores' saturation, the rest at eta_scalar
        (so realizable / peak is the modelled compute time)."""
        return self.breakdown(flops, rows, kind).realizable

    def breakdown(self, flops: float, rows: float, kind: str) -> "FlopBreakdown":
        if not self.enabled or flops == 0:
            return FlopBreakdown(flops, flops, flops, 1.0)
        e = self.eligible.get(kind, 0.0)
        eta = self.eta(rows)
        return FlopBreakdown(theory=flops, tensorcore=flops * e,
                             realizable=flops * (e / eta + (1.0 - e) / self.eta_scalar), eta_tc=eta)


@dataclass
class FlopBreakdown:
    """Theory FLOPs, the tensor-core-eligible part, the peak-equivalent (realizable) cost and the
    tensor-core saturation of one piece of work; breakdowns add up across layers."""
    theory: float
    tensorcore: float
    realizable: float
    eta_tc: float = 1.0

    def __add__(self, o: "FlopBreakdown") -> "FlopBreakdown":
        tc = self.tensorcore + o.tensorcore
        eta = (self.tensorcore * self.eta_tc + o.tensorcore * o.eta_tc) / tc if tc else 1.0  # eligible-FLOP weighted
        return FlopBreakdown(self.theory + o.theory, tc, self.realizable + o.realizable, eta)

    def p_effective_tflops(self, peak_tflops: float) -> float:
        """Throughput the modelled execution sustains on this work: peak x theory / realizable."""
        return peak_tflops * self.theory / self.realizable if self.realizable else peak_tflops


@dataclass
class ParallelismAssumptions:
    tp: int = 1
    ep: int = 1
    dp: int = 1
    pp: int = 1
    ep_payload_bytes: float = 2.0   # 1.0 for an e4m3 dispatch / combine payload

    @property
    def gpus(self) -> int:
        return self.tp * self.ep * self.dp * self.pp


# ----------------------------------------------------------------------------- model inspection
@dataclass
class LayerInfo:
    name: str
    kind: str          # embedding | attention | mlp | shared_expert | expert | router | lm_head
    params: int
    in_features: int = 0
    out_features: int = 0
    active_fraction: float = 1.0


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


def _classify(name: str) -> str:
    n = name.lower()
    if "embed" in n or n.endswith("wte") or n.endswith("wpe"):
        return "embedding"
    if "lm_head" in n or n.endswith("output"):
        return "lm_head"
    if "shared_expert" in n:
        return "shared_expert"
    if ".experts." in n:
        return "expert"
    if "router" in n:
        return "router"
    if any(k in n for k in ("attn", "attention", "q_proj", "k_proj", "v_proj", "o_proj", "qkv", "kv_a", "kv_b",
                            "q_a", "q_b", "out_proj")):
        return "attention"
    return "mlp"


def _collect_layers(model: nn.Module, arch: dict) -> list[LayerInfo]:
    out = []
    E, K = arch["num_experts"], arch["top_k"]
    for name, mod in model.named_modules():
        w = getattr(mod, "weight", None)
        if w is None or not isinstance(w, nn.Parameter) or w.dim() != 2 or any(True for _ in mod.children()):
            continue
        kind = _classify(name)
        frac = (K / E) if kind == "expert" and E else 1.0
        if kind == "embedding":
            out.append(LayerInfo(name, kind, w.numel()))
        else:
            # torch layout [out, in] for this framework's linears (tensor-parallel shards included)
            out.append(LayerInfo(name, kind, w.numel(), w.shape[1], w.shape[0], frac))
    return out


def _kv_bytes_per_token(arch: dict, dtype_bytes: float = 2.0, rank_scale: float = 1.0) -> float:
    L = arch["layers"]
    if arch["mla"]:
        return L * (arch["kv_lora_rank"] * rank_scale + arch["qk_rope_head_dim"]) * dtype_bytes
    return L * 2 * arch["kv_heads"] * rank_scale * arch["head_dim"] * dtype_bytes


def _attn_flops_per_token(arch: dict, ctx: int, causal: bool, hidden_scale: float = 1.0) -> float:
    d_qk = (arch["qk_nope_head_dim"] + arch["qk_rope_head_dim"]) if arch["mla"] else arch["head_dim"]
    d_v = arch["v_head_dim"] if arch["mla"] else arch["head_dim"]
    f = 2 * arch["heads"] * hidden_scale * ctx * (d_qk + d_v) * arch["layers"]
    return f * (0.5 if causal else 1.0)


# ----------------------------------------------------------------------------- the estimate
@dataclass
class ModeKpi:
    """One (mode, execution model, roofline target) operating point, per GPU unless named otherwise."""
    mode: str
    exec_model: str
    target: str
    tokens: int
    flops_theory: float
    flops_realizable: float
    flops_tensorcore: float
    eta_tc: float
    p_effective_tflops: float
    bytes_weights: float
    bytes_activations: float
    bytes_kv: float
    bytes_temporary: float
    bytes_hbm: float
    bytes_net: float
    ai_hbm: float
    ai_total: float
    t_comp_ms: float
    t_hbm_ms: float
    t_net_ms: float
    t_est_ms: float
    regime: str
    mfu_est: float
    tokens_per_s: float
    tokens_per_s_per_gpu: float


@dataclass
class ModeEstimate:
    """Whole-job totals of one mode plus, per roofline target, the efficient-execution estimate."""
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
    params_by_kind: dict
    layers: list
    kv_cache_bytes_per_token: float
    modes: list
    kpis: list


@dataclass
class _Variant:
    """Knobs of the sensitivity grid applied on top of the inspected model."""
    hidden_scale: float = 1.0
    top_k: Optional[int] = None
    kv_rank_scale: float = 1.0
    kv_dtype_bytes: float = 2.0


def _mode_kpi(arch, layers, mode, batch, seq_len, ctx, par: ParallelismAssumptions, xm: ExecutionModel,
              tc: TensorCoreModel, target: RooflineConfig, weight_bytes: float, var: _Variant) -> ModeKpi:
    E = arch["num_experts"]
    K = var.top_k or arch["top_k"]
    hs = var.hidden_scale
    H, L = arch["hidden"] * hs, arch["layers"]
    train = mode == "train"
    tokens = batch if mode == "decode" else batch * seq_len
    causal = mode != "decode"
    mult = 3.0 if train else 1.0
    gpus = par.gpus
    # FLOPs, theory and realizable (per class, rows per GEMM per GPU)
    rows_dense = tokens / max(par.dp * par.ep, 1)
    fb = FlopBreakdown(0.0, 0.0, 0.0)
    w_dense = w_exp = 0.0
    for l in layers:
        if l.kind == "embedding":
            w_dense += l.params * hs
            continue
        frac = (K / E) if (l.kind == "expert" and E) else l.active_fraction
        f = mult * tokens * 2.0 * l.in_features * l.out_features * frac * hs * hs
        rows = rows_dense * (K / E if (l.kind == "expert" and E) else 1.0) * (par.ep if l.kind == "expert" else 1)
        fb = fb + tc.breakdown(f, rows, "linear")
        if l.kind == "expert":
            cover = 1.0 if mode != "decode" else 1.0 - (1.0 - (K / E if E else 1.0)) ** max(tokens, 1)
            w_exp += l.params * hs * hs * cover
        else:
            w_dense += l.params * hs * hs
    fa = mult * tokens * _attn_flops_per_token(arch, ctx, causal, hs)
    fb = fb + tc.breakdown(fa, rows_dense, "attention")
    f_th, f_re = fb.theory, fb.realizable
    # HBM bytes (whole job)
    wb = weight_bytes
    if train:  # forward + backward weight reads, fp32 gradient accumulate (8 B), optimizer pass (28 B)
        wb_dense = w_dense * (2 * wb / xm.weight_reuse + 36.0)
        wb_exp = w_exp * (2 * wb / xm.expert_weight_reuse + 36.0)
    else:
        wb_dense = w_dense * wb / xm.weight_reuse
        wb_exp = w_exp * wb / xm.expert_weight_reuse
    w_bytes = wb_dense + wb_exp
    I_sum = sum(l.out_features for l in layers if l.kind in ("mlp", "shared_expert")) * hs / max(L, 1)
    act_per_tok_layer = (12.0 * H + 3.0 * I_sum) * 2.0
    if E:
        act_per_tok_layer += 3.0 * K * H * 2.0
    act = tokens * L * act_per_tok_layer * xm.activation_factor * (3.0 if train else 1.0)
    act += tokens * L * 6.0 * H * 2.0 * xm.elementwise_factor * (2.0 if train else 1.0)
    kvpt = _kv_bytes_per_token(arch, var.kv_dtype_bytes, var.kv_rank_scale)
    if mode == "decode":
        kv = batch * ctx * kvpt
    elif mode == "prefill":
        kv = tokens * kvpt
    else:
        kv = 0.0
    temp = 0.0
    if xm.attention == "naive":
        heads = arch["heads"] * hs
        q = tokens
        temp = q * ctx * heads * L * 4.0 * 2.0 * (0.5 if causal else 1.0) * (3.0 if train else 1.0)
    # network bytes per GPU
    net = 0.0
    tok_gpu = tokens / max(gpus, 1) * par.tp  # tokens a TP group works on, per TP rank
    if par.tp > 1:
        net += (2.0 if train else 1.0) * 4.0 * tok_gpu * H * 2.0 * L * (par.tp - 1) / par.tp
    if par.ep > 1 and E:
        net += (2.0 if train else 1.0) * 2.0 * (tokens / gpus) * K * H * par.ep_payload_bytes * L * (par.ep - 1) / par.ep
    if train and par.dp > 1:
        params_gpu = (w_dense / (par.tp * par.pp)) + (w_exp / (par.ep * par.tp * par.pp))
        net += params_gpu * (4.0 + 2.0) * (par.dp - 1) / par.dp
    # per-GPU times
    hbm_gpu = wb_dense / (par.tp * par.pp) + wb_exp / (par.ep * par.tp * par.pp) + (act + kv + temp) / gpus
    t_comp = f_re / gpus / (target.peak_tflops * 1e12)
    t_hbm = hbm_gpu / (target.hbm_gbs * 1e9)
    t_net = net / (target.link_gbs * 1e9) if net else 0.0
    t_est = max(t_comp, t_hbm, t_net)
    regime = "compute" if t_est == t_comp else ("hbm" if t_est == t_hbm else "network")
    hbm_total = w_bytes + act + kv + temp
    return ModeKpi(mode=mode, exec_model=xm.name, target=target.name, tokens=tokens, flops_theory=f_th,
                   flops_realizable=f_re, flops_tensorcore=fb.tensorcore, eta_tc=fb.eta_tc,
                   p_effective_tflops=fb.p_effective_tflops(target.peak_tflops), bytes_weights=w_bytes, bytes_activations=act, bytes_kv=kv,
                   bytes_temporary=temp, bytes_hbm=hbm_total, bytes_net=net * gpus,
                   ai_hbm=f_th / hbm_total if hbm_total else 0.0,
                   ai_total=f_th / (hbm_total + net * gpus) if hbm_total + net else 0.0,
                   t_comp_ms=t_comp * 1e3, t_hbm_ms=t_hbm * 1e3, t_net_ms=t_net * 1e3, t_est_ms=t_est * 1e3,
                   regime=regime, mfu_est=(f_th / gpus / (target.peak_tflops * 1e12)) / t_est if t_est else 0.0,
                   tokens_per_s=tokens / t_est if t_est else 0.0,
                   tokens_per_s_per_gpu=tokens / t_est / gpus if t_est else 0.0)


def estimate(model: nn.Module, *, batch: int = 1, seq_len: int = 4096, decode_ctx: int = 4096,
             parallel: Optional[ParallelismAssumptions] = None, targets: Optional[list] = None,
             exec_models: Optional[list] = None, tensor_core: Optional[TensorCoreModel] = None,
             weight_bytes: float = 2.0) -> ModelInfo:
    parallel = parallel or ParallelismAssumptions()
    targets = targets or default_roofline_targets()
    exec_models = exec_models or default_execution_models()
    tc = tensor_core or TensorCoreModel()
    tc.validate()
    for xm in exec_models:
        xm.validate()
    arch = _arch(model)
    layers = _collect_layers(model, arch)
    total = sum(p.numel() for p in model.parameters())
    by_kind: dict = {}
    for l in layers:
        by_kind[l.kind] = by_kind.get(l.kind, 0) + l.params
    active = sum(l.params * l.active_fraction for l in layers if l.kind != "embedding")
    kpis = []
    for mode in ("train", "prefill", "decode"):
        for xm in exec_models:
            for t in targets:
                kpis.append(_mode_kpi(arch, layers, mode, batch, seq_len, decode_ctx, parallel, xm, tc, t,
                                      weight_bytes, _Variant()))
    modes = []
    best_xm = exec_models[-1].name
    for mode in ("train", "prefill", "decode"):
        ks = [k for k in kpis if k.mode == mode and k.exec_model == best_xm]
        k0 = ks[0]
        per = {k.target: dict(time_ms=k.t_est_ms, bound=k.regime, tokens_per_s=k.tokens_per_s,
                              tokens_per_s_per_gpu=k.tokens_per_s_per_gpu, arithmetic_intensity=k.ai_hbm,
                              mfu_est=k.mfu_est) for k in ks}
        modes.append(ModeEstimate(mode, k0.tokens, k0.flops_theory, k0.bytes_hbm, k0.bytes_net, per))
    return ModelInfo(arch, total, active, by_kind, layers, _kv_bytes_per_token(arch), modes, kpis)


# ----------------------------------------------------------------------------- sweeps
def _interp_crossing(xs, ratios) -> Optional[float]:
    """x where ratio (t_comp / t_bound) crosses 1, log-linear between samples."""
    for (x0, r0), (x1, r1) in zip(zip(xs, ratios), zip(xs[1:], ratios[1:])):
        if r0 < 1.0 <= r1:
            if r1 == r0:
                return float(x1)
            a = (math.log(1.0) - math.log(r0)) / (math.log(r1) - math.log(r0))
            return float(math.exp(math.log(x0) + a * (math.log(x1) - math.log(x0))))
    if ratios and ratios[0] >= 1.0:
        return float(xs[0])
    return None


def _one(model, arch, layers, mode, batch, seq_len, ctx, par, xm, target, tc, var=None) -> ModeKpi:
    return _mode_kpi(arch, layers, mode, batch, seq_len, ctx, par, xm, tc, target, 2.0, var or _Variant())


def decode_sweep(model: nn.Module, batch_sizes=(1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024), ctx: int = 4096,
                 parallel: Optional[ParallelismAssumptions] = None, targets: Optional[list] = None,
                 exec_model: Optional[ExecutionModel] = None, tensor_core: Optional[TensorCoreModel] = None) -> list:
    """Decode across batch sizes: per target tokens/s, bound, and the critical batch ``b_crit`` (first
    batch that is compute bound, interpolated) in the last row's ``b_crit``."""
    par = parallel or ParallelismAssumptions()
    targets = targets or default_roofline_targets()
    xm = exec_model or default_execution_models()[-1]
    tc = tensor_core or TensorCoreModel()
    arch = _arch(model)
    layers = _collect_layers(model, arch)
    rows, ratio = [], {t.name: [] for t in targets}
    for b in batch_sizes:
        row = {"batch": b, "bound": {}, "tokens_per_s": {}}
        for t in targets:
            k = _one(model, arch, layers, "decode", b, 1, ctx, par, xm, t, tc)
            row[t.name] = k.tokens_per_s
            row["tokens_per_s"][t.name] = k.tokens_per_s
            row["bound"][t.name] = k.regime
            ratio[t.name].append(k.t_comp_ms / max(k.t_hbm_ms, k.t_net_ms, 1e-12))
        rows.append(row)
    b_crit = {t.name: _interp_crossing(list(batch_sizes), ratio[t.name]) for t in targets}
    for r in rows:
        r["b_crit"] = b_crit
    return rows


def prefill_sweep(model: nn.Module, batch_sizes=(1, 2, 4, 8, 16), seq_len: int = 4096,
                  parallel: Optional[ParallelismAssumptions] = None, target: Optional[RooflineConfig] = None,
                  exec_model: Optional[ExecutionModel] = None) -> list[ModeKpi]:
    par = parallel or ParallelismAssumptions()
    t = target or default_roofline_targets()[1]
    xm = exec_model or default_execution_models()[-1]
    tc = TensorCoreModel()
    arch = _arch(model)
    layers = _collect_layers(model, arch)
    return [_one(model, arch, layers, "prefill", b, seq_len, seq_len, par, xm, t, tc) for b in batch_sizes]


@dataclass
class DecodeEPExplorationConfig:
    ep_sizes: list = field(default_factory=lambda: [1, 2, 4, 8, 16, 32, 64])
    cache_lengths: list = field(default_factory=lambda: [2048, 4096, 8192, 16384])
    alpha: float = 0.9           # close to compute bound: t_comp >= alpha * max(t_hbm, t_net)
    max_batch_per_gpu: int = 16384


def decode_ep_exploration(model: nn.Module, cfg: Optional[DecodeEPExplorationConfig] = None,
                          target: Optional[RooflineConfig] = None, exec_model: Optional[ExecutionModel] = None,
                          ep_payload_bytes: float = 2.0) -> list[dict]:
    """Per (EP size, context): the smallest per-GPU decode batch within ``alpha`` of compute bound
    (DP = EP, TP = 1; each GPU holds E / EP experts and its own batch), or None up to the cap."""
    cfg = cfg or DecodeEPExplorationConfig()
    t = target or default_roofline_targets()[1]
    xm = exec_model or default_execution_models()[-1]
    tc = TensorCoreModel()
    arch = _arch(model)
    layers = _collect_layers(model, arch)
    E = arch["num_experts"] or 1
    out = []
    for ep in cfg.ep_sizes:
        if arch["num_experts"] and ep > E:
            continue
        par = ParallelismAssumptions(ep=ep, ep_payload_bytes=ep_payload_bytes)
        for ctx in cfg.cache_lengths:
            found = None
            b = 1
            while b <= cfg.max_batch_per_gpu:
                k = _one(model, arch, layers, "decode", b * ep, 1, ctx, par, xm, t, tc)
                if k.t_comp_ms >= cfg.alpha * max(k.t_hbm_ms, k.t_net_ms):
                    found = (b, k)
                    break
                b *= 2
            out.append({"ep": ep, "ctx": ctx, "batch_per_gpu": found[0] if found else None,
                        "tokens_per_s_per_gpu": found[1].tokens_per_s_per_gpu if found else None,
                        "regime": found[1].regime if found else "hbm/network up to the cap"})
    return out


@dataclass
class SensitivityConfig:
    name: str = "medium_full_grid"
    kv_dtype_bytes: tuple = (1, 2)
    top_k_values: tuple = (2, 4, 8)
    kv_rank_scales: tuple = (0.5, 1.0, 1.5)
    hidden_scales: tuple = (0.75, 1.0, 1.25)
    cache_lengths: tuple = (2048, 4096, 8192, 16384)
    batch: int = 64


@dataclass
class SensitivityPoint:
    exec_model: str
    kv_dtype_bytes: int
    top_k: int
    kv_rank_scale: float
    hidden_scale: float
    cache_len: int
    ai_hbm: float
    ai_total: float
    t_est_ms: float
    mfu_est: float
    regime: str


def sensitivity_grid(model: nn.Module, cfg: Optional[SensitivityConfig] = None,
                     target: Optional[RooflineConfig] = None, parallel: Optional[ParallelismAssumptions] = None,
                     exec_models: Optional[list] = None) -> list[SensitivityPoint]:
    """Decode estimates over the design grid (scaled copies of the inspected architecture)."""
    cfg = cfg or SensitivityConfig()
    t = target or default_roofline_targets()[1]
    par = parallel or ParallelismAssumptions()
    xms = exec_models or default_execution_models()
    tc = TensorCoreModel()
    arch = _arch(model)
    layers = _collect_layers(model, arch)
    pts = []
    for xm in xms:
        for kvb in cfg.kv_dtype_bytes:
            for k in cfg.top_k_values:
                for kr in cfg.kv_rank_scales:
                    for hs in cfg.hidden_scales:
                        for L in cfg.cache_lengths:
                            var = _Variant(hidden_scale=hs, top_k=k if arch["num_experts"] else None,
                                           kv_rank_scale=kr, kv_dtype_bytes=kvb)
                            m = _one(model, arch, layers, "decode", cfg.batch, 1, L, par, xm, t, tc, var)
                            pts.append(SensitivityPoint(xm.name, kvb, k, kr, hs, L, m.ai_hbm, m.ai_total,
                                                        m.t_est_ms, m.mfu_est, m.regime))
    return pts


# ----------------------------------------------------------------------------- report
def _fmt(x: float, unit: str = "") -> str:
    for s, k in (("P", 1e15), ("T", 1e12), ("G", 1e9), ("M", 1e6), ("K", 1e3)):
        if abs(x) >= k:
            return f"{x / k:.2f} {s}{unit}"
    return f"{x:.2f} {unit}"


def render_markdown(info: ModelInfo, extras: Optional[dict] = None) -> str:
    a = info.architecture
    sec = [0]

    def h(title):
        sec[0] += 1
        return ["", f"## {sec[0]}. {title}", ""]

    lines = ["# Model report"]
    lines += h("Architecture") + ["| field | value |", "|---|---|"] + [f"| {k} | {v} |" for k, v in a.items()]
    lines += ["", f"Total parameters {_fmt(info.total_params)}; active per token {_fmt(info.active_params_per_token)};"
              f" KV cache {_fmt(info.kv_cache_bytes_per_token, 'B')} per token (bf16)."]
    lines += h("Parameters by category") + ["| category | params | share |", "|---|---|---|"]
    tot = max(sum(info.params_by_kind.values()), 1)
    for k, v in sorted(info.params_by_kind.items(), key=lambda kv: -kv[1]):
        lines.append(f"| {k} | {_fmt(v)} | {100.0 * v / tot:.1f} % |")
    lines += h("Largest modules") + ["| module | kind | params | active |", "|---|---|---|---|"]
    for l in sorted(info.layers, key=lambda l: -l.params)[:15]:
        lines.append(f"| {l.name} | {l.kind} | {_fmt(l.params)} | {l.active_fraction:.3f} |")
    lines += h("Mode estimates (per GPU)")
    lines += ["| mode | exec | target | FLOP theory | FLOP tensor-core | eta_tc | FLOP realizable | P_eff TFLOP/s | "
              "HBM bytes | net bytes | AI | t_comp | t_hbm | t_net | t_est | regime | MFU est | tok/s/GPU |",
              "|" + "---|" * 18]
    for k in info.kpis:
        lines.append(f"| {k.mode} | {k.exec_model} | {k.target} | {_fmt(k.flops_theory)} | {_fmt(k.flops_tensorcore)} | "
                     f"{k.eta_tc:.3f} | {_fmt(k.flops_realizable)} | {k.p_effective_tflops:.0f} | "
                     f"{_fmt(k.bytes_hbm, 'B')} | {_fmt(k.bytes_net, 'B')} | {k.ai_hbm:.1f} | {k.t_comp_ms:.3f} | "
                     f"{k.t_hbm_ms:.3f} | {k.t_net_ms:.3f} | {k.t_est_ms:.3f} | {k.regime} | {k.mfu_est:.3f} | "
                     f"{k.tokens_per_s_per_gpu:.1f} |")
    ex = extras or {}
    if ex.get("decode_sweep"):
        rows = ex["decode_sweep"]
        names = list(rows[0]["bound"])
        lines += h("Decode batch sweep") + ["| batch | " + " | ".join(names) + " |", "|---|" + "---|" * len(names)]
        for r in rows:
            lines.append(f"| {r['batch']} | " + " | ".join(f"{r['tokens_per_s'][n]:.0f} tok/s ({r['bound'][n]})"
                                                          for n in names) + " |")
        lines += ["", "Critical batch (decode turns compute bound): " +
                  ", ".join(f"{n}: {('%.1f' % v) if v else 'not reached'}" for n, v in rows[0]["b_crit"].items())]
    if ex.get("prefill_sweep"):
        lines += h("Prefill batch sweep") + ["| batch | t_est (ms) | regime | MFU est | tok/s/GPU |",
                                             "|---|---|---|---|---|"]
        for k in ex["prefill_sweep"]:
            lines.append(f"| {k.tokens // max(1, ex.get('seq_len', 1))} | {k.t_est_ms:.3f} | {k.regime} | "
                         f"{k.mfu_est:.3f} | {k.tokens_per_s_per_gpu:.1f} |")
    if ex.get("ep_exploration"):
        lines += h("Decode expert-parallel exploration (DP = EP, TP = 1)")
        lines += ["| EP | context | batch per GPU near compute bound | tok/s/GPU |", "|---|---|---|---|"]
        for r in ex["ep_exploration"]:
            tps = f"{r['tokens_per_s_per_gpu']:.0f}" if r["tokens_per_s_per_gpu"] else "-"
            lines.append(f"| {r['ep']} | {r['ctx']} | {r['batch_per_gpu'] or 'not reached'} | {tps} |")
    if ex.get("sensitivity"):
        pts = ex["sensitivity"]
        lines += h(f"Sensitivity grid ({len(pts)} points, decode)")
        counts: dict = {}
        for p in pts:
            counts[p.regime] = counts.get(p.regime, 0) + 1
        lines.append("Regimes: " + ", ".join(f"{k} {v}" for k, v in sorted(counts.items())))
        lines += ["", "| exec | kv bytes | top-k | kv rank x | hidden x | context | AI | t_est (ms) | MFU | regime |",
                  "|" + "---|" * 10]
        for p in sorted(pts, key=lambda p: p.t_est_ms)[:8] + sorted(pts, key=lambda p: -p.t_est_ms)[:8]:
            lines.append(f"| {p.exec_model} | {p.kv_dtype_bytes} | {p.top_k} | {p.kv_rank_scale} | {p.hidden_scale} | "
                         f"{p.cache_len} | {p.ai_hbm:.1f} | {p.t_est_ms:.3f} | {p.mfu_est:.3f} | {p.regime} |")
    return "\n".join(lines) + "\n"


def plot_roofline(info: ModelInfo, path: str, targets: Optional[list] = None) -> str:
    """Roofline of every target (attainable TFLOP/s against FLOP per HBM byte) with the model's
    operating points (one per mode and execution model, on the first target) as an SVG file."""
    from .svg_plot import Series, loglog_svg

    targets = targets or default_roofline_targets()
    kp = [k for k in info.kpis if k.t_est_ms > 0 and k.ai_hbm > 0]
    lo = min([k.ai_hbm for k in kp] + [1.0]) / 4
    hi = max([k.ai_hbm for k in kp] + [t.knee for t in targets]) * 4
    xs = [lo * (hi / lo) ** (i / 60) for i in range(61)]
    series = [Series(f"{t.name} roof", xs, [min(t.peak_tflops, x * t.hbm_gbs / 1e3) for x in xs], dashed=True)
              for t in targets]
    first = targets[0].name if targets else None
    for xm in sorted({k.exec_model for k in kp}):
        pts = [k for k in kp if k.exec_model == xm and k.target == first]
        series.append(Series(f"{xm} ({first})", [k.ai_hbm for k in pts],
                             [k.flops_realizable / (k.t_est_ms * 1e-3) / 1e12 for k in pts], kind="points",
                             point_labels=[k.mode for k in pts]))
    return loglog_svg(path, series, title="Roofline and operating points", xlabel="FLOP per HBM byte",
                      ylabel="TFLOP/s per GPU")


def plot_decode_sweep(rows: list, path: str) -> str:
    """Decode tokens/s per GPU against the batch size, one line per target, as an SVG file."""
    from .svg_plot import Series, loglog_svg

    names = list(rows[0]["tokens_per_s"]) if rows else []
    series = [Series(n, [r["batch"] for r in rows], [r["tokens_per_s"][n] for r in rows]) for n in names]
    return loglog_svg(path, series, title="Decode throughput against batch", xlabel="batch (sequences)",
                      ylabel="tokens/s")


def dump_model_info(model: nn.Module, output_path: str, *, sweeps: bool = True,
                    sensitivity: Optional[SensitivityConfig] = None, plots: bool = True, **kw) -> ModelInfo:
    """Write the Markdown report (and a JSON twin, and with ``plots`` SVG charts beside them:
    ``<name>_roofline.svg``, ``<name>_decode_sweep.svg``) for ``model``; returns the estimate."""
    info = estimate(model, **kw)
    extras: dict = {}
    if sweeps:
        par = kw.get("parallel")
        extras["decode_sweep"] = decode_sweep(model, ctx=kw.get("decode_ctx", 4096), parallel=par,
                                              targets=kw.get("targets"))
        extras["seq_len"] = kw.get("seq_len", 4096)
        extras["prefill_sweep"] = prefill_sweep(model, seq_len=kw.get("seq_len", 4096), parallel=par)
        if info.architecture["num_experts"]:
            extras["ep_exploration"] = decode_ep_exploration(model)
        extras["sensitivity"] = sensitivity_grid(model, sensitivity, parallel=par)
    os.makedirs(os.path.dirname(os.path.abspath(output_path)), exist_ok=True)
    base = os.path.splitext(output_path)[0]
    plot_files = []
    if plots:
        plot_files.append(plot_roofline(info, base + "_roofline.svg", kw.get("targets")))
        if extras.get("decode_sweep"):
            plot_files.append(plot_decode_sweep(extras["decode_sweep"], base + "_decode_sweep.svg"))
    with open(output_path, "w") as f:
        f.write(render_markdown(info, extras))
        if plot_files:
            f.write("\n## Plots\n\n" + "\n".join(f"![{os.path.basename(p)}]({os.path.basename(p)})"
                                                     for p in plot_files) + "\n")
    js = {"architecture": info.architecture, "total_params": info.total_params,
          "active_params_per_token": info.active_params_per_token, "params_by_kind": info.params_by_kind,
          "kv_cache_bytes_per_token": info.kv_cache_bytes_per_token,
          "layers": [asdict(l) for l in info.layers], "modes": [asdict(m) for m in info.modes],
          "kpis": [asdict(k) for k in info.kpis]}
    if extras:
        js["decode_sweep"] = extras["decode_sweep"]
        js["prefill_sweep"] = [asdict(k) for k in extras["prefill_sweep"]]
        js["ep_exploration"] = extras.get("ep_exploration", [])
        js["sensitivity"] = [asdict(p) for p in extras["sensitivity"]]
    js["plots"] = [os.path.basename(p) for p in plot_files]
    with open(base + ".json", "w") as f:
        json.dump(js, f, indent=1)
    return info


__all__ = ["RooflineConfig", "default_roofline_targets", "ExecutionModel", "default_execution_models",
           "TensorCoreModel", "ParallelismAssumptions", "ModelInfo", "ModeKpi", "estimate", "dump_model_info",
           "render_markdown", "decode_sweep", "prefill_sweep", "DecodeEPExplorationConfig", "decode_ep_exploration",
           "SensitivityConfig", "SensitivityPoint", "sensitivity_grid", "plot_roofline", "plot_decode_sweep"]
