"""Behaviour a user of the reference relies on when switching: module names and the 3-D
attention API with masks and monitoring, precision-override output dtypes, legacy checkpoints
without persistent low-bit buffers, the per-parameter AdamW, loss edge cases, logging setup,
the Transformer Engine binding contract and the MoE payload-quantisation defaults."""
import argparse
import logging
import math
import sys
import types

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from nano_train_b200.config import ModelConfig
from nano_train_b200.models.transformer import MultiHeadAttention, TransformerModel
from nano_train_b200.precision.mixed_precision import build_module_precision_resolver, resolve_precision_config
from nano_train_b200.runtime.contracts import ModulePrecisionPolicy, PrecisionConfig


def _resolver(**policy):
    if policy:
        return build_module_precision_resolver(PrecisionConfig(mode="fp32",
                                                               module_precision_policy=ModulePrecisionPolicy(**policy)))
    return build_module_precision_resolver(PrecisionConfig(mode="fp32"))


def _gpt(**kw):
    cfg = dict(param_dtype=torch.float32, param_device=None, precision_resolver=_resolver(), hidden_size=32,
               num_layers=2, num_attention_heads=4, intermediate_size=64, vocab_size=97, max_position_embeddings=16,
               dropout=0.0)
    cfg.update(kw)
    return ModelConfig(**cfg)


def test_transformer_state_dict_uses_reference_module_names():
    names = set(TransformerModel(_gpt()).state_dict())
    for n in ("blocks.0.attention.qkv_proj.weight", "blocks.0.attention.out_proj.bias", "blocks.0.attn_norm.weight",
              "blocks.1.mlp_norm.bias", "blocks.1.mlp.fc1.weight", "ln_f.weight", "token_embeddings.weight",
              "position_embeddings.weight"):
        assert n in names, n


def test_explicit_causal_mask_matches_implicit_path():
    torch.manual_seed(0)
    m = TransformerModel(_gpt()).eval()
    ids = torch.randint(0, 97, (2, 9))
    mask = m._create_causal_mask(2, 9, ids.device)
    torch.testing.assert_close(m(ids, attention_mask=mask), m(ids), rtol=1e-5, atol=1e-5)


def test_attention_module_api_mask_and_monitoring():
    torch.manual_seed(0)
    attn = MultiHeadAttention(_gpt(), module_prefix="attention").eval()
    x = torch.randn(2, 5, 32)
    full = attn(x)  # no mask: every position sees every position
    q, k, v = attn.qkv_proj(x).split(32, -1)
    sh = lambda t: t.view(2, 5, 4, 8).transpose(1, 2)  # noqa: E731
    ref = F.scaled_dot_product_attention(sh(q), sh(k), sh(v)).transpose(1, 2).reshape(2, 5, 32)
    torch.testing.assert_close(full, attn.out_proj(ref), rtol=1e-5, atol=1e-5)
    attn.set_monitoring(True, tau=0.0)
    attn(x, attention_mask=torch.zeros(2, 1, 5, 5))
    st = attn._monitor_stats
    assert 0.0 <= st["attn_entropy"] <= math.log(5) + 1e-5 and 0.0 <= st["attn_entropy_norm"] <= 1.0 + 1e-5
    assert 0.0 <= st["frac_logits_gt_tau"] <= 1.0 and math.isfinite(st["max_attn_logit"])
    attn.set_monitoring(False)
    assert attn._monitor_stats is None
    bf = MultiHeadAttention(_gpt(param_dtype=torch.bfloat16), module_prefix="attention").eval()
    out = bf(x.bfloat16(), attention_mask=torch.zeros(2, 1, 5, 5))  # fp32 mask upcasts the scores
    assert out.dtype == torch.bfloat16


def test_compute_dtype_override_sets_the_output_dtype():
    from nano_train_b200.layers import LayerNorm, Linear, RMSNorm

    args = argparse.Namespace(module_compute_dtype_rule=["^lin=fp16", "^ln=bf16", "^rms=fp16"])
    res = build_module_precision_resolver(resolve_precision_config(args, torch.device("cpu")))
    lin = Linear(4, 3, module_path="lin", precision_resolver=res)
    ln = LayerNorm(4, module_path="ln", precision_resolver=res)
    rms = RMSNorm(4, module_path="rms", precision_resolver=res)
    x = torch.randn(2, 4)
    assert lin(x).dtype == torch.float16 and ln(x).dtype == torch.bfloat16 and rms(x).dtype == torch.float16


def test_legacy_state_dict_without_persistent_buffers_loads_strictly():
    from nano_train_b200.layers import Linear

    res = lambda: _resolver(persistent_lowbit_mode="fp8", persistent_lowbit_include=("lin",))  # noqa: E731
    src = Linear(4, 3, module_path="lin", precision_resolver=res())
    legacy = {k: v for k, v in src.state_dict().items() if "_persistent_" not in k}
    dst = Linear(4, 3, module_path="lin", precision_resolver=res())
    dst.load_state_dict(legacy, strict=True)
    assert torch.equal(dst.weight, src.weight)
    assert torch.equal(dst._persistent_fp8_weight.float(), src._persistent_fp8_weight.float())


def test_adamw_matches_torch():
    from nano_train_b200.optimizer import AdamW

    torch.manual_seed(0)
    a, b = nn.Linear(6, 3), nn.Linear(6, 3)
    b.load_state_dict(a.state_dict())
    oa = AdamW(a.parameters(), lr=1e-2, betas=(0.9, 0.99), weight_decay=0.05)
    ob = torch.optim.AdamW(b.parameters(), lr=1e-2, betas=(0.9, 0.99), weight_decay=0.05)
    for _ in range(4):
        x = torch.randn(5, 6)
        for m, o in ((a, oa), (b, ob)):
            o.zero_grad()
            m(x).square().sum().backward()
            o.step()
    for p, q in zip(a.parameters(), b.parameters()):
        torch.testing.assert_close(p, q, rtol=1e-6, atol=1e-7)
    assert oa.state[a.weight]["step"] == 4 and {"exp_avg", "exp_avg_sq"} <= set(oa.state[a.weight])


def test_cross_entropy_reductions_and_all_ignored():
    from nano_train_b200.losses import CrossEntropyLoss

    logits, t = torch.randn(10, 7), torch.randint(0, 7, (10,))
    assert CrossEntropyLoss(reduction="sum")(logits, t).item() == CrossEntropyLoss(reduction="none")(logits, t).sum().item()
    assert CrossEntropyLoss()(logits, torch.full((10,), -100)).item() == 0.0


def test_setup_logging_reference_signature(tmp_path):
    from nano_train_b200.logging import get_logger, setup_logging

    setup_logging(log_level="DEBUG", log_file=str(tmp_path / "x.log"), use_colors=False)
    get_logger("t").debug("hello")
    assert logging.getLogger().level == logging.DEBUG and "hello" in (tmp_path / "x.log").read_text()
    with pytest.raises(ValueError):
        setup_logging(log_level="LOUD")
    setup_logging(log_level="INFO", use_colors=False)


def test_transformer_engine_backend_binds_layer_parameters(monkeypatch):
    from nano_train_b200.precision.backends import build_lowbit_backend_for_mode
    from nano_train_b200.runtime.contracts import LowBitKernelSpec

    te = types.ModuleType("transformer_engine")
    tp = types.ModuleType("transformer_engine.pytorch")

    class _Lin(nn.Module):
        def __init__(self, in_features, out_features, bias=True):
            super().__init__()
            self.weight = nn.Parameter(torch.zeros(out_features, in_features))
            self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

        def forward(self, x):
            return F.linear(x, self.weight, self.bias)

    tp.Linear = _Lin
    te.pytorch = tp
    monkeypatch.setitem(sys.modules, "transformer_engine", te)
    monkeypatch.setitem(sys.modules, "transformer_engine.pytorch", tp)
    be = build_lowbit_backend_for_mode(PrecisionConfig(mode="fp8", fp8_backend="transformer_engine"), mode="fp8",
                                       kernel_spec=LowBitKernelSpec(module_type="linear", in_features=4,
                                                                    out_features=3, has_bias=True))
    with pytest.raises(RuntimeError, match="before parameter binding"):
        be.linear(torch.randn(2, 4), torch.randn(3, 4), torch.randn(3))
    w, bias = nn.Parameter(torch.randn(3, 4)), nn.Parameter(torch.randn(3))
    be.bind_parameters(w, bias)
    x = torch.randn(5, 4, requires_grad=True)
    be.linear(x, w, bias).sum().backward()
    assert w.grad is not None and bias.grad is not None and be._te_linear.weight is w
    assert be.linear(x.detach(), w + 0.0, bias).shape == (5, 3)


def test_moe_payload_quantisation_follows_the_recipe():
    from nano_train_b200.models.moe import ExpertParallelMoE, _comm_quant_dequant

    def build(**over):
        args = argparse.Namespace(precision_recipe="deepseek_v3", fp8=True, fp8_backend="emulated", **over)
        res = build_module_precision_resolver(resolve_precision_config(args, torch.device("cpu")))
        return ExpertParallelMoE(16, 32, 4, 2, ep_rank=0, ep_size=1, precision_resolver=res)

    m = build()
    assert m._comm_quant_enabled and m._comm_quant_granularity == "block_128x128"
    assert m._comm_quant_rounding_mode == "stochastic" and m.global_expert_start == 0
    assert build(fp8_comm_quant=False)._comm_quant_enabled is False
    x = torch.randn(7, 257, requires_grad=True)
    y = _comm_quant_dequant(x, granularity="block_128x128", rounding_mode="stochastic", bits=8)
    assert y.shape == x.shape and y.dtype == x.dtype
    y.sum().backward()
    assert x.grad is not None


def test_mla_without_q_lora_projects_q_directly():
    from nano_train_b200.models.deepseek import DeepSeekModel, DeepSeekModelConfig

    def cfg(q_lora):
        return DeepSeekModelConfig(param_dtype=torch.float32, param_device=None, precision_resolver=_resolver(),
                                   vocab_size=97, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                   num_key_value_heads=4, intermediate_size=128, q_lora_rank=q_lora, kv_lora_rank=16,
                                   qk_nope_head_dim=8, qk_rope_head_dim=8, v_head_dim=8, moe_intermediate_size=32,
                                   n_routed_experts=4, num_experts_per_tok=2, n_group=1, topk_group=1,
                                   max_position_embeddings=32)

    torch.manual_seed(0)
    m = DeepSeekModel(cfg(None))
    names = set(dict(m.named_parameters()))
    assert "blocks.0.attn.q_proj.weight" in names and not any("q_a_proj" in n for n in names)
    assert tuple(m.blocks[0].attn.q_proj.weight.shape) == (4 * 16, 64)
    ids = torch.randint(0, 97, (2, 9))
    logits = m(ids)
    assert logits.shape == (2, 9, 97) and torch.isfinite(logits).all()
    logits.float().mean().backward()
    assert m.blocks[0].attn.q_proj.weight.grad is not None
    with_lora = DeepSeekModel(cfg(24))
    assert "blocks.0.attn.q_a_proj.weight" in dict(with_lora.named_parameters())
