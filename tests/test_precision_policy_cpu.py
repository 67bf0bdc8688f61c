"""Per-module precision policy on CPU: include/exclude patterns, compute-dtype override rules,
rejection of patterns that reach modules without low-bit support, DeepSeek-V3 recipe propagation into
the backends, persistent low-bit weights that train through the fp32 master, the eval artifact hash
and the schedule selector.

Behaviour follows the reference's tests test_module_precision_policy_resolution.py,
test_module_precision_policy_unsupported_module.py, test_fp8_granularity_semantics.py,
test_persistent_lowbit_trainability.py, test_probe_hash.py and test_runtime_schedule_selector.py."""
import argparse
from types import SimpleNamespace

import pytest
import torch

from nano_train_b200.layers import LayerNorm, Linear, RMSNorm
from nano_train_b200.monitoring import eval_artifact_hash
from nano_train_b200.precision.mixed_precision import (build_module_precision_resolver,
                                                       finalize_module_precision_resolver, resolve_precision_config)
from nano_train_b200.runtime.schedules import DefaultScheduleSelector

CPU = torch.device("cpu")


def _resolver(**flags):
    return build_module_precision_resolver(resolve_precision_config(argparse.Namespace(**flags), CPU))


def _fp8(**flags):
    return _resolver(fp8=True, fp8_backend="emulated", **flags)


def test_exclude_pattern_keeps_a_module_in_high_precision():
    r = _fp8(compute_lowbit_exclude=[r"\.fc2$"])
    fc1 = Linear(16, 16, module_path="blk.fc1", precision_resolver=r)
    fc2 = Linear(16, 16, module_path="blk.fc2", precision_resolver=r)
    s = finalize_module_precision_resolver(r)
    assert fc1._compute_lowbit_mode() == "fp8" and fc1._lowbit_backend is not None
    assert fc2._compute_lowbit_mode() is None and fc2._lowbit_backend is None
    assert (s.parameterized_module_count, s.lowbit_capable_module_count, s.compute_lowbit_module_count) == (2, 2, 1)


def test_glob_patterns_and_include_must_match_a_module():
    r = _fp8(module_pattern_type="glob", compute_lowbit_include=["*.mlp.*"])
    a = Linear(8, 8, module_path="layers.0.mlp.fc1", precision_resolver=r)
    b = Linear(8, 8, module_path="layers.0.attention.qkv", precision_resolver=r)
    finalize_module_precision_resolver(r)
    assert a._compute_lowbit_mode() == "fp8" and b._compute_lowbit_mode() is None

    r = _fp8(compute_lowbit_include=["no_such_module"], compute_lowbit_exclude=[])
    Linear(8, 8, module_path="blk.fc1", precision_resolver=r)
    with pytest.raises(ValueError, match="matched zero modules"):
        finalize_module_precision_resolver(r)


def test_lowbit_mode_with_no_assigned_module_is_an_error():
    r = _fp8(compute_lowbit_exclude=[".*"])
    Linear(8, 8, module_path="blk.fc1", precision_resolver=r)
    with pytest.raises(RuntimeError, match="zero modules were assigned"):
        finalize_module_precision_resolver(r)


def test_duplicate_module_path_is_rejected():
    r = _resolver()
    Linear(4, 4, module_path="x", precision_resolver=r)
    with pytest.raises(ValueError, match="Duplicate module_path"):
        Linear(4, 4, module_path="x", precision_resolver=r)


def test_compute_dtype_override_on_a_plain_linear_sets_the_output_dtype():
    r = _resolver(module_compute_dtype_rule=[r"blk\.fc1$=bf16"])
    fc1 = Linear(16, 8, module_path="blk.fc1", precision_resolver=r)
    fc2 = Linear(16, 8, module_path="blk.fc2", precision_resolver=r)
    finalize_module_precision_resolver(r)
    x = torch.randn(3, 16)
    y1, y2 = fc1(x), fc2(x)
    assert y1.dtype == torch.bfloat16 and y2.dtype == torch.float32
    ref = x.bfloat16().float() @ fc1.weight.bfloat16().float().t() + fc1.bias.bfloat16().float()
    torch.testing.assert_close(y1.float(), ref, atol=2e-2, rtol=2e-2)


def test_compute_dtype_override_conflicts_with_lowbit_assignment():
    r = _fp8(module_compute_dtype_rule=[r"fc1=fp32"])
    with pytest.raises(ValueError, match="both low-bit compute and compute-dtype override"):
        Linear(8, 8, module_path="blk.fc1", precision_resolver=r)


def test_unmatched_dtype_rule_and_malformed_rules_are_rejected():
    r = _resolver(module_compute_dtype_rule=["nothing_here=bf16"])
    Linear(4, 4, module_path="blk.fc1", precision_resolver=r)
    with pytest.raises(ValueError, match="rules matched zero modules"):
        finalize_module_precision_resolver(r)
    with pytest.raises(ValueError, match="format"):
        _resolver(module_compute_dtype_rule=["fc1:bf16"])
    with pytest.raises(ValueError, match="dtype must be one of"):
        _resolver(module_compute_dtype_rule=["fc1=int8"])


@pytest.mark.parametrize("cls", [LayerNorm, RMSNorm])
def test_compute_dtype_override_applies_to_norms(cls):
    r = _resolver(module_compute_dtype_rule=[r"norm$=bf16"])
    n = cls(32, module_path="layers.0.attn_norm", precision_resolver=r)
    finalize_module_precision_resolver(r)
    x = torch.randn(2, 5, 32)
    y = n(x)
    assert y.dtype == torch.bfloat16
    xb = x.bfloat16().float()
    if cls is LayerNorm:
        ref = torch.nn.functional.layer_norm(xb, (32,), eps=n.eps)
    else:
        ref = xb * torch.rsqrt(xb.pow(2).mean(-1, keepdim=True) + n.eps)
    torch.testing.assert_close(y.float(), ref, atol=3e-2, rtol=3e-2)


def test_lowbit_pattern_reaching_a_module_without_lowbit_support_is_rejected():
    r = _fp8(compute_lowbit_include=["norm"])
    with pytest.raises(ValueError, match="without low-bit support"):
        LayerNorm(16, module_path="layers.0.attn_norm", precision_resolver=r)
    r = _resolver(fp8_param=True, persistent_lowbit_include=["norm"])
    with pytest.raises(ValueError, match="without low-bit support"):
        LayerNorm(16, module_path="layers.0.mlp_norm", precision_resolver=r)


def test_flag_conflicts():
    with pytest.raises(ValueError, match="At most one"):
        _resolver(fp8=True, fp4=True)
    with pytest.raises(ValueError, match="At most one of --fp8-param/--fp4-param"):
        _resolver(fp8_param=True, fp4_param=True)
    with pytest.raises(ValueError, match="requires --fp8"):
        _resolver(precision_recipe="deepseek_v3", fp4=True)
    with pytest.raises(ValueError, match="--bf16 requires CUDA"):
        _resolver(bf16=True)


def test_deepseek_recipe_propagates_tile_block_stochastic_to_the_backend():
    r = _resolver(precision_recipe="deepseek_v3", fp8_backend="emulated")
    fc = Linear(256, 256, module_path="layers.0.mlp.fc1", precision_resolver=r)
    head = Linear(256, 64, module_path="lm_head", precision_resolver=r)
    router = Linear(256, 8, bias=False, module_path="layers.0.mlp.router.gate", precision_resolver=r)
    s = finalize_module_precision_resolver(r)
    b = fc._lowbit_backend
    assert (b._activation_granularity, b._weight_granularity, b._rounding_mode) == \
        ("tile_1x128", "block_128x128", "stochastic")
    # embeddings, LM head, norms and the router stay in high precision
    assert head._compute_lowbit_mode() is None and router._compute_lowbit_mode() is None
    assert s.high_precision_exception_module_count == 2 and s.compute_lowbit_module_count == 1


def test_recipe_overrides_reach_the_backend():
    r = _resolver(precision_recipe="deepseek_v3", fp8_backend="emulated", fp8_activation_granularity="channel",
                  fp8_weight_granularity="tensor", fp8_rounding="nearest")
    fc = Linear(64, 64, module_path="blk.fc", precision_resolver=r)
    b = fc._lowbit_backend
    assert (b._activation_granularity, b._weight_granularity, b._rounding_mode) == ("channel", "tensor", "nearest")
    with pytest.raises(ValueError, match="granularity must be one of"):
        _resolver(precision_recipe="deepseek_v3", fp8_activation_granularity="row")


@pytest.mark.parametrize("shape", [(3, 100), (2, 5, 200), (1, 130)])
def test_emulated_granularities_run_on_shapes_that_need_padding(shape):
    r = _resolver(precision_recipe="deepseek_v3", fp8_backend="emulated")
    fc = Linear(shape[-1], 70, module_path="blk.fc", precision_resolver=r)
    x = torch.randn(*shape)
    y = fc(x)
    assert y.shape == (*shape[:-1], 70) and torch.isfinite(y).all()
    # e4m3 round trips of both operands: within a few percent of the fp32 product
    ref = x @ fc.weight.t() + fc.bias
    assert float((y - ref).detach().norm() / ref.detach().norm()) < 0.1


@pytest.mark.parametrize("flag", ["fp8_param", "fp4_param"])
def test_persistent_lowbit_weights_train_through_the_master_parameter(flag):
    torch.manual_seed(0)
    r = _resolver(**{flag: True})
    fc = Linear(32, 32, module_path="blk.fc", precision_resolver=r)
    finalize_module_precision_resolver(r)
    assert fc._persistent_mode() == ("fp8" if flag == "fp8_param" else "fp4")
    opt = torch.optim.SGD(fc.parameters(), lr=0.5)
    x, target = torch.randn(64, 32), torch.randn(64, 32) * 0.1
    w0 = fc.weight.detach().clone()
    losses = []
    for _ in range(20):
        opt.zero_grad()
        loss = torch.nn.functional.mse_loss(fc(x), target)
        loss.backward()
        assert fc.weight.grad is not None and fc.weight.grad.abs().sum() > 0  # STE reaches the master
        opt.step()
        fc.refresh_persistent_lowbit_params()
        losses.append(loss.item())
    assert losses[-1] < 0.7 * losses[0]
    assert not torch.equal(fc.weight.detach(), w0)


def test_eval_artifact_hash_is_deterministic_and_sensitive():
    ids, labels = torch.arange(12, dtype=torch.int64), torch.arange(1, 13, dtype=torch.int64)

    def h(**kw):
        base = dict(input_ids_bytes=ids.numpy().tobytes(), labels_bytes=labels.numpy().tobytes(),
                    input_dtype="int64", labels_dtype="int64", input_shape=(3, 4), labels_shape=(3, 4),
                    vocab_size=100, max_seq_length=4, seed=1)
        base.update(kw)
        return eval_artifact_hash(**base)

    a = h()
    assert a == h() and len(a) == 64
    changed = [h(seed=2), h(vocab_size=101), h(input_shape=(4, 3)), h(max_seq_length=5),
               h(labels_bytes=(labels + 1).numpy().tobytes()), h(input_dtype="int32")]
    assert all(c != a for c in changed) and len(set(changed)) == len(changed)


def test_default_schedule_selector():
    plain, pipe = object(), object()
    sel = DefaultScheduleSelector(non_pipeline_schedule=plain, pipeline_schedule=pipe)
    ctx = lambda pp: SimpleNamespace(parallel=SimpleNamespace(pipeline_model_parallel_size=pp))  # noqa: E731
    assert sel.select(ctx(1)) is plain
    assert sel.select(ctx(2)) is pipe and sel.select(ctx(4)) is pipe


def _tiny_deepseek(resolver, overrides):
    from nano_train_b200.models.deepseek import DeepSeekModel, DeepSeekModelConfig

    cfg = DeepSeekModelConfig(param_dtype=torch.float32, param_device=None, precision_resolver=resolver,
                              vocab_size=97, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                              num_key_value_heads=4, intermediate_size=128, q_lora_rank=24, kv_lora_rank=16,
                              qk_nope_head_dim=8, qk_rope_head_dim=8, v_head_dim=8, moe_intermediate_size=32,
                              n_routed_experts=4, num_experts_per_tok=2, n_group=1, topk_group=1,
                              max_position_embeddings=32, module_compute_dtype_overrides=overrides)
    return DeepSeekModel(cfg), cfg


def test_deepseek_exact_path_overrides_disable_lowbit_for_that_module():
    torch.manual_seed(0)
    # out_proj feeds the residual add, so a bf16 output there mixes with the fp32 stream by promotion
    model, cfg = _tiny_deepseek(_fp8(), {"blocks.0.attn.out_proj": "bf16"})
    finalize_module_precision_resolver(cfg.precision_resolver)
    over, other = model.blocks[0].attn.out_proj, model.blocks[1].attn.out_proj
    assert over._compute_lowbit_mode() is None and over._lowbit_backend is None
    assert over._module_compute_dtype_override() == torch.bfloat16
    assert other._compute_lowbit_mode() == "fp8"
    logits = model(torch.randint(0, 97, (2, 7)))
    assert logits.shape == (2, 7, 97) and torch.isfinite(logits).all()


def test_deepseek_exact_path_override_must_match_a_module():
    model, cfg = _tiny_deepseek(_fp8(), {"blocks.9.attn.q_b_proj": "fp32"})
    with pytest.raises(ValueError, match="matched zero modules"):
        finalize_module_precision_resolver(cfg.precision_resolver)
    with pytest.raises(ValueError, match="values must be one of"):
        _tiny_deepseek(_resolver(), {"blocks.0.attn.q_b_proj": "int4"})
