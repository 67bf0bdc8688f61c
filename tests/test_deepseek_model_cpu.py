"""DeepSeek model on CPU: shapes, backward, bf16 parameters with an explicit float mask, meta
initialisation, pipeline stage partitioning (even split with the remainder on early stages, or explicit
splits), stage module ownership, and pipeline stages chained by hand against the whole model.

Behaviour follows the reference's tests/test_deepseek_model.py."""
import argparse

import pytest
import torch

from nano_train_b200.models.deepseek import DeepSeekModel, DeepSeekModelConfig, DeepSeekParallelContext
from nano_train_b200.precision.mixed_precision import build_module_precision_resolver, resolve_precision_config


def _cfg(layers=5, **kw):
    resolver = build_module_precision_resolver(resolve_precision_config(argparse.Namespace(), torch.device("cpu")))
    base = dict(precision_resolver=resolver, param_dtype=torch.float32, param_device=None, vocab_size=97,
                hidden_size=64, num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=4,
                intermediate_size=128, q_lora_rank=24, kv_lora_rank=16, qk_nope_head_dim=8, qk_rope_head_dim=8, v_head_dim=8,
                moe_intermediate_size=32, n_routed_experts=4, num_experts_per_tok=2, n_group=1, topk_group=1,
                max_position_embeddings=32, first_k_dense_replace=1)
    base.update(kw)
    return DeepSeekModelConfig(**base)


def test_forward_shape_and_backward():
    torch.manual_seed(0)
    m = DeepSeekModel(_cfg(layers=2))
    ids = torch.randint(0, 97, (2, 11))
    logits = m(ids)
    assert logits.shape == (2, 11, 97) and torch.isfinite(logits).all()
    torch.nn.functional.cross_entropy(logits.reshape(-1, 97), ids.reshape(-1)).backward()
    missing = [n for n, p in m.named_parameters() if p.grad is None]
    # every parameter gets a gradient except experts that no token was routed to
    assert all(".experts." in n for n in missing), missing


def test_bf16_parameters_with_an_explicit_float_mask():
    torch.manual_seed(0)
    m = DeepSeekModel(_cfg(layers=2, param_dtype=torch.bfloat16))
    ids = torch.randint(0, 97, (2, 9))
    mask = m._create_causal_mask(2, 9, ids.device)
    assert mask.dtype == torch.float32 and mask.shape == (2, 1, 9, 9)
    out = m(ids, attention_mask=mask)
    assert out.shape == (2, 9, 97) and torch.isfinite(out.float()).all()
    torch.testing.assert_close(out.float(), m(ids).float(), atol=3e-2, rtol=3e-2)


def test_meta_initialisation_allocates_no_storage():
    m = DeepSeekModel(_cfg(param_device=torch.device("meta")))
    assert all(p.device.type == "meta" for p in m.parameters())
    assert m.num_parameters > 0


@pytest.mark.parametrize("layers, pp, expected", [(5, 2, (0, 3, 5)), (5, 3, (0, 2, 4, 5)), (8, 4, (0, 2, 4, 6, 8)),
                                                  (7, 1, (0, 7))])
def test_even_stage_partition_puts_the_remainder_on_early_stages(layers, pp, expected):
    for r in range(pp):
        pc = DeepSeekParallelContext(pipeline_model_parallel_rank=r, pipeline_model_parallel_size=pp)
        assert pc.resolve_pp_layer_boundaries(layers) == expected
        assert pc.resolve_pp_layer_range(layers) == (expected[r], expected[r + 1])


def test_explicit_stage_splits_and_their_validation():
    pc = DeepSeekParallelContext(pipeline_model_parallel_rank=1, pipeline_model_parallel_size=2,
                                 pp_layer_splits=(0, 1, 5))
    assert pc.resolve_pp_layer_range(5) == (1, 5)
    with pytest.raises(ValueError, match="last value"):
        pc.resolve_pp_layer_boundaries(6)
    for splits, msg in (((0, 3), "length"), ((1, 2, 5), "start with 0"), ((0, 3, 3), "strictly increasing")):
        with pytest.raises(ValueError, match=msg):
            DeepSeekParallelContext(pipeline_model_parallel_size=2, pp_layer_splits=splits)
    with pytest.raises(ValueError, match="rank must be in"):
        DeepSeekParallelContext(pipeline_model_parallel_rank=2, pipeline_model_parallel_size=2)


def _stage(rank, pp, layers=5, splits=None):
    pc = DeepSeekParallelContext(pipeline_model_parallel_rank=rank, pipeline_model_parallel_size=pp,
                                 pp_layer_splits=splits)
    return DeepSeekModel(_cfg(layers=layers), parallel_context=pc)


def test_stage_module_ownership():
    first, middle, last = _stage(0, 3), _stage(1, 3), _stage(2, 3)
    assert first.token_embeddings is not None and first.lm_head is None and first.final_norm is None
    assert middle.token_embeddings is None and middle.lm_head is None
    assert last.token_embeddings is None and last.lm_head is not None and last.final_norm is not None
    assert [len(s.blocks) for s in (first, middle, last)] == [2, 2, 1]
    assert first.local_layer_range() == (0, 2) and last.local_layer_range() == (4, 5)
    # decoder layers keep their global index in their module paths (dense layer 0, MoE layers after it)
    assert last.blocks[0].attn.q_b_proj.module_path == "blocks.4.attn.q_b_proj"
    with pytest.raises(RuntimeError, match="only valid for pipeline_model_parallel_size==1"):
        first(torch.zeros(1, 4, dtype=torch.long))
    with pytest.raises(ValueError, match="input_ids is required"):
        first.forward_stage(None, None)
    with pytest.raises(ValueError, match="hidden_states is required"):
        last.forward_stage(None, None)


def test_stages_chained_by_hand_match_the_whole_model():
    torch.manual_seed(0)
    whole = DeepSeekModel(_cfg(layers=5))
    whole.eval()
    stages = [_stage(0, 2, splits=(0, 2, 5)), _stage(1, 2, splits=(0, 2, 5))]
    full = whole.state_dict()
    for s in stages:
        start, _ = s.local_layer_range()
        sd = {}
        for k in s.state_dict():
            if k.startswith("blocks."):
                _, i, rest = k.split(".", 2)
                sd[k] = full[f"blocks.{int(i) + start}.{rest}"]
            else:
                sd[k] = full[k]
        s.load_state_dict(sd, strict=True)
        s.eval()
    ids = torch.randint(0, 97, (2, 10))
    with torch.no_grad():
        h = stages[0].forward_stage(ids, None)
        assert h.shape == (2, 10, 64)
        logits = stages[1].forward_stage(None, h)
        torch.testing.assert_close(logits, whole(ids), atol=1e-5, rtol=1e-5)


def test_mla_fused_path_gate():
    """The fused MLA key assembly is taken only for CUDA bf16 tensors with 16-byte rows and the head
    dims of a tcgen05 attention kernel; CPU tensors and other shapes keep the reference formulation."""
    from nano_train_b200.models.deepseek import _mla_fused_ok

    q = torch.zeros(1, 4, 2, 192, dtype=torch.bfloat16)
    kv = torch.zeros(1, 4, 2, 256, dtype=torch.bfloat16)
    k_rope = torch.zeros(1, 4, 576, dtype=torch.bfloat16)[..., 512:]
    assert not _mla_fused_ok(q, kv, k_rope, 128)  # CPU tensors
