"""tcgen05 flash attention (head dims 128, MLA 192/128 and 64) vs fp32 PyTorch and the mma.sync kernel."""
import pytest
import torch

from nano_train_b200.ops.attention import attention_reference

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("B,S,hq,hkv,causal", [(1, 512, 4, 4, True), (2, 300, 4, 2, True), (1, 256, 8, 2, False),
                                               (1, 1024, 8, 8, True), (1, 130, 2, 1, False)])
def test_flash_fwd_tc_matches_reference(B, S, hq, hkv, causal):
    from nano_train_b200.ops._ext import check_status, ext

    torch.manual_seed(B * 1000 + S + hq)
    dev = torch.device("cuda", 0)
    qkv = torch.randn(B, S, hq + 2 * hkv, 128, device=dev, dtype=torch.bfloat16)  # fused-projection layout
    q, k, v = qkv[:, :, :hq], qkv[:, :, hq:hq + hkv], qkv[:, :, hq + hkv:]
    scale = 128 ** -0.5
    o, lse = ext().flash_attn_fwd_tc(q, k, v, scale, causal)
    torch.cuda.synchronize()
    check_status(0)
    ref = attention_reference(q.float(), k.float(), v.float(), causal=causal, scale=scale)
    assert _rel(o, ref) < 1e-2
    o2, lse2 = ext().flash_attn_fwd(q, k, v, scale, causal)
    assert _rel(o, o2) < 1e-2
    torch.testing.assert_close(lse, lse2, rtol=1e-3, atol=1e-3)


def test_flash_fwd_tc_large_scores_rescale_path():
    """Scores with a growing max along the keys exercise the lazy O correction."""
    from nano_train_b200.ops._ext import check_status, ext

    torch.manual_seed(7)
    dev = torch.device("cuda", 0)
    S = 640
    q = torch.randn(1, S, 2, 128, device=dev) * 4
    k = torch.randn(1, S, 2, 128, device=dev) * torch.linspace(0.2, 3.0, S, device=dev)[None, :, None, None]
    v = torch.randn(1, S, 2, 128, device=dev)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    o, lse = ext().flash_attn_fwd_tc(q, k, v, 128 ** -0.5, True)
    torch.cuda.synchronize()
    check_status(0)
    ref = attention_reference(q.float(), k.float(), v.float(), causal=True, scale=128 ** -0.5)
    assert _rel(o, ref) < 1e-2


@pytest.mark.parametrize("B,S,hq,hkv,causal", [(1, 512, 4, 4, True), (2, 300, 4, 2, True), (1, 256, 8, 2, False),
                                               (1, 130, 2, 1, True), (1, 1024, 4, 1, True),
                                               (1, 1024, 2, 2, True), (1, 1024, 2, 2, False)])
@pytest.mark.parametrize("pipe", ["0", "1"])  # serial chain (default) / pipelined variant
def test_flash_bwd_tc_matches_reference(B, S, hq, hkv, causal, pipe, monkeypatch):
    from nano_train_b200.ops._ext import check_status, ext

    monkeypatch.setenv("NTB_ATTN_BWD_PIPE", pipe)
    torch.manual_seed(S + hq * 7 + int(causal))
    dev = torch.device("cuda", 0)
    qkv = torch.randn(B, S, hq + 2 * hkv, 128, device=dev, dtype=torch.bfloat16)
    q, k, v = qkv[:, :, :hq], qkv[:, :, hq:hq + hkv], qkv[:, :, hq + hkv:]
    scale = 128 ** -0.5
    o, lse = ext().flash_attn_fwd_tc(q, k, v, scale, causal)
    do = torch.randn_like(o)
    dq, dk, dv = ext().flash_attn_bwd(do, q, k, v, o, lse, scale, causal)
    torch.cuda.synchronize()
    check_status(0)
    qf, kf, vf = (t.float().detach().requires_grad_(True) for t in (q, k, v))
    attention_reference(qf, kf, vf, causal=causal, scale=scale).backward(do.float())
    for name, g, r in (("dq", dq, qf.grad), ("dk", dk, kf.grad), ("dv", dv, vf.grad)):
        assert _rel(g, r) < 2e-2, (name, _rel(g, r))
    monkeypatch.setenv("NTB_ATTN_BWD_LEGACY", "1")
    dq2, dk2, dv2 = ext().flash_attn_bwd(do, q, k, v, o, lse, scale, causal)
    torch.cuda.synchronize()
    for name, g, r in (("dq", dq, dq2), ("dk", dk, dk2), ("dv", dv, dv2)):
        assert _rel(g, r) < 2e-2, (name, "vs legacy", _rel(g, r))


@pytest.mark.parametrize("dqk,dv", [(192, 128), (64, 64)])
@pytest.mark.parametrize("B,S,hq,hkv,causal", [(1, 512, 4, 4, True), (2, 300, 4, 2, True), (1, 256, 2, 2, False),
                                               (1, 130, 2, 1, True), (1, 1024, 2, 2, True)])
def test_flash_tc_mla_and_hd64_match_reference(dqk, dv, B, S, hq, hkv, causal, monkeypatch):
    """MLA head dims (q/k 192 = [nope 128 | rope 64], v 128) and head dim 64 on the tcgen05 kernels,
    forward and backward, against fp32 PyTorch; q, k, v are strided views of one buffer."""
    from nano_train_b200.ops._ext import check_status, ext

    torch.manual_seed(dqk + S + hq * 3 + int(causal))
    dev = torch.device("cuda", 0)
    width = hq * dqk + hkv * (dqk + dv)
    buf = torch.randn(B, S, width, device=dev, dtype=torch.bfloat16)
    q = buf[..., : hq * dqk].view(B, S, hq, dqk)
    k = buf[..., hq * dqk: hq * dqk + hkv * dqk].view(B, S, hkv, dqk)
    v = buf[..., hq * dqk + hkv * dqk:].view(B, S, hkv, dv)
    scale = dqk ** -0.5
    o, lse = ext().flash_attn_fwd_tc(q, k, v, scale, causal)
    do = torch.randn_like(o)
    dq, dk, dvv = ext().flash_attn_bwd(do, q, k, v, o, lse, scale, causal)
    torch.cuda.synchronize()
    check_status(0)
    qf, kf, vf = (t.float().detach().requires_grad_(True) for t in (q, k, v))
    ref = attention_reference(qf, kf, vf, causal=causal, scale=scale)
    assert _rel(o, ref) < 1e-2
    ref.backward(do.float())
    for name, g, r in (("dq", dq, qf.grad), ("dk", dk, kf.grad), ("dv", dvv, vf.grad)):
        assert _rel(g, r) < 2e-2, (name, _rel(g, r))
    o2, lse2 = ext().flash_attn_fwd(q, k, v, scale, causal)  # the mma.sync kernel as a second opinion
    assert _rel(o, o2) < 1e-2
    torch.testing.assert_close(lse, lse2, rtol=1e-3, atol=1e-3)
    if dqk == 64:  # the pipelined backward variant exists for equal q/k and v widths
        monkeypatch.setenv("NTB_ATTN_BWD_PIPE", "1")
        dq3, dk3, dv3 = ext().flash_attn_bwd(do, q, k, v, o, lse, scale, causal)
        torch.cuda.synchronize()
        check_status(0)
        for name, g, r in (("dq", dq3, qf.grad), ("dk", dk3, kf.grad), ("dv", dv3, vf.grad)):
            assert _rel(g, r) < 2e-2, (name, "pipelined", _rel(g, r))


def test_mla_module_fast_path_matches_reference_path():
    """MultiHeadLatentAttention on the GPU: the fast path (q rotated in place, tcgen05 flash attention)
    against the module's own reference path (materialised causal scores, fp32 softmax), forward and
    backward (input and parameter gradients)."""
    import argparse

    from nano_train_b200.models.deepseek import DeepSeekModelConfig, MultiHeadLatentAttention
    from nano_train_b200.precision.mixed_precision import build_module_precision_resolver, resolve_precision_config

    dev = torch.device("cuda", 0)
    resolver = build_module_precision_resolver(resolve_precision_config(argparse.Namespace(), dev))
    cfg = DeepSeekModelConfig(precision_resolver=resolver, param_dtype=torch.bfloat16, param_device=dev,
                              vocab_size=97, hidden_size=256, num_hidden_layers=1, num_attention_heads=2,
                              num_key_value_heads=2, intermediate_size=256, q_lora_rank=64, kv_lora_rank=64,
                              qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128, moe_intermediate_size=64,
                              n_routed_experts=4, num_experts_per_tok=2, n_group=1, topk_group=1,
                              max_position_embeddings=512, first_k_dense_replace=1)
    torch.manual_seed(0)
    attn = MultiHeadLatentAttention(cfg, module_prefix="layers.0.attn")
    x = torch.randn(2, 256, 256, device=dev, dtype=torch.bfloat16)
    mask = torch.full((256, 256), float("-inf"), device=dev).triu(1)
    outs, grads = [], []
    for m in (None, mask):
        attn.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_(True)
        y = attn(xi, m)
        g = torch.Generator(device=dev).manual_seed(1)
        (y.float() * torch.randn(y.shape, device=dev, generator=g)).sum().backward()
        outs.append((y.detach(), xi.grad.detach()))
        grads.append({n: (p.main_grad if getattr(p, "main_grad", None) is not None else p.grad).detach().clone()
                      for n, p in attn.named_parameters()})
    assert _rel(outs[0][0], outs[1][0]) < 2e-2, _rel(outs[0][0], outs[1][0])
    assert _rel(outs[0][1], outs[1][1]) < 3e-2, _rel(outs[0][1], outs[1][1])
    for n in grads[0]:
        assert _rel(grads[0][n], grads[1][n]) < 3e-2, (n, _rel(grads[0][n], grads[1][n]))
