"""Inspect or train a DeepSeek-V3-like model (reference: examples/deepseek.py).

    python examples/deepseek.py                       # V3 preset on the meta device -> model report
    python examples/deepseek.py --model-preset tiny --no-meta-init --steps 20

The ``deepseek_v3`` preset builds the official-scale configuration (7168
hidden, 61 layers, MLA, 256 routed experts top-8) on the ``meta`` device (no
parameter memory) and writes an analytic model report. The ``tiny`` preset
with ``--no-meta-init`` materialises a small model and trains it on
synthetic tokens.
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.config import _NoOpPrecisionResolver  # noqa: E402
from nano_train_b200.models.deepseek import DeepSeekModel, DeepSeekModelConfig  # noqa: E402
from nano_train_b200.utils.model_info import ParallelismAssumptions, dump_model_info  # noqa: E402


def build(preset: str, device) -> DeepSeekModel:
    common = dict(param_dtype=torch.bfloat16, param_device=device, precision_resolver=_NoOpPrecisionResolver())
    if preset == "deepseek_v3":
        cfg = DeepSeekModelConfig(**common)  # defaults are the V3 shapes
    else:
        cfg = DeepSeekModelConfig(**common, vocab_size=1024, hidden_size=256, num_hidden_layers=4,
                                  num_attention_heads=4, num_key_value_heads=4, intermediate_size=512,
                                  q_lora_rank=128, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=32,
                                  v_head_dim=32, moe_intermediate_size=128, n_routed_experts=8,
                                  num_experts_per_tok=2, n_group=2, topk_group=1, first_k_dense_replace=1,
                                  max_position_embeddings=1024)
    return DeepSeekModel(cfg)


def main():
    ap = argparse.ArgumentParser(description="Train or inspect a DeepSeek-V3-like model.")
    ap.set_defaults(meta_init=True)
    ap.add_argument("--model-preset", choices=["deepseek_v3", "tiny"], default="deepseek_v3")
    ap.add_argument("--meta-init", dest="meta_init", action="store_true")
    ap.add_argument("--no-meta-init", dest="meta_init", action="store_false")
    ap.add_argument("--report", default="outputs/model_reports/deepseek_model_report.md")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--seq_len", type=int, default=128)
    a = ap.parse_args()
    dev = torch.device("meta") if a.meta_init else torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = build(a.model_preset, dev)
    n = sum(p.numel() for p in model.parameters())
    print(f"{a.model_preset}: {n / 1e9:.3f} B parameters ({n * 2 / 2**30:.1f} GiB in bf16)")
    info = dump_model_info(model, a.report, batch=8, seq_len=4096, parallel=ParallelismAssumptions(ep=64))
    train = next(m for m in info.modes if m.mode == "train")
    for name, r in train.per_target.items():
        print(f"  train step estimate on {name}: {r['time_ms']:.1f} ms ({r['bound']}-bound)")
    print(f"report: {a.report}")
    if a.meta_init:
        return
    if dev.type == "cpu":
        model = model.float()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(0)
    V = model.config.vocab_size
    for step in range(a.steps):
        ids = torch.randint(0, V, (2, a.seq_len + 1), generator=g).to(dev)
        logits = model(ids[:, :-1])
        loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, V), ids[:, 1:].reshape(-1))
        opt.zero_grad()
        loss.backward()
        opt.step()
        if step % 5 == 0:
            print(f"step {step} loss {float(loss.detach()):.4f}")


if __name__ == "__main__":
    main()
