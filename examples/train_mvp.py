"""Single-process language-model training with the Trainer (MVP path).

    python examples/train_mvp.py [--data path/to/text.txt] [--max_steps 100] [--seed 42]

Character-level TextDataset when ``--data`` points at a text file, seeded
synthetic tokens otherwise. GPT-2-style TransformerModel (the reference's
default block) under the shared precision flags (bf16 on CUDA and fp32 on CPU by default; --fp8 / --fp4
with their backends, loss scaling where the mode needs it), fused AdamW, cosine LR,
TensorBoard/JSONL metrics and checkpoints under ``--output_dir``.
(reference: examples/train_mvp.py)
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.config import Config, ModelConfig, TrainingConfig  # noqa: E402
from nano_train_b200.dataset import SyntheticTokenDataset, TextDataset, create_dataloader  # noqa: E402
from nano_train_b200.logging import setup_logging  # noqa: E402
from nano_train_b200.models.transformer import TransformerModel  # noqa: E402
from nano_train_b200.precision.mixed_precision import (MixedPrecisionController,  # noqa: E402
                                                       build_module_precision_resolver, dtype_alias_to_torch,
                                                       finalize_module_precision_resolver)
from nano_train_b200.precision.precision_args import (add_mixed_precision_args,  # noqa: E402
                                                      normalize_and_resolve_precision)
from nano_train_b200.trainer import Trainer  # noqa: E402


def main():
    ap = argparse.ArgumentParser(description="MVP training")
    ap.add_argument("--data", default=None)
    ap.add_argument("--max_steps", type=int, default=100)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--batch_size", type=int, default=8)
    ap.add_argument("--seq_len", type=int, default=256)
    ap.add_argument("--hidden_size", type=int, default=256)
    ap.add_argument("--num_layers", type=int, default=4)
    ap.add_argument("--num_heads", type=int, default=4)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--output_dir", default="outputs/nano_train_mvp")
    add_mixed_precision_args(ap)  # --bf16 / --fp16 / --fp8 / --fp4, backends, recipe, per-module rules
    a = ap.parse_args()
    setup_logging()
    torch.manual_seed(a.seed)
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    pc = normalize_and_resolve_precision(a, dev)
    resolver = build_module_precision_resolver(pc)
    if a.data and os.path.exists(a.data):
        ds = TextDataset(a.data, max_seq_length=a.seq_len + 1)
        vocab = ds.vocab_size
    else:
        vocab = 256
        ds = SyntheticTokenDataset(512, a.seq_len, vocab, seed=a.seed)
    n_val = max(1, len(ds) // 10)
    train_ds, val_ds = torch.utils.data.random_split(ds, [len(ds) - n_val, n_val],
                                                     generator=torch.Generator().manual_seed(a.seed))
    mcfg = ModelConfig(param_dtype=dtype_alias_to_torch(pc.params_dtype), param_device=dev,
                       precision_resolver=resolver, hidden_size=a.hidden_size,
                       num_layers=a.num_layers, num_attention_heads=a.num_heads, intermediate_size=4 * a.hidden_size,
                       vocab_size=vocab, max_position_embeddings=max(1024, a.seq_len), dropout=0.0)
    cfg = Config(model=mcfg, training=TrainingConfig(batch_size=a.batch_size, micro_batch_size=a.batch_size,
                                                     learning_rate=a.lr, max_steps=a.max_steps,
                                                     warmup_steps=max(1, a.max_steps // 10), log_steps=10,
                                                     eval_steps=max(10, a.max_steps // 4), save_steps=0),
                 output_dir=a.output_dir, log_dir=os.path.join(a.output_dir, "logs"), seed=a.seed)
    model = TransformerModel(mcfg)
    finalize_module_precision_resolver(resolver)
    trainer = Trainer(model, cfg, create_dataloader(train_ds, a.batch_size), dev,
                      val_loader=create_dataloader(val_ds, a.batch_size, shuffle=False),
                      precision_controller=MixedPrecisionController(pc, device=dev))
    print(trainer.train())


if __name__ == "__main__":
    main()
