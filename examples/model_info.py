"""Analytic model report for the built-in model shapes (reference: examples/model_info.py).

    python examples/model_info.py --model llama3_8b --tp 8 --out outputs/model_reports/llama3_8b.md

Builds the model on the ``meta`` device and writes parameter counts, FLOPs,
bytes and roofline time estimates (H200/B200 spec and measured B200 peaks).
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.models.transformer import TransformerModel, llama3_8b_config  # noqa: E402
from nano_train_b200.utils.model_info import ParallelismAssumptions, decode_sweep, dump_model_info  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["llama3_8b", "gpt2_125m"], default="llama3_8b")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--seq_len", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    meta = torch.device("meta")
    if a.model == "llama3_8b":
        model = TransformerModel(llama3_8b_config(param_device=meta, sequence_parallel=False))
    else:
        from nano_train_b200.config import ModelConfig, _NoOpPrecisionResolver

        model = TransformerModel(ModelConfig(param_dtype=torch.bfloat16, param_device=meta,
                                             precision_resolver=_NoOpPrecisionResolver()))
    out = a.out or f"outputs/model_reports/{a.model}.md"
    info = dump_model_info(model, out, batch=a.batch, seq_len=a.seq_len, parallel=ParallelismAssumptions(tp=a.tp))
    print(f"{a.model}: {info.total_params / 1e9:.3f} B params -> {out}")
    for m in info.modes:
        best = min(m.per_target.items(), key=lambda kv: kv[1]["time_ms"])
        print(f"  {m.mode:8s} {m.flops / 1e12:10.1f} TFLOP  best {best[0]}: {best[1]['time_ms']:.2f} ms "
              f"({best[1]['bound']})")
    for row in decode_sweep(model, parallel=ParallelismAssumptions(tp=a.tp)):
        print("  decode batch", row["batch"], {k: v for k, v in row["bound"].items()})


if __name__ == "__main__":
    main()
