"""Cross-entropy walkthrough (reference: examples/loss_demo.py).

Shows log-softmax + NLL by hand against CrossEntropyLoss, the ignore_index
mask, the reductions, and (on CUDA) the fused kernel against the fp32 math.
"""
import os
import sys

import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.losses import CrossEntropyLoss  # noqa: E402

if __name__ == "__main__":
    torch.manual_seed(0)
    logits = torch.randn(2, 5, 7)
    targets = torch.randint(0, 7, (2, 5))
    targets[0, 0] = -100
    logp = logits.log_softmax(-1)
    manual = -logp.gather(-1, targets.clamp_min(0).unsqueeze(-1)).squeeze(-1)
    mask = targets != -100
    print("manual mean  :", float(manual[mask].mean()))
    print("module mean  :", float(CrossEntropyLoss()(logits, targets)))
    print("module sum   :", float(CrossEntropyLoss(reduction="sum")(logits, targets)))
    print("per-token    :", CrossEntropyLoss(reduction="none")(logits, targets))
    if torch.cuda.is_available():
        lg = torch.randn(4096, 32000, device="cuda", dtype=torch.bfloat16)
        tg = torch.randint(0, 32000, (4096,), device="cuda")
        fused = float(CrossEntropyLoss()(lg, tg))
        ref = float(F.cross_entropy(lg.float(), tg))
        print(f"fused kernel {fused:.6f} vs fp32 {ref:.6f}")
