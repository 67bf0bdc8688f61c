"""4-D parallel DeepSeek training: TP x PP x EP x DP with ZeRO-1/2 and 1F1B.

    python examples/train_4d.py --tensor-model-parallel-size 1 --pipeline-model-parallel-size 1 \
        --expert-model-parallel-size 1
    python examples/launch.py --world-size 4 --backend gloo --script examples/train_4d.py --script-args \
        --tensor-model-parallel-size 1 --pipeline-model-parallel-size 2 --expert-model-parallel-size 2 ...
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/train_4d.py ...
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.runtime.train4d import (DummyTokenDataset, build_tiny_deepseek_config,  # noqa: E402,F401
                                             build_train_4d_components, create_data_loader, gather_moe_metrics,
                                             main, parse_args)

if __name__ == "__main__":
    main()
