"""Vision-language MoE training entry point (text decoder + vision tower stub for synthetic runs).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 tasks/train_vlm.py configs/qwen3_vl_moe.yaml
"""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from placemoe_b200.arguments import parse_args  # noqa: E402
from placemoe_b200.trainer.vlm_trainer import VLMTrainer  # noqa: E402

if __name__ == "__main__":
    args = parse_args()
    trainer = VLMTrainer(args)
    trainer.train()
