"""Text MoE training entry point.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 tasks/train_text.py configs/olmoe_1b_7b.yaml \
        [--train.lr=1e-4 ...]

With ``VEOMNI_PLACEMOE_CONFIG`` set, the PlaceMoE initial artifact is loaded at
startup and hot updates follow the configured intervals.
"""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from placemoe_b200.arguments import parse_args  # noqa: E402
from placemoe_b200.trainer.text_trainer import TextTrainer  # noqa: E402

if __name__ == "__main__":
    args = parse_args()
    trainer = TextTrainer(args)
    trainer.train()
