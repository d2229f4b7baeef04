"""Learning-rate schedules: linear warmup followed by constant, linear or cosine decay.

``LRSchedule(kind, base_lr, warmup_steps, total_steps, min_lr_ratio)(step)``
returns the learning rate of optimizer step ``step`` (0-based).  Warmup ramps
linearly from ``base_lr / warmup_steps`` to ``base_lr``; decay runs over the
remaining steps down to ``min_lr_ratio * base_lr``.  ``as_lambda`` gives the
multiplier form for ``torch.optim.lr_scheduler.LambdaLR``.

Reference parity: veomni/optim/lr_scheduler.py (build_lr_scheduler with
constant / linear / cosine decay, warmup ratio, minimum learning rate).
"""

from __future__ import annotations

import dataclasses
import math

KINDS = ("constant", "linear", "cosine")


@dataclasses.dataclass(frozen=True)
class LRSchedule:
    kind: str = "cosine"
    base_lr: float = 3e-4
    warmup_steps: int = 0
    total_steps: int = 100
    min_lr_ratio: float = 0.0

    def __post_init__(self):
        if self.kind not in KINDS:
            raise ValueError(f"unknown lr schedule {self.kind!r}; expected one of {KINDS}")
        if not 0.0 <= self.min_lr_ratio <= 1.0:
            raise ValueError("min_lr_ratio must be in [0, 1]")

    def multiplier(self, step: int) -> float:
        if self.warmup_steps and step < self.warmup_steps:
            return (step + 1) / self.warmup_steps
        if self.kind == "constant":
            return 1.0
        span = max(1, self.total_steps - self.warmup_steps)
        prog = min(1.0, max(0.0, (step - self.warmup_steps) / span))
        lo = self.min_lr_ratio
        if self.kind == "linear":
            return lo + (1.0 - lo) * (1.0 - prog)
        return lo + (1.0 - lo) * 0.5 * (1.0 + math.cos(math.pi * prog))

    def __call__(self, step: int) -> float:
        return self.base_lr * self.multiplier(step)

    def as_lambda(self):
        return self.multiplier


def build_lr_scheduler(kind: str = "cosine", base_lr: float = 3e-4, warmup_steps: int = 0, total_steps: int = 100,
                       min_lr_ratio: float = 0.0, warmup_ratio: float | None = None) -> LRSchedule:
    if warmup_ratio is not None:
        warmup_steps = int(warmup_ratio * total_steps)
    return LRSchedule(kind, base_lr, warmup_steps, total_steps, min_lr_ratio)
