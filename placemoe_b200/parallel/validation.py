"""MoE dispatch validation records (debug).

``check_dispatch`` verifies the routing invariants of one layer call: every
assignment maps to a slot that holds its logical expert, and the dispatch
plan's per-slot counts add up to the number of assignments.  With
``PM_MOE_VALIDATION_DIR`` set, ``ValidationRecorder`` dumps the routes, the
destination ranks and the plan counts of each checked call (one ``.pt`` per
layer and step) for offline comparison between runs or transports.

Reference parity: veomni/distributed/moe/validation.py:23-130.
"""

from __future__ import annotations

import os

import numpy as np
import torch

ENV_DIR = "PM_MOE_VALIDATION_DIR"


def check_dispatch(idx: torch.Tensor, placement, counts: torch.Tensor | None = None) -> list[str]:
    """Return a list of violated invariants (empty when the call is consistent)."""
    errors = []
    idx_np = idx.detach().cpu().numpy().astype(np.int64)
    mapping = np.asarray(placement.lut_global())
    layout = np.asarray(placement.slot_to_logical)
    slots = mapping[idx_np]
    bad = layout[slots] != idx_np
    if bad.any():
        errors.append(f"{int(bad.sum())} assignments map to a slot without their expert")
    if counts is not None:
        total = int(counts.detach().sum().item())
        if total != idx_np.size:
            errors.append(f"plan counts sum to {total}, expected {idx_np.size}")
    return errors


class ValidationRecorder:
    def __init__(self, root: str | None = None):
        self.root = root if root is not None else os.environ.get(ENV_DIR, "")

    @property
    def enabled(self) -> bool:
        return bool(self.root)

    def record(self, step: int, layer: int, idx: torch.Tensor, placement, counts=None) -> list[str]:
        errs = check_dispatch(idx, placement, counts)
        if self.root:
            os.makedirs(self.root, exist_ok=True)
            dest = np.asarray(placement.lut_global())[idx.cpu().numpy()] // placement.slots_per_rank
            torch.save({"step": step, "layer": layer, "idx": idx.detach().cpu(),
                        "dest": torch.from_numpy(np.ascontiguousarray(dest)),
                        "counts": None if counts is None else counts.detach().cpu(), "errors": errs},
                       os.path.join(self.root, f"step{step:06d}_layer{layer:02d}.pt"))
        return errs
