"""Optimizers and learning-rate schedules.

* :class:`~placemoe_b200.ops.optim.FusedAdamW` — multi-tensor AdamW on the sm_100a kernel.
* :class:`Muon` — Newton-Schulz orthogonalised momentum for hidden matrices
  (attention projections, expert slots as batched matrices).
* :class:`MultiOptimizer` — several optimizers behind one ``step`` / ``param_groups``.
* :func:`build_optimizer`, :func:`build_lr_scheduler`.

Reference parity: veomni/optim/optimizer.py:41-623 (build_optimizer, MultiOptimizer,
EP-aware parameter groups), veomni/optim/muon.py, veomni/optim/lr_scheduler.py.
"""

from .lr_scheduler import LRSchedule, build_lr_scheduler
from .muon import Muon, zeropower_newton_schulz
from .optimizer import MultiOptimizer, build_optimizer, state_tensors

__all__ = ["LRSchedule", "build_lr_scheduler", "Muon", "zeropower_newton_schulz", "MultiOptimizer",
           "build_optimizer", "state_tensors"]
