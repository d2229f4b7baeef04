"""Optimizer construction and the multi-optimizer wrapper.

``build_optimizer(model, "adamw")`` gives the fused AdamW over every parameter.
``build_optimizer(model, "muon")`` gives a :class:`MultiOptimizer` of Muon for
hidden matrices (attention projections and expert slots) and fused AdamW for
embeddings, the LM head, norms and router weights, which is the usual split.

:class:`MultiOptimizer` presents several optimizers as one: ``step``,
``param_groups`` (all groups, so the trainer sets the learning rate in one
loop), ``state`` (merged), ``grad_scale`` (forwarded) and ``_state(p)``
(routed to the optimizer owning ``p``).  ``state_tensors(opt, p)`` lists the
per-parameter state tensors (AdamW moments or the Muon momentum) for the
checkpointer and the expert-migration path, which move them slot by slot.

Reference parity: veomni/optim/optimizer.py:41-623 (build_optimizer,
MultiOptimizer over the EP / non-EP parameter sets, Muon option).
"""

from __future__ import annotations

import torch

from ..ops.optim import FusedAdamW
from .muon import Muon

OPTIMIZERS = ("adamw", "muon")


def state_tensors(opt, p) -> list[tuple[str, torch.Tensor]]:
    """(name, tensor) of the optimizer state of ``p`` with the parameter's shape, in a fixed order."""
    st = opt._state(p)
    return [(k, v) for k, v in sorted(st.items()) if torch.is_tensor(v) and v.shape == p.shape]


class MultiOptimizer:
    def __init__(self, optimizers: dict):
        self.optimizers = dict(optimizers)
        self._owner: dict[int, object] = {}
        for opt in self.optimizers.values():
            for g in opt.param_groups:
                for p in g["params"]:
                    if id(p) in self._owner:
                        raise ValueError("a parameter belongs to two optimizers")
                    self._owner[id(p)] = opt
        self._grad_scale = None

    @property
    def param_groups(self):
        return [g for opt in self.optimizers.values() for g in opt.param_groups]

    @property
    def state(self):
        merged = {}
        for opt in self.optimizers.values():
            merged.update(opt.state)
        return merged

    @property
    def grad_scale(self):
        return self._grad_scale

    @grad_scale.setter
    def grad_scale(self, value):
        self._grad_scale = value
        for opt in self.optimizers.values():
            opt.grad_scale = value

    def _state(self, p):
        return self._owner[id(p)]._state(p)

    def reset_tables(self) -> None:
        for opt in self.optimizers.values():
            opt.reset_tables()

    def sync_params(self) -> None:
        """Make every ``param.data`` current (sharded optimizers gather their masters; collective)."""
        for opt in self.optimizers.values():
            if hasattr(opt, "sync_params"):
                opt.sync_params()

    def reload_from_params(self) -> None:
        """Push loaded ``param.data`` / state into optimizers that keep their own copies."""
        for opt in self.optimizers.values():
            if hasattr(opt, "reload_from_params"):
                opt.reload_from_params()

    @property
    def defaults(self):
        return self._fallback().defaults

    def _fallback(self):
        """The optimizer that takes parameters added later (AdamW when present)."""
        return self.optimizers.get("adamw") or next(iter(self.optimizers.values()))

    def add_param_group(self, group: dict) -> None:
        opt = self._fallback()
        opt.add_param_group(group)
        for p in opt.param_groups[-1]["params"]:
            self._owner[id(p)] = opt

    def step(self, closure=None):
        for opt in self.optimizers.values():
            opt.step()

    def zero_grad(self, set_to_none: bool = True):
        for opt in self.optimizers.values():
            opt.zero_grad(set_to_none=set_to_none)

    def state_dict(self):
        return {name: opt.state_dict() for name, opt in self.optimizers.items()}

    def load_state_dict(self, sd):
        for name, opt in self.optimizers.items():
            opt.load_state_dict(sd[name])


def _is_muon_param(name: str, p: torch.Tensor) -> bool:
    if p.dim() < 2:
        return False
    leaf = name.rsplit(".", 1)[-1]
    return leaf in ("qkv_proj", "o_proj", "gate_up_proj", "down_proj", "gate_proj", "up_proj")


def build_optimizer(model, name: str = "adamw", lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                    weight_decay: float = 0.0, muon_lr: float = 0.02, muon_momentum: float = 0.95,
                    muon_adjust_lr: str = "spectral"):
    if name not in OPTIMIZERS:
        raise ValueError(f"unknown optimizer {name!r}; expected one of {OPTIMIZERS}")
    if name == "adamw":
        return FusedAdamW(model.parameters(), lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
    mats, rest = [], []
    for n, p in model.named_parameters():
        (mats if _is_muon_param(n, p) else rest).append(p)
    opts = {"muon": Muon(mats, lr=muon_lr, momentum=muon_momentum, weight_decay=weight_decay,
                         adjust_lr=muon_adjust_lr)}
    if rest:
        opts["adamw"] = FusedAdamW(rest, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
    return MultiOptimizer(opts)
