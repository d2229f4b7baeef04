"""Fused multi-tensor AdamW on the sm_100a kernel (``csrc/kernels/optim.cu``).

Parameters are fp32 masters.  A gradient is read from ``param.main_grad``
(fp32, written by the expert weight-gradient GEMMs) when present, else from
``param.grad`` (fp32 or bf16).  A parameter may carry ``param.bf16_shadow``, a
bf16 compute copy that the kernel rewrites in the same pass.  CPU parameters
use ``torch.optim.AdamW`` semantics implemented in PyTorch.

Reference parity: build_optimizer / fused AdamW in veomni/optim/optimizer.py:261-330.
"""

from __future__ import annotations

import torch

from ._ext import kernels


def param_grad(p: torch.Tensor):
    g = getattr(p, "main_grad", None)
    if g is not None:
        return g
    g = p.grad
    if g is not None and hasattr(g, "to_local"):
        g = g.to_local()
    return g


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if hasattr(t, "to_local") else t


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self._tables: dict = {}
        self.grad_scale: torch.Tensor | None = None  # optional device scalar (clip coefficient)

    def reset_tables(self) -> None:
        """Drop the cached device tables (parameters or states were re-bound)."""
        self._tables.clear()

    def _state(self, p):
        st = self.state[p]
        if not st:
            lp = _local(p.data)
            st["step"] = 0
            st["exp_avg"] = torch.zeros_like(lp, dtype=torch.float32)
            st["exp_avg_sq"] = torch.zeros_like(lp, dtype=torch.float32)
        return st

    @torch.no_grad()
    def step(self, closure=None):
        for gi, group in enumerate(self.param_groups):
            cuda_items, cpu_items = [], []
            for p in group["params"]:
                g = param_grad(p)
                if g is None:
                    continue
                st = self._state(p)
                st["step"] += 1
                (cuda_items if _local(p.data).is_cuda else cpu_items).append((p, g, st))
            b1, b2 = group["betas"]
            if cuda_items:
                key = (gi, tuple((_local(p.data).data_ptr(), g.data_ptr(), g.dtype) for p, g, _ in cuda_items))
                tab = self._tables.get(gi)
                if tab is None or tab[0] != key:
                    params = [_local(p.data) for p, _, _ in cuda_items]
                    grads = [g.contiguous() if g.is_contiguous() else g.contiguous() for _, g, _ in cuda_items]
                    shadows = [getattr(p, "bf16_shadow", None) for p, _, _ in cuda_items]
                    table, meta = kernels().adamw_build_table(
                        params, grads, [st["exp_avg"] for _, _, st in cuda_items],
                        [st["exp_avg_sq"] for _, _, st in cuda_items], shadows,
                    )
                    tab = (key, table, meta)
                    self._tables[gi] = tab
                step = cuda_items[0][2]["step"]
                kernels().adamw_step(tab[1], tab[2], group["lr"], b1, b2, group["eps"], group["weight_decay"], step,
                                     self.grad_scale)
            for p, g, st in cpu_items:
                lp = _local(p.data)
                gg = g.float() * (float(self.grad_scale) if self.grad_scale is not None else 1.0)
                st["exp_avg"].mul_(b1).add_(gg, alpha=1 - b1)
                st["exp_avg_sq"].mul_(b2).addcmul_(gg, gg, value=1 - b2)
                bc1 = 1 - b1 ** st["step"]
                bc2 = 1 - b2 ** st["step"]
                lp.mul_(1 - group["lr"] * group["weight_decay"])
                denom = (st["exp_avg_sq"] / bc2).sqrt_().add_(group["eps"])
                lp.addcdiv_(st["exp_avg"], denom, value=-group["lr"] / bc1)
                shadow = getattr(p, "bf16_shadow", None)
                if shadow is not None:
                    shadow.copy_(lp)
        return None
