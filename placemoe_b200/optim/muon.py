"""Muon: momentum orthogonalised by a Newton-Schulz iteration, for hidden weight matrices.

For a matrix parameter W with gradient G the step is

    M <- mu M + G                       (momentum buffer, fp32)
    U <- G + mu M  (Nesterov)  or  M
    O <- NS5(U)                         (approximately the orthogonal factor of U)
    W <- W (1 - lr wd) - lr * s * O,    s = max(1, rows / cols) ** 0.5   ("spectral")
                                        s = 0.2 * max(rows, cols) ** 0.5  ("match_rms", AdamW-like RMS)

NS5 is the quintic Newton-Schulz iteration of the published Muon optimizer
(K. Jordan et al., 2024, "Muon: an optimizer for hidden layers"), with its
coefficients (3.4445, -4.7750, 2.0315), run on U / ||U||_F in bf16 on CUDA.
Parameters with three dimensions (expert slots [E, out, in]) are
orthogonalised per slot as a batch, so each expert is its own matrix; slots
are local to a rank under expert parallelism, so no collective is needed.

Gradients come from ``main_grad`` when present (fp32 accumulation buffers)
and are scaled by the optional device scalar ``grad_scale`` (clip coefficient
divided by the micro-batch count); ``bf16_shadow`` compute copies are
rewritten after the update.

Reference parity: veomni/optim/muon.py (Muon with Newton-Schulz, used for
2-D hidden weights, AdamW for the rest).
"""

from __future__ import annotations

import torch

from ..ops.optim import param_grad

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _ns_matrix_cuda(x: torch.Tensor, steps: int) -> torch.Tensor:
    """Newton-Schulz iterations of one wide bf16 matrix [m, n] (m <= n) on the tcgen05 GEMMs."""
    from ..ops.gemm import gemm_nn, gemm_nt

    a, b, c = NS_COEFFS
    x = x.contiguous()
    for _ in range(steps):
        s = gemm_nt(x, x)  # x x^T   [m, m]
        y = torch.add(s, gemm_nn(s, s), alpha=c / b).mul_(b)  # b*s + c*s^2
        x = torch.add(gemm_nn(y, x), x, alpha=a)  # a*x + y x
    return x


def zeropower_newton_schulz(g: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Approximate orthogonal factor of the last two dims of ``g`` (batched over leading dims).

    CUDA runs the three products of every iteration on the tcgen05 GEMM kernels (bf16 operands, fp32
    accumulation), one matrix at a time; the kernels need both dims to be multiples of 8, other shapes
    (tiny test matrices) are rejected.  CPU runs the same iteration in fp32 with torch matmuls.
    """
    if g.dim() < 2:
        raise ValueError("Newton-Schulz needs a matrix")
    a, b, c = NS_COEFFS
    x = g.to(torch.bfloat16) if g.is_cuda else g.float()
    tall = x.size(-2) > x.size(-1)
    if tall:
        x = x.mT
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + eps)
    if x.is_cuda:
        if x.size(-2) % 8 or x.size(-1) % 8:
            raise ValueError(f"Muon on CUDA needs matrix dims that are multiples of 8, got {tuple(x.shape[-2:])}")
        lead = x.shape[:-2]
        flat = x.reshape(-1, x.size(-2), x.size(-1))
        x = torch.stack([_ns_matrix_cuda(m, steps) for m in flat.unbind(0)]).reshape(*lead, *x.shape[-2:])
    else:
        for _ in range(steps):
            s = x @ x.mT
            y = b * s + c * (s @ s)
            x = a * x + y @ x
    if tall:
        x = x.mT
    return x


class Muon(torch.optim.Optimizer):
    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True, ns_steps: int = 5,
                 weight_decay: float = 0.0, adjust_lr: str = "spectral"):
        if adjust_lr not in ("spectral", "match_rms"):
            raise ValueError("adjust_lr must be 'spectral' or 'match_rms'")
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                                      weight_decay=weight_decay, adjust_lr=adjust_lr))
        for group in self.param_groups:
            for p in group["params"]:
                if p.dim() < 2:
                    raise ValueError("Muon takes matrices (or batches of matrices) only")
        self.grad_scale: torch.Tensor | None = None

    def _state(self, p):
        st = self.state[p]
        if not st:
            st["step"] = 0
            st["momentum_buffer"] = torch.zeros_like(p.data, dtype=torch.float32)
        return st

    def reset_tables(self) -> None:
        """No cached tables (present for the optimizer protocol of the trainer)."""

    @staticmethod
    def _scale(p, kind: str) -> float:
        rows, cols = p.shape[-2], p.shape[-1]
        if kind == "spectral":
            return max(1.0, rows / cols) ** 0.5
        return 0.2 * max(rows, cols) ** 0.5

    @torch.no_grad()
    def step(self, closure=None):
        for group in self.param_groups:
            mu, lr = group["momentum"], group["lr"]
            for p in group["params"]:
                g = param_grad(p)
                if g is None:
                    continue
                st = self._state(p)
                st["step"] += 1
                g = g.float()
                if self.grad_scale is not None:
                    g = g * self.grad_scale.to(g.device)
                buf = st["momentum_buffer"]
                buf.mul_(mu).add_(g)
                u = g.add(buf, alpha=mu) if group["nesterov"] else buf
                o = zeropower_newton_schulz(u, group["ns_steps"]).to(p.dtype)
                if group["weight_decay"]:
                    p.data.mul_(1.0 - lr * group["weight_decay"])
                p.data.add_(o, alpha=-lr * self._scale(p, group["adjust_lr"]))
                shadow = getattr(p, "bf16_shadow", None)
                if shadow is not None:
                    shadow.copy_(p.data)
        return None
