"""Mixed-precision parameter handling shared by every layer on the CUDA path.

Each trainable parameter is an fp32 master.  Kernels read a bf16 compute copy
(``param.bf16_shadow``) and accumulate fp32 gradients straight into
``param.main_grad`` (the weight-gradient GEMMs use an fp32 accumulate
epilogue), so no per-micro-batch cast or gradient-add pass exists.  The fused
AdamW kernel rewrites the bf16 copy when it updates the master.  A master
changed by other means (``load_state_dict``, a migration) bumps the tensor's
version counter, which triggers a refresh of the copy on next use.

CPU tensors keep plain PyTorch autograd (``.grad``).
"""

from __future__ import annotations

import torch

from ._ext import kernels
from .gemm import _mat, gemm_nn, gemm_nt, gemm_tn


def main_grad(p: torch.Tensor) -> torch.Tensor:
    g = getattr(p, "main_grad", None)
    if g is None or g.shape != p.shape or g.device != p.device:
        g = torch.zeros(p.shape, device=p.device, dtype=torch.float32)
        p.main_grad = g
    return g


def shadow(p: torch.Tensor) -> torch.Tensor:
    """bf16 compute copy of an fp32 master parameter (created / refreshed on demand)."""
    sh = getattr(p, "bf16_shadow", None)
    ver = p._version
    if sh is None or sh.shape != p.shape or sh.device != p.device:
        sh = p.detach().to(torch.bfloat16)
        p.bf16_shadow = sh
        p._shadow_version = ver
    elif getattr(p, "_shadow_version", None) != ver:
        sh.copy_(p.detach())
        p._shadow_version = ver
    return sh


def mark_shadow_fresh(p: torch.Tensor) -> None:
    """Called after a kernel updated both the master and its copy in place."""
    p._shadow_version = p._version


def zero_main_grads(params) -> None:
    for p in params:
        g = getattr(p, "main_grad", None)
        if g is not None:
            g.zero_()


class _LinearMP(torch.autograd.Function):
    """y = x @ w^T with w's bf16 copy; dW accumulates into master.main_grad (fp32)."""

    @staticmethod
    def forward(ctx, x, w16, master, fp32_out):
        x2 = _mat(x)
        ctx.save_for_backward(x2, w16)
        ctx.master = master
        ctx.xshape = x.shape
        y = gemm_nt(x2, w16, out_dtype=torch.float32 if fp32_out else torch.bfloat16)
        return y.view(*x.shape[:-1], w16.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w16 = ctx.saved_tensors
        dy2 = _mat(dy.to(torch.bfloat16))
        dx = gemm_nn(dy2, w16).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        if ctx.master.requires_grad:
            gemm_tn(dy2, x2, out=main_grad(ctx.master), accumulate=True)
        return dx, None, None, None


def linear(x: torch.Tensor, w: torch.Tensor, fp32_out: bool = False) -> torch.Tensor:
    """x @ w^T.  CUDA: tcgen05 GEMMs with fp32 master-gradient accumulation.  CPU: F.linear."""
    if not x.is_cuda:
        return torch.nn.functional.linear(x, w)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    return _LinearMP.apply(x, shadow(w), w, fp32_out)


class _RMSNormMP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, master, eps):
        x2 = x.contiguous()
        y, rstd = kernels().rmsnorm_fwd(x2, master.detach(), eps)
        ctx.save_for_backward(x2, rstd)
        ctx.master = master
        return y

    @staticmethod
    def backward(ctx, dy):
        x, rstd = ctx.saved_tensors
        m = ctx.master
        dw = main_grad(m) if m.requires_grad else torch.zeros(m.shape, device=m.device, dtype=torch.float32)
        dx = kernels().rmsnorm_bwd(dy.contiguous().to(torch.bfloat16), x, m.detach(), rstd, dw)
        return dx, None, None


class _AddRMSNormMP(torch.autograd.Function):
    """(h, y) = (x + res, rmsnorm(x + res)) in one pass; the backward folds the gradient reaching h
    through the residual path into the norm's backward (dx = dres = norm backward + dh)."""

    @staticmethod
    def forward(ctx, x, res, master, eps):
        h, y, rstd = kernels().add_rmsnorm_fwd(x.contiguous(), res.contiguous(), master.detach(), eps)
        ctx.save_for_backward(h, rstd)
        ctx.master = master
        return h, y

    @staticmethod
    def backward(ctx, dh, dy):
        h, rstd = ctx.saved_tensors
        m = ctx.master
        if dy is None:
            return dh, dh, None, None
        dw = main_grad(m) if m.requires_grad else torch.zeros(m.shape, device=m.device, dtype=torch.float32)
        dy = dy.contiguous().to(torch.bfloat16)
        if dh is None:
            dx = kernels().rmsnorm_bwd(dy, h, m.detach(), rstd, dw)
        else:
            dx = kernels().rmsnorm_bwd_add(dy, h, m.detach(), rstd, dw, dh.contiguous().to(torch.bfloat16))
        return dx, dx, None, None


def add_rmsnorm(x: torch.Tensor, res: torch.Tensor | None, w: torch.Tensor, eps: float):
    """(h, rmsnorm(h)) with h = x + res (h = x when ``res`` is None): the decoder's residual add fused
    with the norm that follows it."""
    if res is None:
        return x, rmsnorm(x, w, eps)
    if not x.is_cuda:
        from .norm import rmsnorm_reference

        h = x + res
        return h, rmsnorm_reference(h, w, eps)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if res.dtype != torch.bfloat16:
        res = res.to(torch.bfloat16)
    return _AddRMSNormMP.apply(x, res, w, eps)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    if not x.is_cuda:
        from .norm import rmsnorm_reference

        return rmsnorm_reference(x, w, eps)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    return _RMSNormMP.apply(x, w, eps)


class _EmbeddingMP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w16, master, anchor):
        ctx.save_for_backward(ids)
        ctx.master = master
        return w16.index_select(0, ids)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        if ctx.master.requires_grad:
            main_grad(ctx.master).index_add_(0, ids, dy.float())
        return None, None, None, None


def embedding(ids: torch.Tensor, w: torch.Tensor, anchor: torch.Tensor | None = None) -> torch.Tensor:
    """Row lookup; on CUDA the backward scatters into the master's fp32 main_grad.

    ``anchor`` is any tensor that requires grad (autograd needs one input that does, so the
    backward runs); the model passes a dummy requiring-grad scalar.
    """
    if not ids.is_cuda:
        return torch.nn.functional.embedding(ids, w)
    if anchor is None:
        anchor = torch.zeros((), device=ids.device, requires_grad=True)
    return _EmbeddingMP.apply(ids, shadow(w), w, anchor)
