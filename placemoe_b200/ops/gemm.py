"""Dense GEMM ops on the tcgen05 kernel (``csrc/kernels/gemm_sm100.cuh``, ``gemm_dense.cu``).

``linear(x, w)`` computes ``x @ w.T`` in bf16 with fp32 accumulation; its
backward issues the data gradient (``dy @ w``, B operand MN-major) and the
weight gradient (``dy.T @ x``, both operands MN-major) on the same kernel
family.  CPU tensors use ``torch.nn.functional.linear`` (reference path).

Reference parity: dense projections of the Qwen3-MoE / OLMoE decoders run
through torch/cuBLAS in the reference
(veomni/models/transformers/qwen3_moe/generated/patched_modeling_qwen3_moe_gpu.py).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import kernels


def _mat(t: torch.Tensor) -> torch.Tensor:
    t = t.reshape(-1, t.shape[-1])
    if t.stride(-1) != 1 or (t.stride(0) * t.element_size()) % 16 or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def gemm_nt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
            accumulate: bool = False) -> torch.Tensor:
    """out[M, N] = a[M, K] @ b[N, K]^T."""
    a2, b2 = _mat(a), _mat(b)
    if out is None:
        out = torch.empty(a2.shape[0], b2.shape[0], device=a.device, dtype=out_dtype)
    kernels().dense_gemm(a2, b2, out, False, False, accumulate)
    return out


def gemm_nn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = a[M, K] @ b[K, N]."""
    a2, b2 = _mat(a), _mat(b)
    if out is None:
        out = torch.empty(a2.shape[0], b2.shape[1], device=a.device, dtype=torch.bfloat16)
    kernels().dense_gemm(a2, b2, out, False, True, False)
    return out


def gemm_tn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
            accumulate: bool = False) -> torch.Tensor:
    """out[M, N] = a[K, M]^T @ b[K, N]  (weight-gradient layout)."""
    a2, b2 = _mat(a), _mat(b)
    if out is None:
        out = torch.empty(a2.shape[1], b2.shape[1], device=a.device, dtype=out_dtype)
    kernels().dense_gemm(a2, b2, out, True, True, accumulate)
    return out


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        y = gemm_nt(x, w)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy2 = _mat(dy.to(torch.bfloat16))
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm_nn(dy2, w).view(x.shape)
        if ctx.needs_input_grad[1]:
            dw = gemm_tn(dy2, _mat(x), out_dtype=w.dtype if w.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y = x @ w.T (no bias)."""
    if not x.is_cuda:
        return F.linear(x, w)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if w.dtype != torch.bfloat16:
        w = w.to(torch.bfloat16)
    return _Linear.apply(x, w)
