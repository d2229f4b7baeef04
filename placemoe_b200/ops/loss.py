"""Chunked fused linear cross-entropy (lm-head GEMM + CE + backward GEMMs).

For each chunk of tokens: logits = h_chunk @ W^T (tcgen05 GEMM, bf16), the CE
kernel turns the logits into d(loss)/d(logits) in place while accumulating the
loss, then dh_chunk = dlogits @ W and dW += dlogits^T @ h_chunk (fp32
accumulation).  The [tokens, vocab] logits tensor never exists in full; the
backward work is done during the forward call and replayed by autograd.

Reference parity: veomni/ops/kernels/cross_entropy/ (chunked CE and the Liger
fused linear cross-entropy).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import kernels
from .gemm import gemm_nn, gemm_nt, gemm_tn

IGNORE_INDEX = -100


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, chunk, denom):
        from .mp import shadow

        h2 = h.reshape(-1, h.shape[-1]).to(torch.bfloat16).contiguous()
        wb = shadow(w) if w.dtype == torch.float32 else w.to(torch.bfloat16).contiguous()
        n = h2.shape[0]
        labels = labels.reshape(-1).to(torch.int64).contiguous()
        loss_sum = torch.zeros((), device=h.device, dtype=torch.float32)
        dh = torch.empty_like(h2)
        dw = torch.empty(w.shape, device=w.device, dtype=torch.float32)  # the first chunk stores, later ones add
        if n == 0:
            dw.zero_()
        kn = kernels()
        scale = 1.0 / float(denom)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            logits = gemm_nt(h2[s:e], wb)
            kn.ce_fwd_bwd(logits, labels[s:e], IGNORE_INDEX, scale, loss_sum, None)
            gemm_nn(logits, wb, out=dh[s:e])
            gemm_tn(logits, h2[s:e], out=dw, accumulate=s > 0)
        ctx.save_for_backward(dh, dw)
        ctx.shape = h.shape
        ctx.master = w
        return loss_sum * scale

    @staticmethod
    def backward(ctx, g):
        from .mp import main_grad

        dh, dw = ctx.saved_tensors
        dh = (dh.float() * g).to(torch.bfloat16).reshape(ctx.shape)
        w = ctx.master
        if w.dtype == torch.float32 and w.requires_grad:
            main_grad(w).addcmul_(dw, g)  # one pass, g stays on the device
            return dh, None, None, None, None
        return dh, (dw * g).to(w.dtype), None, None, None


def fused_linear_cross_entropy(h, w, labels, chunk: int = 8192, denom=None):
    """Mean CE over non-ignored labels of (h @ w^T).  ``denom`` overrides the divisor (global token count)."""
    if denom is None:
        denom = max(int((labels != IGNORE_INDEX).sum().item()), 1)
    if not h.is_cuda:
        logits = F.linear(h.reshape(-1, h.shape[-1]).float(), w.float())
        return F.cross_entropy(logits, labels.reshape(-1), ignore_index=IGNORE_INDEX, reduction="sum") / denom
    return _FusedLinearCE.apply(h, w, labels, chunk, denom)
