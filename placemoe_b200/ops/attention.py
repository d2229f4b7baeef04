"""Causal GQA attention over packed fixed-length sequences, optionally with several documents per row.

q: [T, Hq, D], k/v: [T, Hkv, D] with T = batch * seq_len (token-major, as
produced by the fused QKV-norm-RoPE kernel).  Returns [T, Hq, D].

CUDA tensors run the tcgen05 flash-attention kernels
(``csrc/kernels/attention_sm100.cu``) when they are built in; CPU tensors run
the PyTorch reference below.

Reference parity: veomni/ops/kernels/attention/__init__.py:151-353 (flash
attention forward/backward through FA2/FA3/FA4).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ._ext import kernels


def doc_bounds(cu_seqlens: torch.Tensor, num_tokens: int, seq_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token (first position, end position) of its document, relative to its row of seq_len tokens.

    ``cu_seqlens`` holds the cumulative document boundaries over the flattened tokens
    (first entry 0, last entry ``num_tokens``); every row boundary must also be a document
    boundary.  Returns two int32 tensors of ``num_tokens`` entries.
    """
    cu = cu_seqlens.to(torch.int64)
    if cu[0].item() != 0 or cu[-1].item() != num_tokens:
        raise ValueError("cu_seqlens must start at 0 and end at the token count")
    lens = cu[1:] - cu[:-1]
    if (lens <= 0).any():
        raise ValueError("documents must be non-empty")
    starts = torch.repeat_interleave(cu[:-1], lens)
    ends = torch.repeat_interleave(cu[1:], lens)
    row0 = torch.arange(num_tokens, device=cu.device) // seq_len * seq_len
    if ((ends - 1) // seq_len != starts // seq_len).any():
        raise ValueError("a document crosses a row of seq_len tokens")
    return (starts - row0).to(torch.int32), (ends - row0).to(torch.int32)


def attention_reference(q, k, v, seq_len, docs=None):
    t, hq, d = q.shape
    hkv = k.shape[1]
    b = t // seq_len
    qf = q.float().reshape(b, seq_len, hq, d).transpose(1, 2)
    kf = k.float().reshape(b, seq_len, hkv, d).transpose(1, 2)
    vf = v.float().reshape(b, seq_len, hkv, d).transpose(1, 2)
    if hq != hkv:
        kf = kf.repeat_interleave(hq // hkv, dim=1)
        vf = vf.repeat_interleave(hq // hkv, dim=1)
    s = (qf @ kf.transpose(-1, -2)) / math.sqrt(d)
    mask = torch.ones(seq_len, seq_len, dtype=torch.bool, device=q.device).tril()
    if docs is not None:  # keys of earlier documents are masked: key >= first position of the query's document
        lo = docs[0].to(q.device).long().reshape(b, seq_len)
        keys = torch.arange(seq_len, device=q.device)
        mask = mask[None] & (keys[None, None, :] >= lo[:, :, None])  # [b, q, k]
        mask = mask[:, None]
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2).reshape(t, hq, d).to(q.dtype)


def _has_kernel() -> bool:
    return hasattr(kernels(), "attn_fwd")


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seq_len, doc_lo, doc_hi):
        o, lse = kernels().attn_fwd(q, k, v, seq_len, doc_lo)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.seq_len = seq_len
        ctx.doc_hi = doc_hi
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = kernels().attn_bwd(q, k, v, o, lse, do.contiguous(), ctx.seq_len, ctx.doc_hi)
        return dq, dk, dv, None, None, None


def causal_attention(q, k, v, seq_len: int, docs=None):
    """``docs``: optional (doc_lo, doc_hi) int32 per-token document bounds (:func:`doc_bounds`)
    for rows that pack several documents; attention then stays inside each document."""
    if not q.is_cuda:
        return attention_reference(q, k, v, seq_len, docs)
    if _has_kernel():
        lo, hi = (None, None) if docs is None else (docs[0].contiguous(), docs[1].contiguous())
        return _FlashAttn.apply(q.contiguous(), k.contiguous(), v.contiguous(), seq_len, lo, hi)
    if docs is not None:
        raise RuntimeError("packed documents need the attention kernel")
    # Interim path until the tcgen05 attention kernel is part of the build.
    t, hq, d = q.shape
    hkv = k.shape[1]
    b = t // seq_len
    qq = q.reshape(b, seq_len, hq, d).transpose(1, 2)
    kk = k.reshape(b, seq_len, hkv, d).transpose(1, 2)
    vv = v.reshape(b, seq_len, hkv, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=hq != hkv)
    return o.transpose(1, 2).reshape(t, hq, d)
