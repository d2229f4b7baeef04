"""Causal GQA attention over packed fixed-length sequences.

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


def attention_reference(q, k, v, seq_len):
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
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2).reshape(t, hq, d).to(q.dtype)


def _has_kernel() -> bool:
    return hasattr(kernels(), "attn_fwd")


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seq_len):
        o, lse = kernels().attn_fwd(q, k, v, seq_len)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.seq_len = seq_len
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = kernels().attn_bwd(q, k, v, o, lse, do.contiguous(), ctx.seq_len)
        return dq, dk, dv, None


def causal_attention(q, k, v, seq_len: int):
    if not q.is_cuda:
        return attention_reference(q, k, v, seq_len)
    if _has_kernel():
        return _FlashAttn.apply(q.contiguous(), k.contiguous(), v.contiguous(), seq_len)
    # Interim path until the tcgen05 attention kernel is part of the build.
    t, hq, d = q.shape
    hkv = k.shape[1]
    b = t // seq_len
    qq = q.reshape(b, seq_len, hq, d).transpose(1, 2)
    kk = k.reshape(b, seq_len, hkv, d).transpose(1, 2)
    vv = v.reshape(b, seq_len, hkv, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=hq != hkv)
    return o.transpose(1, 2).reshape(t, hq, d)
