"""RMSNorm and fused QK-norm + RoPE (``csrc/kernels/norm_rope.cu``).

CPU tensors run the PyTorch reference formulas below; CUDA tensors run the
sm_100a kernels.  The rotary convention is rotate-half with a fp32
inverse-frequency table ``theta ** (-2i / head_dim)``.

Reference parity: veomni/ops/liger/__init__.py:52-133 (RMSNorm, RoPE) and the
Qwen3-MoE / OLMoE attention blocks in veomni/models/transformers/.
"""

from __future__ import annotations

import torch

from ._ext import kernels


def rmsnorm_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r * w.float()).to(x.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        x2 = x.contiguous()
        y, rstd = kernels().rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        dx = kernels().rmsnorm_bwd(dy.contiguous().to(torch.bfloat16), x, w, rstd, dw)
        return dx, dw.to(w.dtype), None


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    if not x.is_cuda:
        return rmsnorm_reference(x, w, eps)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    return _RMSNorm.apply(x, w, eps)


def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))


def _rotate(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    # x: [T, H, D] float
    ang = pos.float()[:, None] * inv_freq[None, :]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def qkv_rope_reference(qkv, pos, inv_freq, qw, kw, hq, hkv, d, q_group, k_group, eps):
    t = qkv.shape[0]
    x = qkv.float()
    q = x[:, : hq * d]
    k = x[:, hq * d: (hq + hkv) * d]
    v = x[:, (hq + hkv) * d:]

    def norm(z, w, g):
        if not g:
            return z
        zz = z.reshape(t, -1, g)
        r = torch.rsqrt(zz.pow(2).mean(-1, keepdim=True) + eps)
        return (zz * r * w.float()).reshape(t, -1)

    q = _rotate(norm(q, qw, q_group).reshape(t, hq, d), pos, inv_freq)
    k = _rotate(norm(k, kw, k_group).reshape(t, hkv, d), pos, inv_freq)
    return q.to(qkv.dtype), k.to(qkv.dtype), v.reshape(t, hkv, d).to(qkv.dtype)


_ROPE_TABLES: dict = {}


def rope_table(inv_freq: torch.Tensor, length: int) -> torch.Tensor:
    """(cos, sin) of p * inv_freq for positions p < length: [length, D/2, 2] fp32 (cached)."""
    key = (inv_freq.data_ptr(), inv_freq.device, inv_freq.numel())
    tab = _ROPE_TABLES.get(key)
    if tab is None or tab.shape[0] < length:
        n = max(length, tab.shape[0] * 2 if tab is not None else 0)
        ang = torch.arange(n, device=inv_freq.device, dtype=torch.float64)[:, None] * inv_freq.double()[None, :]
        tab = torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().contiguous()
        _ROPE_TABLES[key] = tab
    return tab


class _QkvRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qw, kw, pos, rope, hq, hkv, d, q_group, k_group, eps):
        qkv = qkv.contiguous()
        qwd = qw.detach() if qw is not None else None
        kwd = kw.detach() if kw is not None else None
        q, k, v, rq, rk = kernels().qkv_rope_fwd(qkv, pos, rope, qwd, kwd, hq, hkv, d, q_group, k_group, eps)
        ctx.save_for_backward(qkv, pos, rope, rq, rk)
        ctx.masters = (qw, kw)
        ctx.cfg = (hq, hkv, d, q_group, k_group)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        from .mp import main_grad

        qkv, pos, rope, rq, rk = ctx.saved_tensors
        hq, hkv, d, q_group, k_group = ctx.cfg
        qw, kw = ctx.masters

        def acc(m):
            if m is None:
                return None
            return main_grad(m) if m.requires_grad else torch.zeros(m.shape, device=qkv.device, dtype=torch.float32)

        bf = torch.bfloat16
        dqkv = kernels().qkv_rope_bwd(
            dq.contiguous().to(bf), dk.contiguous().to(bf), dv.contiguous().to(bf), qkv, pos, rope,
            qw.detach() if qw is not None else None, kw.detach() if kw is not None else None, rq, rk,
            acc(qw), acc(kw), hq, hkv, d, q_group, k_group,
        )
        return dqkv, None, None, None, None, None, None, None, None, None, None


def qkv_norm_rope(qkv, q_norm_w, k_norm_w, pos, inv_freq, hq, hkv, d, q_group, k_group, eps, max_pos=None):
    """Split a fused QKV projection [T, (hq+2hkv)*d] into rotated, normalised q, k and v.

    ``q_group``/``k_group`` are the RMSNorm group sizes (``d`` for per-head
    norms, the full width for OLMoE-style norms, 0 for none).  On CUDA the
    norm weights are fp32 masters whose gradients accumulate into ``main_grad``
    and the rotation reads a (cos, sin) table covering positions < ``max_pos``
    (default: the number of tokens); a position outside it raises the device
    error flag.
    """
    if not qkv.is_cuda:
        return qkv_rope_reference(qkv, pos, inv_freq, q_norm_w, k_norm_w, hq, hkv, d, q_group, k_group, eps)
    for w in (q_norm_w, k_norm_w):
        if w is not None and w.dtype != torch.float32:
            raise TypeError("QK-norm weights must be fp32 masters on the CUDA path")
    rope = rope_table(inv_freq, int(max_pos) if max_pos else qkv.shape[0])
    return _QkvRope.apply(qkv.to(torch.bfloat16), q_norm_w, k_norm_w, pos.to(torch.int32), rope, hq, hkv, d,
                          q_group, k_group, eps)
