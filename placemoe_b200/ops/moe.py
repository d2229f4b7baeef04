"""Single-device MoE block on the sm_100a kernels, plus its PyTorch reference.

Data path of one MoE layer on one GPU (``moe_block``):

1. router logits ``x @ Wg^T`` (tcgen05 GEMM, fp32 out) -> softmax/top-k kernel
   (logical top-k; optional fixed bias for the skewed benchmarks);
2. dispatch plan: logical expert -> physical slot through the placement LUT,
   stable counting sort into 128-row-aligned expert segments (no host sync);
3. row gather -> grouped fc1 GEMM with fused SwiGLU and routing-weight scale
   -> grouped fc2 GEMM;
4. combine = sum of each token's k expert rows.

Backward mirrors it: row gather of dy, fc2 dgrad fused with the SwiGLU
backward (also yields the routing-weight gradient), fc1 dgrad, grouped weight
gradients accumulated straight into fp32 ``main_grad`` buffers, router
backward with the load-balancing-loss gradient folded in.

Reference parity: the fused-MoE forward of
veomni/ops/kernels/moe/group_gemm.py:634-961 (non-EP path) and the router of
veomni/models/transformers/qwen3_moe/generated/patched_modeling_qwen3_moe_gpu.py:306-337.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ._ext import kernels

ALIGN = 128  # expert segment alignment for single-CTA GEMM tiles
PAIR_ALIGN = 256  # alignment for CTA-pair (cta_group::2) tiles of 256 rows
# Average rows per expert slot from which 256-row segments pay: pair tiles move a third
# fewer operand bytes per SM, and the extra padding (~64 rows per slot on average) is
# small against segments of this length.
PAIR_MIN_ROWS = 768


def segment_align(assignments: int, num_slots: int) -> int:
    """Segment alignment of a dispatch plan with ``assignments`` rows over ``num_slots`` slots."""
    return PAIR_ALIGN if assignments >= PAIR_MIN_ROWS * max(num_slots, 1) else ALIGN


def capacity_rows(num_tokens: int, top_k: int, num_slots: int, align: int = ALIGN) -> int:
    """Upper bound of dispatched rows: every assignment plus per-slot padding."""
    return num_tokens * top_k + num_slots * (align - 1) + align


@dataclass
class RouterOut:
    idx: torch.Tensor  # [T, k] int32 logical experts
    weight: torch.Tensor  # [T, k] fp32
    prob_sum: torch.Tensor  # [E] fp32 sum over tokens of softmax probabilities
    count: torch.Tensor  # [E] fp32 number of assignments per logical expert


def router_reference(logits: torch.Tensor, bias, k: int, renorm: bool) -> RouterOut:
    z = logits.float() + (bias.float() if bias is not None else 0.0)
    p = torch.softmax(z, dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    count = torch.zeros(p.shape[-1], dtype=torch.float32, device=p.device)
    count.index_add_(0, idx.reshape(-1), torch.ones(idx.numel(), device=p.device))
    return RouterOut(idx.to(torch.int32), w, p.sum(0), count)


def load_balancing_loss(prob_sum: torch.Tensor, count: torch.Tensor, num_tokens: int, top_k: int) -> torch.Tensor:
    """Switch-style auxiliary loss  E * sum_e f_e * P_e  (f_e: assignment fraction, P_e: mean prob)."""
    e = prob_sum.numel()
    f = count / max(num_tokens * top_k, 1)
    p = prob_sum / max(num_tokens, 1)
    return e * (f * p).sum()


def apply_router_replay(replay, layer: int, logits, bias, w, idx, renorm: bool):
    """Record the routes, or substitute recorded ones (weights recomputed from ``logits``)."""
    if replay is None or replay.mode == "off":
        return w, idx
    if replay.mode == "record":
        replay.record(layer, idx)
        return w, idx
    from .router_replay import replay_weights

    idx = replay.fetch(layer).to(idx.device, idx.dtype)
    return replay_weights(logits, bias, idx, renorm), idx


def moe_block_reference(x, wg, bias, w1, w2, k, renorm, aux_coef=0.0, lut=None, return_route=False, replay=None,
                        layer: int = 0):
    """Eager oracle.  x [T, H]; wg [E, H]; w1 [S, 2I, H]; w2 [S, H, I]; lut: logical -> slot."""
    t = x.shape[0]
    logits = x.float() @ wg.float().t()
    z = logits + (bias.float() if bias is not None else 0.0)
    p = torch.softmax(z, dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    w, idx = apply_router_replay(replay, layer, logits, bias, w, idx, renorm)
    slots = lut[idx] if lut is not None else idx
    inter = w1.shape[1] // 2
    y = torch.zeros(t, x.shape[1], dtype=torch.float32, device=x.device)
    xf = x.float()
    for s in torch.unique(slots).tolist():
        tok, kk = torch.nonzero(slots == s, as_tuple=True)
        gu = xf[tok] @ w1[s].float().t()
        h = F.silu(gu[:, :inter]) * gu[:, inter:]
        o = h @ w2[s].float().t()
        y.index_add_(0, tok, o * w[tok, kk][:, None])
    aux = None
    if aux_coef:
        count = torch.zeros(p.shape[-1], dtype=torch.float32, device=x.device)
        count.index_add_(0, idx.reshape(-1), torch.ones(idx.numel(), device=x.device))
        aux = aux_coef * load_balancing_loss(p.sum(0), count, t, k)
    if return_route:
        return y.to(x.dtype), aux, idx
    return y.to(x.dtype), aux


def _accum_main_grad(param: torch.Tensor) -> torch.Tensor:
    g = getattr(param, "main_grad", None)
    if g is None:
        g = torch.zeros(param.shape, device=param.device, dtype=torch.float32)
        param.main_grad = g
    return g


def wgrad_target(param: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """(main_grad buffer, accumulate) for a weight-gradient GEMM.

    After ``mark_grads_stale`` the buffer holds last step's values: the first
    GEMM of the step overwrites it (an fp32 store instead of a read-modify-
    write, and no zero fill) and later micro-batches accumulate.
    """
    g = _accum_main_grad(param)
    if getattr(param, "_main_grad_stale", False):
        param._main_grad_stale = False
        return g, False
    return g, True


def mark_grads_stale(params) -> None:
    """Start a new accumulation without zeroing: the next weight-gradient GEMM overwrites."""
    for p in params:
        if getattr(p, "main_grad", None) is not None:
            p._main_grad_stale = True


def settle_stale_grads(params) -> None:
    """Zero the buffers that no GEMM overwrote since ``mark_grads_stale`` (unused parameters)."""
    for p in params:
        if getattr(p, "_main_grad_stale", False):
            p.main_grad.zero_()
            p._main_grad_stale = False


class ExpertFFN(torch.autograd.Function):
    """Grouped SwiGLU expert FFN over dispatched rows.

    Inputs: xd [rows, H] bf16 (expert-contiguous segments aligned to ``align``
    rows: 128, or 256 for CTA-pair tiles), scale [rows] fp32 routing weights,
    w1 [S, 2I, H] / w2 [S, H, I] bf16 compute copies, offsets [S+1] int32.
    Weight gradients are accumulated into the fp32 ``main_grad`` of ``p1`` /
    ``p2`` (the master parameters).
    """

    @staticmethod
    def forward(ctx, xd, scale, w1, w2, offsets, p1, p2, align=ALIGN):
        kn = kernels()
        rows = xd.shape[0]
        inter = w1.shape[1] // 2
        h = torch.empty(rows, inter, device=xd.device, dtype=torch.bfloat16)
        gu = torch.empty(rows, 2 * inter, device=xd.device, dtype=torch.bfloat16)
        kn.moe_fc1_swiglu(xd, w1, offsets, scale, h, gu, align, None)
        y = torch.empty(rows, w2.shape[1], device=xd.device, dtype=torch.bfloat16)
        kn.moe_grouped_gemm(h, w2, offsets, y, False, align)
        ctx.save_for_backward(xd, scale, w1, w2, offsets, h, gu)
        ctx.params = (p1, p2)
        ctx.align = align
        return y

    @staticmethod
    def backward(ctx, dy):
        xd, scale, w1, w2, offsets, h, gu = ctx.saved_tensors
        p1, p2 = ctx.params
        kn = kernels()
        dy = dy.contiguous()
        rows = xd.shape[0]
        dgu = torch.empty_like(gu)
        dscale = torch.zeros(rows, device=xd.device, dtype=torch.float32)
        kn.moe_fc2_dgrad_dswiglu(dy, w2, offsets, gu, scale, dgu, dscale, ctx.align)
        dx = torch.empty_like(xd)
        kn.moe_grouped_gemm(dgu, w1, offsets, dx, True, ctx.align)
        if p2 is not None and p2.requires_grad:
            kn.moe_wgrad(dy, h, offsets, *wgrad_target(p2), None)
        if p1 is not None and p1.requires_grad:
            kn.moe_wgrad(dgu, xd, offsets, *wgrad_target(p1), None)
        return dx, dscale, None, None, None, None, None, None


_DENSE_META: dict = {}


def dense_swiglu_mlp(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """down(silu(gate x) * up x) for dense decoders; w_gate_up [1, 2I, H] (gate rows first), w_down [1, H, I].

    CUDA runs the grouped SwiGLU GEMMs with one group covering every token
    (rows padded to the segment alignment), so the dense MLP shares the fused
    epilogues and fp32 master-gradient accumulation of the expert path.
    """
    inter = w_gate_up.shape[1] // 2
    if not x.is_cuda:
        gu = x.float() @ w_gate_up[0].float().t()
        return ((F.silu(gu[:, :inter]) * gu[:, inter:]) @ w_down[0].float().t()).to(x.dtype)
    from .mp import shadow

    t = x.shape[0]
    rows = -(-t // ALIGN) * ALIGN
    key = (rows, x.device)
    meta = _DENSE_META.get(key)
    if meta is None:
        meta = (torch.tensor([0, rows], dtype=torch.int32, device=x.device),
                torch.ones(rows, dtype=torch.float32, device=x.device))
        _DENSE_META[key] = meta
    offsets, scale = meta
    xb = x.to(torch.bfloat16).contiguous()
    if rows != t:
        xb = F.pad(xb, (0, 0, 0, rows - t))
    y = ExpertFFN.apply(xb, scale, shadow(w_gate_up), shadow(w_down), offsets, w_gate_up, w_down, ALIGN)
    return y[:t] if rows != t else y


class GatheredExpertFFN(torch.autograd.Function):
    """Expert FFN over dispatched rows of the token matrix, with optional recomputation.

    x [T, H] bf16 tokens; row_token [rows] int32 is the token of every
    dispatched row (-1 on padding), row_of the dispatched rows of every token,
    k per token (for the backward sum).  The dispatched copy xd = x[row_token]
    feeds the grouped GEMMs; with ``keep_rows=False`` it is dropped after the
    forward and gathered again in the backward, which trades one gather for
    ``rows x H`` bf16 of activation memory per layer.  (The GEMM kernels can
    also read the rows straight from x with TMA row gathers -- ``gather_idx``
    -- but four-row gathers issue too slowly to feed the tensor cores.)
    Returns the expert outputs [rows, H]; the input gradient is returned per
    token (summed over its dispatched rows).
    """

    @staticmethod
    def forward(ctx, x, scale, w1, w2, offsets, row_token, end, row_of, p1, p2, align=ALIGN, keep_rows=True):
        kn = kernels()
        rows = row_token.numel()
        inter = w1.shape[1] // 2
        xd = torch.empty(rows, x.shape[1], device=x.device, dtype=torch.bfloat16)
        kn.gather_rows(x, row_token, end, xd)
        h = torch.empty(rows, inter, device=x.device, dtype=torch.bfloat16)
        gu = torch.empty(rows, 2 * inter, device=x.device, dtype=torch.bfloat16)
        kn.moe_fc1_swiglu(xd, w1, offsets, scale, h, gu, align, None)
        y = torch.empty(rows, w2.shape[1], device=x.device, dtype=torch.bfloat16)
        kn.moe_grouped_gemm(h, w2, offsets, y, False, align)
        ctx.save_for_backward(x, xd if keep_rows else None, scale, w1, w2, offsets, row_token, end, row_of, h, gu)
        ctx.params = (p1, p2)
        ctx.align = align
        return y

    @staticmethod
    def backward(ctx, dy):
        x, xd, scale, w1, w2, offsets, row_token, end, row_of, h, gu = ctx.saved_tensors
        p1, p2 = ctx.params
        kn = kernels()
        dy = dy.contiguous()
        rows = row_token.numel()
        dgu = torch.empty_like(gu)
        dscale = torch.zeros(rows, device=x.device, dtype=torch.float32)
        kn.moe_fc2_dgrad_dswiglu(dy, w2, offsets, gu, scale, dgu, dscale, ctx.align)
        dxd = torch.empty(rows, x.shape[1], device=x.device, dtype=torch.bfloat16)
        kn.moe_grouped_gemm(dgu, w1, offsets, dxd, True, ctx.align)
        if p2 is not None and p2.requires_grad:
            kn.moe_wgrad(dy, h, offsets, *wgrad_target(p2), None)
        if p1 is not None and p1.requires_grad:
            if xd is None:
                xd = torch.empty(rows, x.shape[1], device=x.device, dtype=torch.bfloat16)
                kn.gather_rows(x, row_token, end, xd)
            kn.moe_wgrad(dgu, xd, offsets, *wgrad_target(p1), None)
        dx = torch.empty_like(x)
        kn.sum_rows(dxd, row_of, dx)
        return dx, dscale, None, None, None, None, None, None, None, None, None, None


class _GatherRows(torch.autograd.Function):
    """out[r] = x[row_token[r]]; backward sums rows back per token through row_of."""

    @staticmethod
    def forward(ctx, x, row_token, end, row_of, rows):
        out = torch.empty(rows, x.shape[1], device=x.device, dtype=x.dtype)
        kernels().gather_rows(x, row_token, end, out)
        ctx.save_for_backward(row_of)
        ctx.t = x.shape[0]
        return out

    @staticmethod
    def backward(ctx, dout):
        (row_of,) = ctx.saved_tensors
        dx = torch.empty(ctx.t, dout.shape[1], device=dout.device, dtype=dout.dtype)
        kernels().sum_rows(dout.contiguous(), row_of, dx)
        return dx, None, None, None, None


class _SumRows(torch.autograd.Function):
    """out[t] = sum_k src[row_of[t, k]]; backward gathers dy rows."""

    @staticmethod
    def forward(ctx, src, row_of, row_token, end, t):
        out = torch.empty(t, src.shape[1], device=src.device, dtype=src.dtype)
        kernels().sum_rows(src, row_of, out)
        ctx.save_for_backward(row_token, end)
        ctx.rows = src.shape[0]
        return out

    @staticmethod
    def backward(ctx, dy):
        row_token, end = ctx.saved_tensors
        dsrc = torch.empty(ctx.rows, dy.shape[1], device=dy.device, dtype=dy.dtype)
        kernels().gather_rows(dy.contiguous(), row_token, end, dsrc)
        return dsrc, None, None, None, None


class _ScaleGather(torch.autograd.Function):
    """Per-row routing weights (rows of the dispatch plan) from [T, k] weights."""

    @staticmethod
    def forward(ctx, w, row_scale, row_of):
        ctx.save_for_backward(row_of)
        ctx.wshape = w.shape
        return row_scale

    @staticmethod
    def backward(ctx, dscale):
        (row_of,) = ctx.saved_tensors
        return kernels().gather_scalar(dscale.contiguous(), row_of).view(ctx.wshape), None, None


class _Router(torch.autograd.Function):
    """logits -> (top-k weights); backward produces d(logits) incl. the aux-loss term."""

    @staticmethod
    def forward(ctx, logits, bias, k, renorm, aux_grad_holder):
        idx, w, ps, cnt = kernels().router_topk_fwd(logits, bias, k, renorm)
        ctx.save_for_backward(logits, idx)
        ctx.bias = bias
        ctx.renorm = renorm
        ctx.holder = aux_grad_holder
        ctx.mark_non_differentiable(idx, ps, cnt)
        return w, idx, ps, cnt

    @staticmethod
    def backward(ctx, dw, _didx, _dps, _dcnt):
        logits, idx = ctx.saved_tensors
        aux = ctx.holder.get("grad")
        if dw is None:
            dw = torch.zeros(idx.shape, device=logits.device, dtype=torch.float32)
        dl = kernels().router_topk_bwd(logits, ctx.bias, idx, dw.float().contiguous(), aux, ctx.renorm)
        return dl, None, None, None, None


class _AuxLoss(torch.autograd.Function):
    """aux = coef * E * sum_e f_e P_e; its gradient wrt p[t, e] (coef*E*f_e/T) is handed to the router backward."""

    @staticmethod
    def forward(ctx, anchor, prob_sum, count, t, k, coef, holder):
        e = prob_sum.numel()
        f = count / max(t * k, 1)
        holder["grad_vec"] = coef * e * f / max(t, 1)
        ctx.holder = holder
        return (coef * e * (f * prob_sum / max(t, 1)).sum()).reshape(())

    @staticmethod
    def backward(ctx, g):
        ctx.holder["grad"] = (ctx.holder["grad_vec"] * g).float().contiguous()
        return None, None, None, None, None, None, None


def moe_block(x, wg, bias, w1_bf16, w2_bf16, p1, p2, k, renorm, num_slots, lut=None, aux_coef=0.0, keep_rows=True,
              replay=None, layer: int = 0):
    """Single-device MoE layer. Returns (y [T, H] bf16, aux_loss or None, router stats).

    ``keep_rows=False`` recomputes the dispatched input rows in the backward
    instead of keeping them (see :class:`GatheredExpertFFN`).
    """
    t, hdim = x.shape
    kn = kernels()
    logits = linear_fp32(x, wg)
    holder: dict = {}
    w, idx, ps, cnt = _Router.apply(logits, bias, k, renorm, holder)
    aux = None
    if replay is not None and replay.mode == "replay":
        w, idx = apply_router_replay(replay, layer, logits, bias, w, idx, renorm)
        idx = idx.to(torch.int32).contiguous()
    else:
        if aux_coef:
            aux = _AuxLoss.apply(w, ps, cnt, t, k, float(aux_coef), holder)
        apply_router_replay(replay, layer, logits, bias, w, idx, renorm)
    align = segment_align(t * k, num_slots)
    cap = capacity_rows(t, k, num_slots, align)
    offsets, counts, row_of, row_token, row_scale = kn.moe_plan(idx, lut, w.detach(), num_slots, cap, align)
    end = offsets[num_slots:]
    scale = _ScaleGather.apply(w, row_scale, row_of)
    yd = GatheredExpertFFN.apply(x.contiguous(), scale, w1_bf16, w2_bf16, offsets, row_token, end, row_of, p1, p2,
                                 align, keep_rows)
    y = _SumRows.apply(yd, row_of, row_token, end, t)
    return y, aux, idx


def linear_fp32(x, w):
    """x @ w^T with an fp32 result (router logits); dW accumulates into w.main_grad."""
    from .mp import linear

    return linear(x, w, fp32_out=True)
