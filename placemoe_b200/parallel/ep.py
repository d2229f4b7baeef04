"""Expert parallelism with per-destination deduplicated dispatch and pre-reduced combine.

Forward of one MoE layer on EP rank r:

1. router on the local tokens -> logical top-k (unchanged by placement);
2. M[r] maps each logical expert to a physical slot -> (destination GPU, local slot);
3. dedup: a token is sent ONCE to every destination GPU that holds at least
   one of its experts, together with per-assignment metadata
   (row index, local slot, routing weight);
4. the receiver expands rows to assignments, runs its local expert slots
   (grouped SwiGLU GEMMs on the GPU) and PRE-REDUCES the weighted outputs of
   all assignments of a received row into one partial sum;
5. partial sums travel back (one row per (token, destination)) and are summed
   into the token.

The transport here is ``torch.distributed.all_to_all_single`` with split
sizes exchanged first (works on gloo for the CPU tests and on NCCL as the
baseline); :mod:`placemoe_b200.parallel.p2p_moe` replaces it on B200 with
fused peer-memory kernels and no host synchronisation.

Reference parity: rank_dedup_dispatch / rank_dedup_combine
(veomni/distributed/moe/hiermoe/all_to_all.py:979-1055, :2029-2263,
:2266-2294, :2539-2564) and the pair all-to-all of
veomni/distributed/moe/comm.py:167-303.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops import moe as moe_ops


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_splits, recv_splits, group):
        ctx.splits = (send_splits, recv_splits)
        ctx.group = group
        out = x.new_empty((sum(recv_splits), *x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        send_splits, recv_splits = ctx.splits
        out = g.new_empty((sum(send_splits), *g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), send_splits, recv_splits, group=ctx.group)
        return out, None, None, None


def all_to_all(x, send_splits, recv_splits, group=None):
    return _AllToAll.apply(x, list(send_splits), list(recv_splits), group)


def _exchange_counts(counts: torch.Tensor, group) -> torch.Tensor:
    out = torch.empty_like(counts)
    dist.all_to_all_single(out, counts.contiguous(), group=group)
    return out


def build_dispatch(dest: torch.Tensor, lslot: torch.Tensor, world: int):
    """Per-destination dedup bookkeeping (index-only, no autograd).

    dest, lslot: [T, k] int64.  Returns
      send_tok   [S]   token of every sent row, ordered by (dest, token);
      row_counts [W]   rows sent to each destination;
      asg_row    [A]   sent-row index (within its destination chunk) of every assignment,
                       ordered by (dest, token, k);
      asg_slot   [A]   local slot at the destination;  asg_src [A] flat (t*k + j) index;
      asg_counts [W]   assignments sent to each destination.
    """
    t, k = dest.shape
    dev = dest.device
    onehot_t = torch.zeros(world, t, dtype=torch.long, device=dev)
    onehot_t[dest.reshape(-1), torch.arange(t, device=dev).repeat_interleave(k)] = 1  # [W, T]
    onehot = onehot_t.t()  # [T, W] 1 if the token goes to that GPU
    row_counts = onehot_t.sum(1)
    # send order: destination-major, token-minor
    d_idx, t_idx = torch.nonzero(onehot_t, as_tuple=True)
    send_tok = t_idx
    # position of (t, d) within destination d's chunk (scanned along the contiguous axis)
    pos_in_d = (torch.cumsum(onehot_t, 1) - 1).t()  # [T, W]
    flat_d = dest.reshape(-1)
    flat_t = torch.arange(t, device=dev).repeat_interleave(k)
    order = torch.argsort(flat_d * (t * k) + torch.arange(t * k, device=dev))
    asg_dest = flat_d[order]
    asg_row = pos_in_d[flat_t[order], asg_dest]
    asg_slot = lslot.reshape(-1)[order]
    asg_counts = torch.bincount(flat_d, minlength=world)
    return send_tok, row_counts, asg_row, asg_slot, order, asg_counts, d_idx


class ExpertParallel:
    """Multi-rank MoE forward for one process group (EP == the group)."""

    def __init__(self, group=None, capture_routes: bool = False):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.capture_routes = capture_routes
        self.stats = {}

    # ------------------------------------------------------------------ router
    def _route(self, blk, x, bias, aux_coef):
        cfg = blk.cfg
        k = cfg.num_experts_per_tok
        t = x.shape[0]
        if x.is_cuda:
            logits = moe_ops.linear_fp32(x, blk.gate)
            holder: dict = {}
            w, idx, ps, cnt = moe_ops._Router.apply(logits, bias, k, cfg.norm_topk_prob, holder)
            replay = getattr(blk, "router_replay", None)
            if replay is not None and replay.mode == "replay":
                w, idx = moe_ops.apply_router_replay(replay, blk.layer_idx, logits, bias, w, idx, cfg.norm_topk_prob)
                return w, idx.long(), None
            aux = moe_ops._AuxLoss.apply(w, ps, cnt, t, k, float(aux_coef), holder) if aux_coef else None
            moe_ops.apply_router_replay(replay, blk.layer_idx, logits, bias, w, idx, cfg.norm_topk_prob)
            return w, idx.long(), aux
        logits = x.float() @ blk.gate.float().t()
        z = logits + (bias.float() if bias is not None else 0.0)
        p = torch.softmax(z, -1)
        w, idx = torch.topk(p, k, dim=-1)
        if cfg.norm_topk_prob:
            w = w / w.sum(-1, keepdim=True)
        w, idx = moe_ops.apply_router_replay(getattr(blk, "router_replay", None), blk.layer_idx, logits, bias, w, idx,
                                             cfg.norm_topk_prob)
        aux = None
        if aux_coef:
            count = torch.zeros(p.shape[-1], device=x.device).index_add_(0, idx.reshape(-1),
                                                                        torch.ones(idx.numel(), device=x.device))
            aux = aux_coef * moe_ops.load_balancing_loss(p.sum(0), count, t, k)
        return w, idx, aux

    # ------------------------------------------------------------- forward
    def moe_forward(self, blk, x, bias, aux_coef):
        t, h = x.shape
        k = blk.cfg.num_experts_per_tok
        w, idx, aux = self._route(blk, x, bias, aux_coef)
        pl = blk.placement
        dest_tab, slot_tab = pl.route_tables(x.device)
        dest = dest_tab.long()[idx]
        lslot = slot_tab.long()[idx]
        send_tok, row_counts, asg_row, asg_slot, order, asg_counts, _ = build_dispatch(dest, lslot, self.world)
        counts = torch.stack([row_counts, asg_counts], 1).to(torch.int64)  # [W, 2]
        rcounts = _exchange_counts(counts, self.group)
        host = torch.cat([counts, rcounts], 1).cpu()  # single host sync (baseline transport)
        send_rows, send_asg = host[:, 0].tolist(), host[:, 1].tolist()
        recv_rows, recv_asg = host[:, 2].tolist(), host[:, 3].tolist()

        xs = x.index_select(0, send_tok)
        recv_x = all_to_all(xs, send_rows, recv_rows, self.group)
        meta = torch.stack([asg_row, asg_slot], 1)
        recv_meta = all_to_all(meta, send_asg, recv_asg, self.group)
        w_sorted = w.reshape(-1)[order]
        recv_w = all_to_all(w_sorted.float(), send_asg, recv_asg, self.group)
        # global receive-row index of every received assignment
        row_base = torch.repeat_interleave(
            torch.cumsum(torch.tensor([0] + recv_rows[:-1], device=x.device), 0),
            torch.tensor(recv_asg, device=x.device))
        recv_row = recv_meta[:, 0] + row_base
        recv_slot = recv_meta[:, 1]
        partial = self._local_experts(blk, recv_x, recv_row, recv_slot, recv_w, sum(recv_rows))
        back = all_to_all(partial, recv_rows, send_rows, self.group)
        y = torch.zeros(t, h, device=x.device, dtype=torch.float32).index_add(0, send_tok, back.float())
        self.stats = {"sent_rows": sum(send_rows), "sent_assignments": sum(send_asg),
                      "dedup_ratio": sum(send_asg) / max(sum(send_rows), 1)}
        if self.capture_routes:
            blk.last_route = idx.detach()
        return y.to(x.dtype), aux, idx

    def _local_experts(self, blk, recv_x, recv_row, recv_slot, recv_w, nrows):
        """Pre-reduced expert outputs, one row per received row."""
        h = recv_x.shape[1]
        if not recv_x.is_cuda:
            inter = blk.gate_up_proj.shape[1] // 2
            partial = torch.zeros(nrows, h, dtype=torch.float32, device=recv_x.device)
            xf = recv_x.float()
            for s in torch.unique(recv_slot).tolist():
                sel = torch.nonzero(recv_slot == s, as_tuple=True)[0]
                rows = recv_row[sel]
                gu = xf[rows] @ blk.gate_up_proj[s].float().t()
                o = (F.silu(gu[:, :inter]) * gu[:, inter:]) @ blk.down_proj[s].float().t()
                partial = partial.index_add(0, rows, o * recv_w[sel][:, None])
            return partial.to(recv_x.dtype)
        return _cuda_local_experts(blk, recv_x, recv_row, recv_slot, recv_w, nrows)


def _cuda_local_experts(blk, recv_x, recv_row, recv_slot, recv_w, nrows):
    kn = moe_ops.kernels()
    n = recv_slot.shape[0]
    spr = blk.num_local_slots
    k = blk.cfg.num_experts_per_tok
    align = moe_ops.segment_align(n, spr)
    cap = moe_ops.capacity_rows(n, 1, spr, align)
    slot32 = recv_slot.to(torch.int32).reshape(n, 1).contiguous()
    offsets, counts, row_of, row_token, row_scale = kn.moe_plan(slot32, None, recv_w.detach().contiguous(), spr,
                                                                cap, align)
    end = offsets[spr:]
    # dispatched row -> received row.  Rows at or beyond offsets[spr] are not written by the
    # plan (uninitialised), so they are masked by the device-side end before any indexing.
    in_plan = torch.arange(cap, device=recv_x.device, dtype=torch.int32) < end
    rt = torch.where(in_plan & (row_token >= 0), row_token, torch.full_like(row_token, -1))
    row_src = torch.where(rt >= 0, recv_row.to(torch.int32)[rt.clamp_min(0).long()], rt)
    # received row -> its dispatched rows, padded to k entries
    first = torch.zeros(nrows + 1, dtype=torch.long, device=recv_x.device)
    first.index_add_(0, recv_row + 1, torch.ones_like(recv_row))
    first = torch.cumsum(first, 0)
    pos = torch.arange(n, device=recv_x.device) - first[recv_row]
    table = torch.full((nrows, k), -1, dtype=torch.int32, device=recv_x.device)
    table[recv_row, pos] = row_of.view(-1)
    scale = moe_ops._ScaleGather.apply(recv_w, row_scale, row_of)
    w1, w2 = blk.compute_weights()
    row_src = row_src.to(torch.int32).contiguous()
    yd = moe_ops.GatheredExpertFFN.apply(recv_x.contiguous(), scale, w1, w2, offsets, row_src, end, table,
                                         blk.gate_up_proj, blk.down_proj, align, blk.keep_expert_rows)
    return moe_ops._SumRows.apply(yd, table, row_src, end, nrows)
