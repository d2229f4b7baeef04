"""Expert parallelism over NVLink peer memory, without host synchronisation.

Each rank owns a symmetric arena (``torch.distributed._symmetric_memory``),
mapped into every peer; a device table holds the peer base addresses.  One MoE
layer call (rank r, world W, T tokens, top-k):

  1. router -> logical top-k; M[r] -> (destination GPU, local slot) per assignment;
  2. dedup bookkeeping on the device: which tokens go to which GPU, their row
     position per destination, assignment order (destination, token, k);
  3. every rank writes its per-destination (row, assignment) counts into all
     peers' count matrices; device barrier;
  4. from the count matrix each rank derives where its rows land in every
     destination's receive region (prefix over lower ranks) -- no host reads;
  5. rows (deduplicated: once per destination) and per-assignment metadata
     (receive row, local slot, routing weight, source index) are stored
     straight into the destinations' receive regions; device barrier;
  6. the receiver builds its expert plan from the metadata (device-side
     valid counts), gathers rows, runs the grouped SwiGLU GEMMs and pre-reduces
     the (weight-scaled) outputs of every received row;
  7. each partial sum is stored back into its source's return region at the
     source's send position; device barrier;
  8. the source sums its returned partials per token.

Backward runs the same phases in reverse (dy out to the destinations, data
gradients and routing-weight gradients back).  Barriers are bounded waits: a
peer that never arrives makes the kernel record an error the host raises.

Reference parity: rank_dedup_dispatch / rank_dedup_combine of
veomni/distributed/moe/hiermoe/all_to_all.py:2029-2264, :2539-2564 with the
NCCL all-to-all data plane replaced by peer stores.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops import moe as moe_ops
from ..ops import p2p_status

BARRIER_TIMEOUT_S = 30.0


class PhaseTimer:
    """Optional CUDA-event marks at phase boundaries (set ``p2p_ep.TIMER = PhaseTimer()``)."""

    def __init__(self):
        self.marks: list[tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str) -> None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.marks.append((name, e))

    def phases(self) -> dict[str, float]:
        out: dict[str, float] = {}
        for (_, a), (name, b) in zip(self.marks, self.marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


TIMER: PhaseTimer | None = None


def _mark(name: str) -> None:
    if TIMER is not None:
        TIMER.mark(name)


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class SymmetricArena:
    """A symmetric byte buffer carved into regions for one EP group."""

    def __init__(self, group, world: int, rank: int, tokens: int, k: int, hidden: int, device):
        import torch.distributed._symmetric_memory as symm_mem

        self.group, self.world, self.rank, self.tokens, self.k, self.hidden = group, world, rank, tokens, k, hidden
        rows = world * tokens  # at most every token of every source
        asg = world * tokens * k
        lay = {}
        off = 0
        for name, nbytes in (("flags", 64 * 4), ("counts", world * world * 2 * 4), ("recv_rows", rows * hidden * 2),
                             ("recv_meta", asg * 4 * 4), ("back_rows", rows * hidden * 2), ("back_words", asg * 4)):
            lay[name] = off
            off += _align(nbytes)
        self.layout = lay
        self.nbytes = off
        self.buf = symm_mem.empty(off, dtype=torch.uint8, device=device)
        self.buf.zero_()
        gname = group.group_name if group is not None else dist.group.WORLD.group_name
        self.handle = symm_mem.rendezvous(self.buf, gname)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.epoch = 0
        dist.barrier(group=group)

    def view(self, name: str, shape, dtype) -> torch.Tensor:
        off = self.layout[name]
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.tensor([], dtype=dtype).element_size()
        return self.buf[off: off + nbytes].view(dtype).view(*shape)

    def barrier(self):
        self.epoch += 1
        moe_ops.kernels().p2p_barrier(self.peers, self.layout["flags"], self.rank, self.epoch, BARRIER_TIMEOUT_S,
                                      p2p_status(self.buf.device))

    def fits(self, tokens: int, k: int, hidden: int) -> bool:
        return tokens <= self.tokens and k == self.k and hidden == self.hidden


def _dispatch_tables(dest: torch.Tensor, world: int):
    """dest [T, k] int64 -> onehot [T, W], pos_in_d [T, W], asg order pos [T, k] within destination.

    Built with scatter and row-wise scans only: ``F.one_hot`` validates its
    input with a device-to-host read, and a scan along a long outer dimension
    with W inner columns runs on W threads.  Scans run over [W, n] rows.
    """
    t, k = dest.shape
    dev = dest.device
    onehot_t = torch.zeros(world, t, dtype=torch.int32, device=dev)
    tok = torch.arange(t, device=dev).unsqueeze(1).expand(t, k)
    onehot_t[dest.reshape(-1), tok.reshape(-1)] = 1  # [W, T] (duplicates write the same 1)
    pos_t = torch.cumsum(onehot_t, 1, dtype=torch.int32) - 1  # [W, T]
    flat = dest.reshape(-1)
    oh_asg_t = torch.zeros(world, t * k, dtype=torch.int32, device=dev)
    oh_asg_t[flat, torch.arange(t * k, device=dev)] = 1  # [W, T*k] in (t, j) order
    asg_pos = (torch.cumsum(oh_asg_t, 1, dtype=torch.int32) - 1).gather(0, flat.view(1, -1)).view(t, k)
    # [T, W] row-major: the index tables built from these are handed to kernels as flat arrays
    return onehot_t.t().contiguous(), pos_t.t().contiguous(), asg_pos, oh_asg_t.sum(1)


class _P2PMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, blk, arena: SymmetricArena, dest, lslot):
        kn = moe_ops.kernels()
        W, r = arena.world, arena.rank
        t, h = x.shape
        k = dest.shape[1]
        dev = x.device
        _mark("start")
        onehot, pos_in_d, asg_pos, asg_to = _dispatch_tables(dest, W)
        rows_to = onehot.sum(0)
        # ---- 3) counts all-gather
        row = torch.stack([rows_to, asg_to], 1).to(torch.int32).contiguous()  # [W, 2]
        _mark("fwd.tables")
        kn.p2p_allgather_words(row, arena.peers, arena.layout["counts"], r)
        arena.barrier()
        _mark("fwd.counts_exchange")
        C = arena.view("counts", (W, W, 2), torch.int32).clone()  # [src, dst, (rows, asg)]
        # ---- 4) where my rows / assignments land at each destination
        excl = torch.cumsum(C, 0) - C  # prefix over sources
        row_off = excl[r, :, 0]  # [W]
        asg_off = excl[r, :, 1]
        # (torch.cumsum promotes int32 to int64: index tables are cast back to int32 for the kernels)
        dst_row = torch.where(onehot > 0, row_off[None, :] + pos_in_d,
                              torch.full_like(pos_in_d, -1)).to(torch.int32)  # [T, W]
        dst_asg = (asg_off[dest] + asg_pos).to(torch.int32)  # [T, k]
        # ---- 5) rows + metadata out
        tok = torch.arange(t, device=dev, dtype=torch.int32)
        src_rows = tok[:, None].expand(t, W).reshape(-1).contiguous()
        ranks = torch.arange(W, device=dev, dtype=torch.int32)[None, :].expand(t, W).reshape(-1).contiguous()
        dflat = dst_row.reshape(-1).contiguous()
        kn.p2p_put_rows(x.contiguous(), src_rows, ranks, dflat, None, t * W, arena.peers, arena.layout["recv_rows"], h)
        recv_row_at_dest = dst_row.gather(1, dest)  # [T, k] receive row of each assignment at its destination
        meta = torch.stack([recv_row_at_dest.to(torch.int32), lslot.to(torch.int32),
                            w.detach().float().contiguous().view(torch.int32),
                            torch.arange(t * k, device=dev, dtype=torch.int32).view(t, k)], 2)  # [T, k, 4]
        d32 = dest.to(torch.int32)
        for c in range(4):
            kn.p2p_put_words(meta[:, :, c].contiguous().reshape(-1), d32.reshape(-1).contiguous(),
                             (dst_asg * 4 + c).reshape(-1).to(torch.int32).contiguous(), None, t * k, arena.peers,
                             arena.layout["recv_meta"])
        _mark("fwd.offsets_and_puts")
        arena.barrier()
        _mark("fwd.dispatch_barrier")
        # ---- 6) receiver side
        n_rows = C[:, r, 0].sum()  # device scalars
        n_asg = C[:, r, 1].sum()
        R_cap = W * arena.tokens
        # expert work is sized for `asg_cap` received assignments (a multiple of the balanced
        # share); the largest count seen is kept on the device and checked once per step
        ep = blk.ep
        A_cap = ep.asg_cap(arena)
        torch.maximum(ep.max_recv, n_asg.reshape(1).to(torch.int32), out=ep.max_recv)
        recv_x = arena.view("recv_rows", (R_cap, h), torch.bfloat16)
        rmeta = arena.view("recv_meta", (R_cap * k, 4), torch.int32)[:A_cap]
        valid = torch.arange(A_cap, device=dev) < n_asg
        slots = torch.where(valid, rmeta[:, 1], torch.full_like(rmeta[:, 1], -1)).contiguous()
        rrow = torch.where(valid, rmeta[:, 0], torch.full_like(rmeta[:, 0], -1)).contiguous()
        rw = torch.where(valid, rmeta[:, 2].view(torch.float32), torch.zeros_like(rmeta[:, 2].view(torch.float32)))
        loc = _local_plan(blk, rrow, slots, rw.contiguous(), R_cap, k, arena.tokens * k)
        # return address of every received assignment's routing-weight gradient
        asg_from = C[:, r, 1]
        a_idx = torch.arange(A_cap, device=dev)
        src_a = torch.searchsorted(torch.cumsum(asg_from, 0), a_idx, right=True).clamp_max(W - 1)
        loc["asg_src_rank"] = torch.where(valid, src_a, torch.full_like(src_a, -1)).to(torch.int32).contiguous()
        loc["asg_src_idx"] = torch.where(valid, rmeta[:, 3], torch.full_like(rmeta[:, 3], -1)).contiguous()
        _mark("fwd.local_plan")
        xd = torch.empty(loc["cap"], h, device=dev, dtype=torch.bfloat16)
        kn.gather_rows(recv_x, loc["row_src"], loc["end"], xd)
        w1, w2 = blk.compute_weights()
        inter = w1.shape[1] // 2
        hbuf = torch.empty(loc["cap"], inter, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(loc["cap"], 2 * inter, device=dev, dtype=torch.bfloat16)
        kn.moe_fc1_swiglu(xd, w1, loc["offsets"], loc["row_scale"], hbuf, gu, loc["align"], None)
        yd = torch.empty(loc["cap"], h, device=dev, dtype=torch.bfloat16)
        kn.moe_grouped_gemm(hbuf, w2, loc["offsets"], yd, False, loc["align"])
        _mark("fwd.expert_gemms")
        partial = torch.empty(R_cap, h, device=dev, dtype=torch.bfloat16)
        kn.sum_rows(yd, loc["table"], partial)
        # ---- 7) partial sums back to the sources
        back_dst_rank, back_dst_row = _return_targets(C, r, R_cap, dev)
        kn.p2p_put_rows(partial, None, back_dst_rank, back_dst_row, n_rows.to(torch.int32).reshape(1), R_cap,
                        arena.peers, arena.layout["back_rows"], h)
        _mark("fwd.combine_puts")
        arena.barrier()
        _mark("fwd.combine_barrier")
        # ---- 8) sum per token
        send_base = torch.cumsum(C[r, :, 0], 0) - C[r, :, 0]  # my send-order base per destination
        back_pos = torch.where(onehot > 0, send_base[None, :] + pos_in_d, torch.full_like(pos_in_d, -1)).to(torch.int32)
        back = arena.view("back_rows", (R_cap, h), torch.bfloat16)
        y = torch.empty(t, h, device=dev, dtype=torch.bfloat16)
        kn.sum_rows(back, back_pos.contiguous(), y)
        _mark("fwd.token_sum")
        ctx.save_for_backward(xd, hbuf, gu, w1, w2, dst_row.contiguous(), back_pos.contiguous(), d32,
                              dst_asg.to(torch.int32), C)
        ctx.loc = loc
        ctx.blk, ctx.arena, ctx.shape = blk, arena, (t, h, k)
        return y

    @staticmethod
    def backward(ctx, dy):
        kn = moe_ops.kernels()
        xd, hbuf, gu, w1, w2, dst_row, back_pos, d32, dst_asg, C = ctx.saved_tensors
        loc, blk, arena = ctx.loc, ctx.blk, ctx.arena
        t, h, k = ctx.shape
        W, r = arena.world, arena.rank
        dev = dy.device
        R_cap = W * arena.tokens
        _mark("start")
        dy = dy.contiguous().to(torch.bfloat16)
        # combine backward: dy rows to the destinations (same positions as the forward dispatch)
        tok = torch.arange(t, device=dev, dtype=torch.int32)
        src_rows = tok[:, None].expand(t, W).reshape(-1).contiguous()
        ranks = torch.arange(W, device=dev, dtype=torch.int32)[None, :].expand(t, W).reshape(-1).contiguous()
        kn.p2p_put_rows(dy, src_rows, ranks, dst_row.reshape(-1).contiguous(), None, t * W, arena.peers,
                        arena.layout["recv_rows"], h)
        _mark("bwd.dy_puts")
        arena.barrier()
        _mark("bwd.dy_barrier")
        recv_dy = arena.view("recv_rows", (R_cap, h), torch.bfloat16)
        dyd = torch.empty(loc["cap"], h, device=dev, dtype=torch.bfloat16)
        kn.gather_rows(recv_dy, loc["row_src"], loc["end"], dyd)
        dgu = torch.empty_like(gu)
        dscale = torch.zeros(loc["cap"], device=dev, dtype=torch.float32)
        kn.moe_fc2_dgrad_dswiglu(dyd, w2, loc["offsets"], gu, loc["row_scale"], dgu, dscale, loc["align"])
        dxd = torch.empty_like(xd)
        kn.moe_grouped_gemm(dgu, w1, loc["offsets"], dxd, True, loc["align"])
        if blk.down_proj.requires_grad:
            kn.moe_wgrad(dyd, hbuf, loc["offsets"], *moe_ops.wgrad_target(blk.down_proj), None)
        if blk.gate_up_proj.requires_grad:
            kn.moe_wgrad(dgu, xd, loc["offsets"], *moe_ops.wgrad_target(blk.gate_up_proj), None)
        _mark("bwd.expert_gemms")
        # dispatch backward: per received row, sum over its assignments -> back to the source
        dpart = torch.empty(R_cap, h, device=dev, dtype=torch.bfloat16)
        kn.sum_rows(dxd, loc["table"], dpart)
        n_rows = C[:, r, 0].sum().to(torch.int32).reshape(1)
        back_dst_rank, back_dst_row = _return_targets(C, r, R_cap, dev)
        kn.p2p_put_rows(dpart, None, back_dst_rank, back_dst_row, n_rows, R_cap, arena.peers,
                        arena.layout["back_rows"], h)
        # routing-weight gradients: per received assignment -> source flat (t*k + j) index
        dw_asg = kn.gather_scalar(dscale, loc["row_of"])  # [A_cap]
        n_asg = torch.clamp(C[:, r, 1].sum(), max=dw_asg.numel()).to(torch.int32).reshape(1)
        kn.p2p_put_words(dw_asg.contiguous().view(torch.int32), loc["asg_src_rank"], loc["asg_src_idx"], n_asg,
                         dw_asg.numel(), arena.peers, arena.layout["back_words"])
        _mark("bwd.back_puts")
        arena.barrier()
        _mark("bwd.back_barrier")
        back = arena.view("back_rows", (R_cap, h), torch.bfloat16)
        dx = torch.empty(t, h, device=dev, dtype=torch.bfloat16)
        kn.sum_rows(back, back_pos, dx)
        dw = arena.view("back_words", (R_cap * k,), torch.float32)[: t * k].clone().view(t, k)
        _mark("bwd.token_sum")
        rs = getattr(blk.ep, "replica_sync", None)
        if rs is not None:  # this layer's expert gradients are final: reduce replicas on the side stream
            rs.layer_ready(blk)
        return dx, dw, None, None, None, None


def _return_targets(C: torch.Tensor, r: int, R_cap: int, dev):
    """For every received row: (source rank, position in the source's send order)."""
    recv_counts = C[:, r, 0]  # rows from each source
    base = torch.cumsum(recv_counts, 0) - recv_counts
    R = torch.arange(R_cap, device=dev)
    src = torch.searchsorted(torch.cumsum(recv_counts, 0), R, right=True).clamp_max(C.shape[0] - 1)
    # source's send base for destination r
    src_send_base = (torch.cumsum(C[:, :, 0], 1) - C[:, :, 0])[:, r]
    pos = src_send_base[src] + (R - base[src])
    valid = R < recv_counts.sum()
    return (torch.where(valid, src, torch.full_like(src, -1)).to(torch.int32).contiguous(),
            torch.where(valid, pos, torch.full_like(pos, -1)).to(torch.int32).contiguous())


def _local_plan(blk, rrow, slots, rw, R_cap, k, expected_asg):
    """Expert plan over received assignments (invalid ones carry slot -1)."""
    kn = moe_ops.kernels()
    A = slots.shape[0]
    spr = blk.num_local_slots
    # alignment from the expected (balanced) share of assignments, not the capacity A
    align = moe_ops.segment_align(expected_asg, spr)
    cap = moe_ops.capacity_rows(A, 1, spr, align)
    offsets, counts, row_of, row_token, row_scale = kn.moe_plan(slots.view(A, 1), None, rw, spr, cap, align)
    end = offsets[spr:]
    dev = slots.device
    in_plan = torch.arange(cap, device=dev, dtype=torch.int32) < end
    rt = torch.where(in_plan & (row_token >= 0), row_token, torch.full_like(row_token, -1))
    row_src = torch.where(rt >= 0, rrow[rt.clamp_min(0).long()], rt).contiguous()
    # received row -> its dispatched rows (<= k per row), for pre-reduction
    valid = slots >= 0
    rr = torch.where(valid, rrow, torch.full_like(rrow, R_cap)).long()
    cnt = torch.zeros(R_cap + 2, dtype=torch.long, device=dev)
    cnt.index_add_(0, rr + 1, torch.ones_like(rr))
    first = torch.cumsum(cnt, 0)
    pos = (torch.arange(A, device=dev) - first[rr]).clamp(0, k - 1)
    table = torch.full((R_cap + 1, k), -1, dtype=torch.int32, device=dev)
    table[rr, pos] = torch.where(valid, row_of, torch.full_like(row_of, -1))
    table = table[:R_cap].contiguous()
    return {"cap": cap, "offsets": offsets, "end": end, "row_of": row_of, "row_src": row_src,
            "row_scale": row_scale, "table": table, "align": align}


class EPCapacityExceeded(RuntimeError):
    """A rank received more expert assignments than its buffers hold in this step."""


class P2PExpertParallel:
    """Drop-in replacement of :class:`ExpertParallel` on CUDA with the peer-memory transport.

    Expert buffers are sized for ``capacity_factor`` times the balanced share
    of received assignments (at most all of them), so no host read of the
    received count is needed per layer.  The largest count of the step is
    checked once per step (:meth:`check_capacity`, before the optimizer); on
    overflow the trainer grows the factor and recomputes the step.
    """

    def __init__(self, group=None, capture_routes: bool = False, capacity_factor: float = 2.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.capture_routes = capture_routes
        self.capacity_factor = capacity_factor
        self.arena: SymmetricArena | None = None
        self.max_recv: torch.Tensor | None = None
        self.replica_sync = None  # p2p_sync.ReplicaGradSync, set by the trainer
        from .ep import ExpertParallel

        self._router = ExpertParallel._route.__get__(self)

    def _arena_for(self, t, k, h, device):
        if self.arena is None or not self.arena.fits(t, k, h):
            self.arena = SymmetricArena(self.group, self.world, self.rank, t, k, h, device)
        if self.max_recv is None or self.max_recv.device != device:
            self.max_recv = torch.zeros(1, dtype=torch.int32, device=device)
        return self.arena

    def asg_cap(self, arena: SymmetricArena) -> int:
        """Received assignments the expert buffers are sized for (at most everything)."""
        full = arena.world * arena.tokens * arena.k
        return min(full, int(math.ceil(self.capacity_factor * arena.tokens * arena.k)))

    def check_capacity(self) -> None:
        """Raise :class:`EPCapacityExceeded` if any rank overflowed since the last check (one host read)."""
        if self.max_recv is None or self.arena is None:
            return
        worst = self.max_recv.clone()
        dist.all_reduce(worst, op=dist.ReduceOp.MAX, group=self.group)
        self.max_recv.zero_()
        cap = self.asg_cap(self.arena)
        if int(worst.item()) > cap:
            raise EPCapacityExceeded(f"received {int(worst.item())} expert assignments, capacity {cap} "
                                     f"(capacity_factor {self.capacity_factor})")

    def moe_forward(self, blk, x, bias, aux_coef):
        t, h = x.shape
        k = blk.cfg.num_experts_per_tok
        w, idx, aux = self._router(blk, x, bias, aux_coef)
        dest_tab, slot_tab = blk.placement.route_tables(x.device)
        dest = dest_tab.long()[idx]
        lslot = slot_tab.long()[idx]
        arena = self._arena_for(t, k, h, x.device)
        y = _P2PMoE.apply(x, w, blk, arena, dest, lslot)
        return y, aux, idx
