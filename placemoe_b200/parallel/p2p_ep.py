"""Expert parallelism over NVLink peer memory with fused dispatch / combine kernels.

Each EP group owns one symmetric arena (``torch.distributed._symmetric_memory``)
mapped into every peer.  One MoE layer on rank r (T tokens, top-k, S local
slots) runs four launches forward and six backward, none of them a torch op
on index tables:

forward
  1. ``ep_dispatch`` (one cooperative kernel): bucket counts -> count rows to
     every peer -> barrier -> every rank derives each destination's aligned
     expert segments and its own rows' places in them -> each token row is
     stored once per destination GPU straight into that GPU's expert-
     contiguous input slab (the layer's slab), with a 16-byte record per
     assignment -> barrier -> local copies for a token's other assignments on
     the same GPU, routing weights extracted;
  2. grouped fc1 GEMM with the SwiGLU and routing-weight epilogue, reading
     the slab in place;  3. grouped fc2 GEMM;
  4. ``ep_combine``: every (token, GPU) primary's rows are pre-reduced in fp32
     and stored into the source's return rows -> barrier -> token sums.
backward
  ``ep_scatter`` (dy once per (token, GPU), local copies), fc2 dgrad +
  dSwiGLU, fc1 dgrad, then ``ep_combine`` of the data gradients (with the
  routing-weight gradients riding along) while the two grouped weight-gradient
  GEMMs run on a side stream: they do not feed dx, so their tensor-core work
  overlaps the combine's NVLink traffic.  The output-gradient buffer is double
  buffered by layer parity, and a layer's combine waits for the previous
  layer's weight gradients, which keeps a peer's scatter from refilling a
  buffer that a weight gradient still reads.

The receive slab of every layer lives until the layer's backward (the fc1
weight gradient reads it), so the arena holds one slab per MoE layer: the
same bytes the dispatched rows occupied as saved activations before, now
written by the senders instead of gathered by the receiver.

Capacity: a slab holds ``capacity_factor`` x the balanced share of received
assignments plus segment padding.  The largest row count of the step is
kept in the device status block and checked once per step
(:meth:`P2PExpertParallel.check_capacity`); on overflow the trainer grows the
factor and recomputes the step, and rows beyond the slab are dropped, never
written out of bounds.

Every wait is bounded (wall-clock budget, sticky error status read by the
trainer every step).

Reference parity: rank_dedup_dispatch / rank_dedup_combine of
veomni/distributed/moe/hiermoe/all_to_all.py:2029-2264, :2539-2564 with the
NCCL all-to-all data plane replaced by peer stores issued from the kernels.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops import moe as moe_ops
from ..ops import p2p_status

BARRIER_TIMEOUT_S = 20.0


class PhaseTimer:
    """CUDA-event time of every EP communication kernel (set ``p2p_ep.TIMER = PhaseTimer()``).

    ``phases()`` sums the elapsed time per kernel name; these kernels run on
    the compute stream, so their total is the exposed all-to-all time.
    """

    def __init__(self):
        self.spans: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def span(self, name: str):
        timer = self

        class _Span:
            def __enter__(self):
                self.a = torch.cuda.Event(enable_timing=True)
                self.b = torch.cuda.Event(enable_timing=True)
                self.a.record()

            def __exit__(self, *exc):
                self.b.record()
                timer.spans.append((name, self.a, self.b))

        return _Span()

    def phases(self) -> dict[str, float]:
        out: dict[str, float] = {}
        for name, a, b in self.spans:
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def total_ms(self) -> float:
        return sum(self.phases().values())


TIMER: PhaseTimer | None = None


class _NoSpan:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


def _span(name: str):
    return TIMER.span(name) if TIMER is not None else _NoSpan()


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class EpArena:
    """Symmetric arena of one EP group: barrier flags, count matrix, return rows, per-layer slabs."""

    def __init__(self, group, world: int, rank: int, tokens: int, k: int, hidden: int, slots: int, layers: int,
                 capacity_factor: float, device):
        kn = moe_ops.kernels()
        self.group, self.world, self.rank = group, world, rank
        self.tokens, self.k, self.hidden, self.slots, self.layers = tokens, k, hidden, slots, layers
        self.capacity_factor = capacity_factor
        self.device = torch.device(device)
        full = world * tokens * k
        self.asg_cap = min(full, int(math.ceil(capacity_factor * tokens * k)))
        # alignment from the balanced share of assignments per slot
        self.align = moe_ops.segment_align(tokens * k, slots)
        self.cap = _align(self.asg_cap + slots * (self.align - 1), self.align)
        self.kpad = _align(k, 4)
        lay = {}
        off = 0

        def region(name, nbytes):
            nonlocal off
            lay[name] = off
            off += _align(nbytes)

        region("flags", 64 * 4)
        region("counts", 2 * world * world * slots * 4)
        region("back", tokens * world * hidden * 2)
        region("dw", tokens * k * 4)
        region("dy", self.cap * hidden * 2)  # output gradients of even layers
        region("dy1", self.cap * hidden * 2)  # odd layers: a layer's weight gradient may still read its
        # dy rows while the next layer's scatter fills the other buffer
        self.slab_off = []
        for _ in range(layers):
            x0 = off
            region("x", self.cap * hidden * 2)
            m0 = off
            region("meta", self.cap * 16)
            t0 = off
            region("tab", self.cap * self.kpad * 4)
            p0 = off
            region("prim", (self.cap + 1) * 4)  # primary rows of this GPU (count, then positions)
            self.slab_off.append((x0, m0, t0, p0))
        del lay["x"], lay["meta"], lay["tab"], lay["prim"]
        self.layout = lay
        self.nbytes = off
        if world > 1:
            import torch.distributed._symmetric_memory as symm_mem

            self.buf = symm_mem.empty(off, dtype=torch.uint8, device=self.device)
            self.buf[: lay["dy"]].zero_()
            gname = group.group_name if group is not None else dist.group.WORLD.group_name
            handle = symm_mem.rendezvous(self.buf, gname)
            ptrs = [int(p) for p in handle.buffer_ptrs]
        else:  # one rank: a plain allocation, the peer table holds only itself
            self.buf = torch.zeros(off, dtype=torch.uint8, device=self.device)
            ptrs = [self.buf.data_ptr()]
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.scratch = torch.zeros(int(kn.ep_scratch_ints(world, slots)), dtype=torch.int32, device=self.device)
        self.status = p2p_status(self.device)
        self.epoch = 0
        self.parity = 0
        if world > 1:
            dist.barrier(group=group)

    def fits(self, tokens: int, k: int, hidden: int, slots: int, layers: int, capacity_factor: float) -> bool:
        return (tokens <= self.tokens and k == self.k and hidden == self.hidden and slots == self.slots
                and layers <= self.layers and capacity_factor <= self.capacity_factor)

    def geo(self, slab: int, toggle: bool = False) -> list[int]:
        if toggle:
            self.parity ^= 1
        x0, m0, t0, p0 = self.slab_off[slab]
        L = self.layout
        dy = L["dy1"] if slab % 2 else L["dy"]
        return [self.world, self.rank, self.slots, self.k, self.hidden, self.tokens, self.cap, self.align, self.kpad,
                self.parity, L["flags"], L["counts"], x0, m0, t0, L["back"], L["dw"], dy, p0]

    def epochs(self, n: int) -> int:
        """First epoch of a launch that runs ``n`` peer barriers."""
        first = self.epoch + 1
        self.epoch += n
        return first

    def x_view(self, slab: int) -> torch.Tensor:
        x0 = self.slab_off[slab][0]
        return self.buf[x0: x0 + self.cap * self.hidden * 2].view(torch.bfloat16).view(self.cap, self.hidden)

    def dy_view(self, slab: int = 0) -> torch.Tensor:
        o = self.layout["dy1"] if slab % 2 else self.layout["dy"]
        return self.buf[o: o + self.cap * self.hidden * 2].view(torch.bfloat16).view(self.cap, self.hidden)


class _FusedEPMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, idx, blk, arena: EpArena, slab: int):
        kn = moe_ops.kernels()
        t, h = x.shape
        k = idx.shape[1]
        dev = x.device
        S, cap = arena.slots, arena.cap
        x = x.contiguous()
        dest_tab, slot_tab = blk.placement.route_tables(dev)
        pos = torch.empty(t, k, dtype=torch.int32, device=dev)
        dst = torch.empty(t, k, dtype=torch.int32, device=dev)
        offsets = torch.empty(S + 1, dtype=torch.int32, device=dev)
        row_scale = torch.empty(cap, dtype=torch.float32, device=dev)
        with _span("dispatch"):
            kn.ep_dispatch(x, idx, w.detach().float().contiguous(), dest_tab, slot_tab, arena.peers,
                           arena.geo(slab, toggle=True), arena.scratch, arena.status, arena.epochs(2),
                           BARRIER_TIMEOUT_S, pos, dst, offsets, row_scale)
        xd = arena.x_view(slab)
        w1, w2 = blk.compute_weights()
        inter = w1.shape[1] // 2
        hbuf = torch.empty(cap, inter, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(cap, 2 * inter, device=dev, dtype=torch.bfloat16)
        kn.moe_fc1_swiglu(xd, w1, offsets, row_scale, hbuf, gu, arena.align, None)
        yd = torch.empty(cap, h, device=dev, dtype=torch.bfloat16)
        kn.moe_grouped_gemm(hbuf, w2, offsets, yd, False, arena.align)
        y = torch.empty(t, h, device=dev, dtype=torch.bfloat16)
        with _span("combine"):
            kn.ep_combine(yd, None, pos, dst, offsets, arena.peers, arena.geo(slab), arena.scratch, arena.status,
                          arena.epochs(1), BARRIER_TIMEOUT_S, y, None)
        ctx.save_for_backward(hbuf, gu, w1, w2, pos, dst, offsets, row_scale)
        ctx.blk, ctx.arena, ctx.slab = blk, arena, slab
        return y

    @staticmethod
    def backward(ctx, dy):
        kn = moe_ops.kernels()
        hbuf, gu, w1, w2, pos, dst, offsets, row_scale = ctx.saved_tensors
        blk, arena, slab = ctx.blk, ctx.arena, ctx.slab
        t, k = pos.shape
        dev = dy.device
        cap = arena.cap
        dy = dy.contiguous().to(torch.bfloat16)
        with _span("scatter"):
            kn.ep_scatter(dy, pos, dst, offsets, arena.peers, arena.geo(slab), arena.scratch, arena.status,
                          arena.epochs(1), BARRIER_TIMEOUT_S)
        dyd = arena.dy_view(slab)
        xd = arena.x_view(slab)
        dgu = torch.empty_like(gu)
        dscale = torch.zeros(cap, device=dev, dtype=torch.float32)
        kn.moe_fc2_dgrad_dswiglu(dyd, w2, offsets, gu, row_scale, dgu, dscale, arena.align)
        dxd = torch.empty(cap, arena.hidden, device=dev, dtype=torch.bfloat16)
        kn.moe_grouped_gemm(dgu, w1, offsets, dxd, True, arena.align)
        ep = blk.ep
        # The weight gradients do not feed dx: they run on the weight-gradient stream while the combine
        # moves the data gradients over NVLink (the two kernels fit on an SM together).  Before this
        # layer's combine, the stream also waits for the previous MoE layer's weight gradients: a peer
        # can only start refilling that layer's dy buffer (two layers on) after passing this barrier.
        done = ep.wgrad_async(blk, dyd, hbuf, dgu, xd, offsets)
        ep.wait_previous_wgrad()
        dx = torch.empty(t, arena.hidden, device=dev, dtype=torch.bfloat16)
        dw = torch.empty(t, k, device=dev, dtype=torch.float32)
        with _span("combine_bwd"):
            kn.ep_combine(dxd, dscale, pos, dst, offsets, arena.peers, arena.geo(slab), arena.scratch, arena.status,
                          arena.epochs(1), BARRIER_TIMEOUT_S, dx, dw)
        ep.previous_wgrad = done
        rs = getattr(ep, "replica_sync", None)
        if rs is not None:  # this layer's expert gradients are final once `done` fires: reduce replicas
            rs.layer_ready(blk, after=done)
        return dx, dw, None, None, None, None


class EPCapacityExceeded(RuntimeError):
    """A rank received more expert assignments than its buffers hold in this step."""


class P2PExpertParallel:
    """Expert parallelism on CUDA with the fused peer-memory dispatch / combine kernels.

    ``num_layers`` (set by :func:`parallelize_model`) sizes the arena with one
    receive slab per MoE layer; ``blk.ep_slab`` is the layer's slab.
    """

    def __init__(self, group=None, capture_routes: bool = False, capacity_factor: float = 2.0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.capture_routes = capture_routes
        self.capacity_factor = capacity_factor
        self.num_layers = 1
        self.arena: EpArena | None = None
        self.replica_sync = None  # p2p_sync.ReplicaGradSync, set by the trainer
        self.wgrad_stream: torch.cuda.Stream | None = None
        self.pending_wgrad: list = []
        self.previous_wgrad = None
        from .ep import ExpertParallel

        self._router = ExpertParallel._route.__get__(self)

    # ------------------------------------------------------------ weight gradients on a side stream
    def wgrad_async(self, blk, dyd, hbuf, dgu, xd, offsets) -> torch.cuda.Event:
        """Launch the layer's two expert weight-gradient GEMMs on the weight-gradient stream, ordered after
        the work issued so far on the current stream; returns the event that marks their end."""
        cur = torch.cuda.current_stream(dyd.device)
        if self.wgrad_stream is None or self.wgrad_stream.device != dyd.device:
            self.wgrad_stream = torch.cuda.Stream(device=dyd.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        kn = moe_ops.kernels()
        with torch.cuda.stream(self.wgrad_stream):
            self.wgrad_stream.wait_event(ready)
            if blk.down_proj.requires_grad:
                kn.moe_wgrad(dyd, hbuf, offsets, *moe_ops.wgrad_target(blk.down_proj), None)
            if blk.gate_up_proj.requires_grad:
                kn.moe_wgrad(dgu, xd, offsets, *moe_ops.wgrad_target(blk.gate_up_proj), None)
            done = torch.cuda.Event()
            done.record(self.wgrad_stream)
        for t in (hbuf, dgu, offsets):  # allocated on the current stream, read on the side stream
            t.record_stream(self.wgrad_stream)
        self.pending_wgrad.append(done)
        return done

    def wait_previous_wgrad(self) -> None:
        if self.previous_wgrad is not None:
            torch.cuda.current_stream().wait_event(self.previous_wgrad)

    def wait_wgrads(self) -> None:
        """Make the current stream wait for every launched weight gradient (before the optimizer)."""
        cur = torch.cuda.current_stream()
        for ev in self.pending_wgrad:
            cur.wait_event(ev)
        self.pending_wgrad.clear()
        self.previous_wgrad = None

    def _arena_for(self, t, k, h, slots, device) -> EpArena:
        layers = max(1, self.num_layers)
        if self.arena is None or not self.arena.fits(t, k, h, slots, layers, self.capacity_factor):
            tokens = max(t, self.arena.tokens if self.arena is not None else 0)
            self.arena = None
            torch.cuda.current_stream(device).synchronize()
            # the symmetric arena comes from the driver, not from torch's cache: return cached blocks first
            torch.cuda.empty_cache()
            self.arena = EpArena(self.group, self.world, self.rank, tokens, k, h, slots, layers,
                                 self.capacity_factor, device)
        return self.arena

    @property
    def max_recv(self):
        return None if self.arena is None else self.arena.status[2:3]

    def check_capacity(self) -> None:
        """Raise :class:`EPCapacityExceeded` if any rank overflowed since the last check (one host read).

        ``last_overflow_rows`` keeps the largest row count seen, so the caller can size the next
        arena for what the step needed (:meth:`grow_capacity`) instead of blindly doubling it."""
        if self.arena is None:
            return
        worst = self.arena.status[2:3].clone()
        if self.world > 1:
            dist.all_reduce(worst, op=dist.ReduceOp.MAX, group=self.group)
        self.arena.status[2].zero_()
        rows = int(worst.item())
        if rows > self.arena.cap:
            self.last_overflow_rows = rows
            raise EPCapacityExceeded(f"received {rows} expert rows, slab holds {self.arena.cap} "
                                     f"(capacity_factor {self.capacity_factor})")

    def grow_capacity(self, margin: float = 1.15) -> float:
        """New capacity factor after an overflow: the rows the step needed plus ``margin``, at least a quarter
        more than before, at most the world size (every assignment of every source)."""
        a = self.arena
        rows = getattr(self, "last_overflow_rows", 0)
        need = (rows - a.slots * (a.align - 1)) / float(a.tokens * a.k) if a is not None and rows else 0.0
        self.capacity_factor = min(float(self.world), max(self.capacity_factor * 1.25, need * margin))
        return self.capacity_factor

    def moe_forward(self, blk, x, bias, aux_coef):
        t, h = x.shape
        k = blk.cfg.num_experts_per_tok
        w, idx, aux = self._router(blk, x, bias, aux_coef)
        if self.pending_wgrad:  # a receive slab may still be read by a weight gradient of the last backward
            self.wait_wgrads()
        arena = self._arena_for(t, k, h, blk.num_local_slots, x.device)
        slab = getattr(blk, "ep_slab", 0)
        y = _FusedEPMoE.apply(x, w, idx.to(torch.int32).contiguous(), blk, arena, slab)
        return y, aux, idx
