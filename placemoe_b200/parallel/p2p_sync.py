"""Bulk peer copies over NVLink: replica-gradient reduction and expert-state migration.

One growable symmetric buffer per process group (``PeerExchange``), mapped
into every peer, with its own barrier flags.  Two users:

* **Replica-gradient reduction.**  After the last micro-batch's backward of an
  MoE layer, every rank stages the fp32 gradients of its replicated expert
  slots into its buffer, a device barrier publishes them, and each copy's
  gradient is overwritten with the sum of all copies read straight from the
  peers (``p2p_sum_f32``), then a second barrier frees the buffer.  It runs
  on a side stream ordered after the layer's weight-gradient GEMMs, so it
  overlaps the same layer's attention backward on the main stream; the
  optimizer waits for it.
* **Expert-state migration.**  Source ranks stage the packed state of each
  outgoing slot (fp32 weights plus both AdamW moments); destinations pull it
  with ``p2p_pull``.  Offsets follow the globally ordered transfer list, so
  every rank computes them without exchanging metadata.

Every wait is a bounded device barrier (``p2p_barrier``): a peer that never
arrives makes the kernel record an error the host raises.

Reference parity: the replica-gradient schedules of
veomni/distributed/moe/hiermoe/expert_swap.py:6931-7107 (pairwise / owner-star
``batch_isend_irecv``, hidden mode overlapped with attention backward) and the
state migration transport of expert_swap.py:1358-1542.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import moe as moe_ops
from ..ops import p2p_status

FLAGS_BYTES = 256
BARRIER_TIMEOUT_S = 20.0


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerExchange:
    """A symmetric buffer (flags + data) for bulk peer copies within one process group."""

    def __init__(self, group, device, nbytes: int = 64 << 20):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.epoch = 0
        self.capacity = 0
        self.buf = None
        self.peers = None
        self._alloc(nbytes)

    def _alloc(self, nbytes: int) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        nbytes = _align(nbytes, 1 << 20)
        self.buf = None
        self.buf = symm_mem.empty(FLAGS_BYTES + nbytes, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        gname = self.group.group_name if self.group is not None else dist.group.WORLD.group_name
        handle = symm_mem.rendezvous(self.buf, gname)
        self.peers = torch.tensor([int(p) for p in handle.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.capacity = nbytes
        self.epoch = 0
        dist.barrier(group=self.group)

    def ensure(self, nbytes: int) -> None:
        """Grow to hold ``nbytes`` (collective: every rank passes the same size)."""
        if nbytes > self.capacity:
            torch.cuda.current_stream(self.device).synchronize()
            self._alloc(max(nbytes, 2 * self.capacity))

    def data(self, dtype=torch.float32) -> torch.Tensor:
        return self.buf[FLAGS_BYTES:].view(dtype)

    def barrier(self) -> None:
        """Bounded device barrier over every rank of the group (each rank must call it equally often)."""
        self.epoch += 1
        moe_ops.kernels().p2p_barrier(self.peers, 0, self.rank, self.epoch, BARRIER_TIMEOUT_S,
                                      p2p_status(self.device))


# ---------------------------------------------------------------- replica gradients
class _LayerSyncPlan:
    """Static per-layer schedule: which local slots to stage, which sums to compute.

    ``active`` is a property of the layer, the same on every rank: a layer with
    any replicated expert runs the exchange (and both of its barriers) on every
    rank of the group, also on a rank that holds none of the copies.  Barriers
    count arrivals over the whole group, so a rank that skipped one would leave
    its peers waiting.
    """

    def __init__(self, placement, device):
        spr = placement.slots_per_rank
        rank = placement.rank
        self.version = placement.version
        self.stage: list[int] = []
        self.sums: list[tuple[int, torch.Tensor, torch.Tensor]] = []  # (local slot, src ranks, src slot ids)
        groups = placement.replica_groups()
        self.active = len(groups) > 0
        for slots in groups:
            members = [(int(s) // spr, int(s) % spr) for s in slots.tolist()]
            mine = [j for (r, j) in members if r == rank]
            if not mine:
                continue
            self.stage.extend(mine)
            ranks = torch.tensor([r for r, _ in members], dtype=torch.int32, device=device)
            local = torch.tensor([j for _, j in members], dtype=torch.int64, device=device)
            for j in mine:
                self.sums.append((j, ranks, local))
        self.stage = sorted(set(self.stage))


class ReplicaGradSync:
    """Per-layer replica-gradient reduction over peer memory, overlapped with the backward."""

    def __init__(self, exchange: PeerExchange):
        self.x = exchange
        self.armed = False
        self.stream = torch.cuda.Stream(device=exchange.device)
        self._plans: dict[str, _LayerSyncPlan] = {}
        self._pending: list[torch.cuda.Event] = []
        self.layers_synced = 0

    def _plan(self, blk) -> _LayerSyncPlan:
        pl = blk.placement
        plan = self._plans.get(blk.layer_key)
        if plan is None or plan.version != pl.version:
            plan = _LayerSyncPlan(pl, self.x.device)
            self._plans[blk.layer_key] = plan
        return plan

    def layer_ready(self, blk, after: torch.cuda.Event | None = None) -> None:
        """Called at the end of a layer's expert backward (main stream); ``after``: the event that marks
        the end of the layer's weight gradients when they run on another stream."""
        if not self.armed:
            return
        plan = self._plan(blk)
        if not plan.active:  # no replicated expert in this layer on any rank
            return
        ready = after
        if ready is None:
            ready = torch.cuda.Event()
            ready.record()
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            sync_layer(blk, plan, self.x)
            done = torch.cuda.Event()
            done.record(self.stream)
        self._pending.append(done)
        self.layers_synced += 1

    def wait(self) -> None:
        """Make the current stream wait for every launched layer sync."""
        cur = torch.cuda.current_stream(self.x.device)
        for ev in self._pending:
            cur.wait_event(ev)
        self._pending.clear()


def sync_layer(blk, plan: _LayerSyncPlan, x: PeerExchange) -> None:
    kn = moe_ops.kernels()
    for p in (blk.gate_up_proj, blk.down_proj):
        g = moe_ops._accum_main_grad(p)
        per = g[0].numel()
        spr = g.shape[0]
        x.ensure(spr * per * 4)
        buf = x.data(torch.float32)[: spr * per].view(spr, per)
        for j in plan.stage:
            buf[j].copy_(g[j].reshape(-1))
        x.barrier()
        for j, ranks, local in plan.sums:
            kn.p2p_sum_f32(g[j].view(-1), x.peers, ranks, local * (per * 4) + FLAGS_BYTES)
        x.barrier()


# ---------------------------------------------------------------- migration
def p2p_transfer(x: PeerExchange, transfers, spr: int, rank: int, outgoing: dict, staging: dict) -> None:
    """Move packed slot states for ``transfers`` (global order) through the exchange buffer.

    ``outgoing[i]`` is this rank's packed state for transfer i (source here,
    destination elsewhere); ``staging[dst]`` receives transfer i's payload when
    the destination is here.  All payloads have the same size.
    """
    kn = moe_ops.kernels()
    remote = [(i, s, d) for i, (s, d) in enumerate(transfers) if s // spr != d // spr]
    if not remote:
        return
    nbytes = None
    for t in list(outgoing.values()) + list(staging.values()):
        nbytes = t.numel() * t.element_size()
        break
    if nbytes is None:  # this rank neither sends nor receives: size from any slot is unknown, use 0
        nbytes = 0
    # every rank must agree on the slot payload size and the buffer size
    size = torch.tensor([nbytes], dtype=torch.int64, device=x.device)
    dist.all_reduce(size, op=dist.ReduceOp.MAX, group=x.group)
    nbytes = int(size.item())
    per_src: dict[int, int] = {}
    offset: dict[int, int] = {}
    for i, s, _d in remote:
        r = s // spr
        offset[i] = per_src.get(r, 0) * nbytes
        per_src[r] = per_src.get(r, 0) + 1
    x.ensure(max(per_src.values()) * nbytes)
    data = x.data(torch.uint8)
    for i, s, _d in remote:
        if s // spr == rank:
            src = outgoing[i]
            data[offset[i]: offset[i] + nbytes].copy_(src.view(torch.uint8).reshape(-1))
    x.barrier()
    for i, s, d in remote:
        if d // spr == rank:
            kn.p2p_pull(staging[d].view(torch.uint8).reshape(-1), x.peers, s // spr, FLAGS_BYTES + offset[i])
    x.barrier()
