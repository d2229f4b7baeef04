"""Expert-state migration for full (L, M) installs at a step boundary.

For every physical slot whose logical expert changes, the new contents
(fp32 master weights of ``gate_up_proj`` and ``down_proj`` plus both AdamW
moments of each) are copied from a copy of that expert under the OLD layout:
a copy on the destination GPU first, else the old owner, else the lowest
slot holding it.  Every rank derives the same transfer list from the two
plans, so no metadata exchange is needed.

Consensus: before anything moves, one all-reduce checks that every rank installs the same plan
from the same current layout and holds per-slot state of the same layout (tensor count, sizes,
dtypes); otherwise every rank raises ``MigrationConsensusError`` and nothing changes (the
reference does this in its debug mode, expert_swap.py:1302-1392).

Atomicity: staging buffers are allocated first and every rank confirms (an
all-reduce of a status word) before any transfer is posted, so a local
failure aborts everywhere without leaving a peer waiting; transfers then land
in the staging buffers and the live tensors are written only after a second
agreement, so every rank ends on the old placement or every rank on the new.  Emptied slots are
zeroed.  bf16 compute copies of changed parameters are refreshed afterwards.

Transports: a peer-memory copy over NVLink when the trainer holds a peer
exchange buffer (``p2p_sync.p2p_transfer``: sources stage, destinations pull
with the ``p2p_pull`` kernel), else ``batch_isend_irecv`` in a globally
ordered schedule (NCCL or gloo).

Reference parity: veomni/distributed/moe/hiermoe/expert_swap.py:1358-1542
(_cover_grouped_slot_entries_atomic), :1580-1716 (optimizer state binding),
:10818-10918 (full install).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from ..placemoe.types import EMPTY_EXPERT, LayerPlan


def plan_transfers(old_layout: np.ndarray, old_owners: np.ndarray, new_layout: np.ndarray,
                   spr: int) -> list[tuple[int, int]]:
    """(source slot, destination slot) for every slot whose logical expert changes."""
    out = []
    for g in range(len(new_layout)):
        e = int(new_layout[g])
        if e == EMPTY_EXPERT or e == int(old_layout[g]):
            continue
        holders = np.flatnonzero(old_layout == e)
        if len(holders) == 0:
            raise ValueError(f"expert {e} has no copy under the old layout")
        same = holders[holders // spr == g // spr]
        if len(same):
            src = int(same[0])
        elif int(old_owners[e]) in holders:
            src = int(old_owners[e])
        else:
            src = int(holders[0])
        out.append((src, g))
    return out


def _slot_state(blk, opt, j: int) -> list[torch.Tensor]:
    """Parameter and optimizer-state rows of local slot j (AdamW moments or Muon momentum)."""
    from ..optim import state_tensors

    ts = []
    for p in (blk.gate_up_proj, blk.down_proj):
        ts.append(p.data[j])
        ts.extend(t[j] for _, t in state_tensors(opt, p))
    return ts


def _pack(ts: list[torch.Tensor]) -> torch.Tensor:
    return torch.cat([t.reshape(-1).float() for t in ts])


def allocate_staging(like: torch.Tensor) -> torch.Tensor:
    """Staging copy of one slot's packed state (a separate function so tests can inject failures)."""
    return like.clone()


def _agree(ok: bool, world: int, group) -> bool:
    status = torch.tensor([0 if ok else 1], dtype=torch.int64)
    if world > 1:
        if dist.get_backend(group) == "nccl":
            status = status.cuda()
        dist.all_reduce(status, group=group)
    return int(status.item()) == 0


class MigrationConsensusError(RuntimeError):
    """Ranks disagree on what a migration installs or moves; raised on every rank, nothing is changed."""


def _same_on_all_ranks(values: list[int], world: int, group) -> list[bool]:
    """Per value: did every rank pass the same integer?  (one MIN all-reduce of [v, -v])"""
    t = torch.tensor(values + [-v for v in values], dtype=torch.int64)
    if world > 1:
        if dist.get_backend(group) == "nccl":
            t = t.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    t = t.cpu().tolist()
    n = len(values)
    return [t[i] == -t[n + i] for i in range(n)]


def _digest(*arrays) -> int:
    """CRC-32 over the arrays' values (integers as int64, so equal plans hash equally whatever their dtype)."""
    import zlib

    h = 0
    for a in arrays:
        a = np.asarray(a)
        if a.dtype.kind in "iub" and a.dtype != np.uint8:
            a = a.astype(np.int64)
        h = zlib.crc32(np.ascontiguousarray(a).tobytes(), h)
    return h


def _payload_signature(blk, opt) -> int:
    """Layout of one slot's migrated state: tensor count, sizes and dtypes (identical on every rank
    unless one rank's optimizer holds different state)."""
    ts = _slot_state(blk, opt, 0)
    return _digest(np.array([len(ts)] + [t.numel() for t in ts], dtype=np.int64),
                   np.frombuffer(",".join(str(t.dtype) for t in ts).encode(), dtype=np.uint8))


def _unpack_into(buf: torch.Tensor, ts: list[torch.Tensor]) -> None:
    off = 0
    for t in ts:
        n = t.numel()
        t.copy_(buf[off: off + n].view_as(t))
        off += n


@torch.no_grad()
def migrate_layer(trainer, blk, new_plan: LayerPlan, group=None) -> int:
    """Install ``new_plan`` on ``blk`` with parameter + optimizer-state migration. Returns moved slots."""
    pl = blk.placement
    opt = trainer.optimizer
    for p in (blk.gate_up_proj, blk.down_proj):
        opt._state(p)
    spr = pl.slots_per_rank
    rank = pl.rank
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    old_layout, old_owners = pl.slot_to_logical.copy(), pl.owner_slots.copy()
    new_layout = np.asarray(new_plan.slot_to_logical)
    # 0) consensus: every rank installs the same plan from the same old layout and moves state of the
    #    same layout per slot; otherwise each rank would derive different transfers (mismatched
    #    send/recv pairs).  Checked before anything is allocated or sent, and raised on every rank.
    same_plan, same_old, same_payload = _same_on_all_ranks(
        [_digest(new_layout, np.asarray(new_plan.source_logical_to_physical), np.asarray(new_plan.owner_slots)),
         _digest(old_layout, old_owners), _payload_signature(blk, opt)], world, group)
    if not (same_plan and same_old):
        raise MigrationConsensusError(f"{blk.layer_key}: ranks disagree on the placement "
                                      f"({'new plan' if not same_plan else 'current layout'}); nothing moved")
    if not same_payload:
        raise MigrationConsensusError(f"{blk.layer_key}: asymmetric migration payload (per-slot parameter / "
                                      "optimizer-state layout differs between ranks); nothing moved")
    transfers = plan_transfers(old_layout, old_owners, new_layout, spr)
    # 1) preflight: every rank allocates its staging and send buffers; a failure anywhere
    #    aborts on every rank before any transfer is posted (nobody waits on a missing peer)
    staging: dict[int, torch.Tensor] = {}
    sends: list[tuple[int, torch.Tensor]] = []
    outgoing: dict[int, torch.Tensor] = {}  # transfer index -> packed state (remote destination)
    recvs: list[tuple[int, int]] = []
    try:
        for i, (src, dst) in enumerate(transfers):  # globally consistent order
            rs, rd = src // spr, dst // spr
            if rd == rank and rs == rank:
                staging[dst] = allocate_staging(_pack(_slot_state(blk, opt, src - rank * spr)))
            elif rs == rank:
                buf = allocate_staging(_pack(_slot_state(blk, opt, src - rank * spr)))
                sends.append((rd, buf))
                outgoing[i] = buf
            elif rd == rank:
                staging[dst] = allocate_staging(torch.empty_like(_pack(_slot_state(blk, opt, 0))))
                recvs.append((rs, dst))
        ok = True
    except Exception:
        ok = False
    if not _agree(ok, world, group):
        return 0  # every rank keeps the old placement
    # 2) transfers: a peer-memory copy kernel when the group has a peer exchange buffer,
    #    else send/recv in the same global order on every rank
    xchg = getattr(trainer, "peer_exchange", None)
    try:
        if xchg is not None and world > 1:
            from .p2p_sync import p2p_transfer

            p2p_transfer(xchg, transfers, spr, rank, outgoing, staging)
        else:
            ops = []
            si = 0
            for src, dst in transfers:
                rs, rd = src // spr, dst // spr
                if rs == rank and rd != rank:
                    ops.append(dist.P2POp(dist.isend, sends[si][1], rd, group=group))
                    si += 1
                elif rd == rank and rs != rank:
                    ops.append(dist.P2POp(dist.irecv, staging[dst], rs, group=group))
            if ops:
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
        ok = True
    except Exception:
        ok = False
    # 3) publish only when every rank's transfers completed
    if not _agree(ok, world, group):
        return 0
    moved = 0
    for dst, buf in staging.items():
        _unpack_into(buf, _slot_state(blk, opt, dst - rank * spr))
        moved += 1
    for j in range(spr):
        if new_layout[rank * spr + j] == EMPTY_EXPERT and old_layout[rank * spr + j] != EMPTY_EXPERT:
            for t in _slot_state(blk, opt, j):
                t.zero_()
    for p in (blk.gate_up_proj, blk.down_proj):
        p.view(-1)[:1].add_(0)  # version bump -> bf16 copy refreshed before the next forward
    pl.install_layout(new_plan)
    return moved
