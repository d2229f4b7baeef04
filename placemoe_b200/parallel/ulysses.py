"""Ulysses sequence parallelism: attention over whole sequences while every rank holds a sequence chunk.

A sequence-parallel (SP) group of P ranks shares the same batch of B
sequences of length S; rank r holds tokens [r*S/P, (r+1)*S/P) of each.
Everything per token (embeddings, norms, QKV / output projections, MoE, the
loss) runs on the local chunk.  Attention needs whole sequences, so q, k, v
are re-split from (local tokens, all heads) to (all tokens, H/P heads)
before it, and the output back after it:

    q, k, v [B*S/P, H*D]  --seq->heads-->  [B*S, H/P*D]  --attention-->  --heads->seq-->  [B*S/P, H*D]

CUDA: one cooperative kernel per exchange stores every (token, head group)
chunk straight into the owning rank's region of a symmetric buffer and
copies the received region out after a bounded barrier
(``csrc/kernels/sp_exchange.cu``).  CPU / gloo: ``all_to_all_single``, the
same data movement, kept as the oracle for the tests.

Gradients need no extra reduction: the backward of one exchange is the
other exchange, and the dense-gradient all-reduce over all ranks then sums
the per-chunk contributions.

Reference parity: veomni/distributed/sequence_parallel/ulysses.py:64-320
(all-to-all around attention) and comm.py:245-335 (group set-up).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import moe as moe_ops
from ..ops import p2p_status

BARRIER_TIMEOUT_S = 20.0
_FLAGS = 256


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class UlyssesGroup:
    """One SP group: its process group, this rank's position, and (CUDA) the exchange buffer."""

    def __init__(self, group, device, max_elements: int):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.capacity = 0
        self.epoch = 0
        self.parity = 0
        if self.device.type == "cuda":
            self.status = p2p_status(self.device)
            self.scratch = torch.zeros(2, dtype=torch.int32, device=self.device)
            self._alloc(max_elements)

    def _alloc(self, elements: int) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        region = _align(elements * 2)
        self.buf = None
        self.buf = symm_mem.empty(_FLAGS + 2 * region, dtype=torch.uint8, device=self.device)
        self.buf[:_FLAGS].zero_()
        gname = self.group.group_name if self.group is not None else dist.group.WORLD.group_name
        handle = symm_mem.rendezvous(self.buf, gname)
        self.peers = torch.tensor([int(p) for p in handle.buffer_ptrs], dtype=torch.int64, device=self.device)
        self.region = region
        self.capacity = elements
        self.epoch = 0
        dist.barrier(group=self.group)

    def exchange(self, x: torch.Tensor, to_heads: bool, batch: int, chunk: int, width: int) -> torch.Tensor:
        """seq->heads: x [batch*chunk, width] -> [batch*chunk*P, width/P]; heads->seq: the inverse
        (``width`` is always the sequence-side row width, all heads)."""
        p = self.size
        if p == 1:
            return x
        if not x.is_cuda:
            return _exchange_reference(x, to_heads, batch, chunk, width, p, self.group)
        n = batch * chunk * width
        if n > self.capacity:  # collective: every rank of the group makes the same calls
            torch.cuda.current_stream(self.device).synchronize()
            self._alloc(max(n, 2 * self.capacity))
        shape = (batch * chunk * p, width // p) if to_heads else (batch * chunk, width)
        out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
        self.epoch += 1
        self.parity ^= 1
        geo = [p, self.rank, batch, chunk, width, int(to_heads), 0, _FLAGS + self.parity * self.region]
        moe_ops.kernels().sp_exchange(x.to(torch.bfloat16).contiguous(), out, self.peers, geo, self.scratch,
                                      self.status, self.epoch, BARRIER_TIMEOUT_S)
        return out


def _exchange_reference(x, to_heads, batch, chunk, width, p, group):
    cp = width // p
    if to_heads:
        send = x.reshape(batch, chunk, p, cp).permute(2, 0, 1, 3).contiguous()  # [dest, b, i, cp]
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)  # [src, b, i, cp]
        return recv.permute(1, 0, 2, 3).reshape(batch * chunk * p, cp)  # rows: b, src chunk, i
    send = x.reshape(batch, p, chunk, cp).permute(1, 0, 2, 3).contiguous()  # [owner of positions, b, i, cp]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)  # [head group, b, i, cp]
    return recv.permute(1, 2, 0, 3).reshape(batch * chunk, width)


class _SeqToHeads(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, grp, batch, chunk, width):
        ctx.args = (grp, batch, chunk, width)
        return grp.exchange(x, True, batch, chunk, width)

    @staticmethod
    def backward(ctx, g):
        grp, batch, chunk, width = ctx.args
        return grp.exchange(g.contiguous(), False, batch, chunk, width), None, None, None, None


class _HeadsToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, grp, batch, chunk, width):
        ctx.args = (grp, batch, chunk, width)
        return grp.exchange(y, False, batch, chunk, width)

    @staticmethod
    def backward(ctx, g):
        grp, batch, chunk, width = ctx.args
        return grp.exchange(g.contiguous(), True, batch, chunk, width), None, None, None, None


def seq_to_heads(x: torch.Tensor, grp: UlyssesGroup, batch: int, chunk: int) -> torch.Tensor:
    """[batch*chunk, heads, D] on local tokens -> [batch*chunk*P, heads/P, D] on whole sequences."""
    t, h, d = x.shape
    if h % grp.size:
        raise ValueError(f"{h} heads do not split over {grp.size} sequence-parallel ranks")
    out = _SeqToHeads.apply(x.reshape(t, h * d), grp, batch, chunk, h * d)
    return out.view(t * grp.size, h // grp.size, d)


def heads_to_seq(y: torch.Tensor, grp: UlyssesGroup, batch: int, chunk: int) -> torch.Tensor:
    """[batch*chunk*P, heads/P, D] -> [batch*chunk, heads*D]."""
    tf, hp, d = y.shape
    return _HeadsToSeq.apply(y.reshape(tf, hp * d), grp, batch, chunk, hp * d * grp.size)


def build_ulysses_groups(size: int, device, max_elements: int) -> UlyssesGroup | None:
    """Consecutive ranks form SP groups of ``size``; every rank creates every group (collective)."""
    if size <= 1:
        return None
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % size:
        raise ValueError(f"ulysses_size {size} does not divide the world size {world}")
    mine = None
    for g in range(world // size):
        ranks = list(range(g * size, (g + 1) * size))
        pg = dist.new_group(ranks) if size < world else None
        if rank in ranks:
            mine = UlyssesGroup(pg, device, max_elements)
    return mine
