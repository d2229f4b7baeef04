"""Route capture for the planner.

After a training step every MoE block holds the logical top-k routes of its
last forward (``blk.last_route``, [T, k]).  ``RouteRecorder.record_step``
gathers them from every EP rank (one ``all_gather_object`` per step for all
layers; capture steps only) and rank 0 writes one
``hiermoe-local-route-bundle-v1`` file per layer and step.  With micro-batches
the routes of all micro-batches of the step are concatenated.

Reference parity: route capture of
veomni/distributed/moe/hiermoe/expert_swap.py:10616-10682.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..placemoe.routes import write_route_bundle


class RouteRecorder:
    def __init__(self, model, root: str, group=None):
        self.model = model
        self.root = root
        self.group = group
        self._pending: dict[int, list[torch.Tensor]] = {}
        self._stream = None  # CUDA stream that carries queued route copies
        self.enabled = False
        for blk in model.moe_blocks():
            blk.route_sink = self

    def collect(self, blk, route: torch.Tensor) -> None:
        """Queue a copy of one layer's routes.  On CUDA the copy goes to pinned host memory without a
        host synchronisation (in stream order, so later kernels may reuse ``route``); the host reads
        it in :meth:`record_step`, once per step, after one stream synchronisation."""
        if not self.enabled:
            return
        r = route.detach()
        if r.is_cuda:
            host = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
            host.copy_(r, non_blocking=True)
            self._stream = torch.cuda.current_stream(r.device)
            self._pending.setdefault(blk.layer_idx, []).append(host)
        else:
            self._pending.setdefault(blk.layer_idx, []).append(r.to(torch.long))

    def record_step(self, step: int) -> list[str]:
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        if self._stream is not None:
            self._stream.synchronize()  # the queued device-to-host route copies have landed
            self._stream = None
        local = {}
        for blk in self.model.moe_blocks():
            mine = [r.to(torch.long) for r in self._pending.get(blk.layer_idx, [])]
            local[blk.layer_idx] = (torch.cat(mine, 0) if mine
                                    else torch.zeros(0, blk.cfg.num_experts_per_tok, dtype=torch.long))
        # one collective per step for all layers
        if world > 1:
            gathered = [None] * world
            dist.all_gather_object(gathered, local, group=self.group)
        else:
            gathered = [local]
        paths = []
        if rank == 0:
            for blk in self.model.moe_blocks():
                per_rank = [g[blk.layer_idx] for g in gathered]
                paths.append(str(write_route_bundle(self.root, step, blk.layer_idx, per_rank)))
        self._pending.clear()
        return paths
