"""Route capture for the planner.

After a training step every MoE block holds the logical top-k routes of its
last forward (``blk.last_route``, [T, k]).  ``RouteRecorder.record_step``
gathers them from every EP rank (``all_gather_object``; this is off the hot
path and runs only on capture steps) and rank 0 writes one
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
        self.enabled = False
        for blk in model.moe_blocks():
            blk.route_sink = self

    def collect(self, blk, route: torch.Tensor) -> None:
        if self.enabled:
            self._pending.setdefault(blk.layer_idx, []).append(route.detach().to("cpu", torch.long))

    def record_step(self, step: int) -> list[str]:
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        paths = []
        for blk in self.model.moe_blocks():
            mine = self._pending.get(blk.layer_idx, [])
            local = torch.cat(mine, 0) if mine else torch.zeros(0, blk.cfg.num_experts_per_tok, dtype=torch.long)
            if world > 1:
                gathered = [None] * world
                dist.all_gather_object(gathered, local, group=self.group)
            else:
                gathered = [local]
            if rank == 0:
                paths.append(str(write_route_bundle(self.root, step, blk.layer_idx, gathered)))
        self._pending.clear()
        return paths
