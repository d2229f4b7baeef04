"""Gradient reduction and parallelization wiring.

Dense parameters (attention, norms, router, embeddings, lm head) are
replicated on every rank as bf16 compute copies; their fp32 gradients live in
ONE flat bucket (each parameter's ``main_grad`` is a view of it), so the whole
dense gradient is reduced with a single collective per step.  Expert slots are
sharded by expert parallelism and need no data-parallel reduction; copies of
the same logical expert on different GPUs are summed by
:func:`sync_replica_gradients`.

``parallelize_model`` applies this layout: EP placement per MoE layer, the
flat dense gradient bucket and the replica groups.

Reference parity: FSDP2 data parallelism of veomni/distributed/torch_parallelize.py:92-428
(grad divide factor :320-335) and the replica-gradient synchronisation of
veomni/distributed/moe/hiermoe/expert_swap.py:6589-7252.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from ..placemoe.types import PlaceMoETopology
from .ep import ExpertParallel
from .placement import build_placements


def is_expert_param(name: str) -> bool:
    return name.endswith("gate_up_proj") or name.endswith("down_proj")


class DenseGradBucket:
    """One fp32 buffer backing ``main_grad`` of every dense parameter."""

    def __init__(self, params: list[torch.Tensor], device):
        self.params = params
        n = sum(p.numel() for p in params)
        self.flat = torch.zeros(n, dtype=torch.float32, device=device)
        off = 0
        for p in params:
            p.main_grad = self.flat[off: off + p.numel()].view(p.shape)
            off += p.numel()

    def zero(self):
        self.flat.zero_()

    def reduce(self, group=None):
        """Sum over the data-parallel group (the loss is pre-divided by the world size)."""
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)


def sync_replica_gradients(model, placements: dict, group=None) -> int:
    """Sum the gradients of all physical copies of each logical expert (copies stay identical).

    Every rank packs the main_grad of each of its replicated slots into a
    buffer indexed by (replica-group id); one all-reduce sums the copies.
    Returns the number of replica groups synchronised.
    """
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return 0
    total = 0
    for blk in model.moe_blocks():
        pl = placements.get(blk.layer_key)
        if pl is None:
            continue
        groups = pl.replica_groups()
        if not groups:
            continue
        total += len(groups)
        spr = pl.slots_per_rank
        lo = pl.rank * spr
        for p in (blk.gate_up_proj, blk.down_proj):
            g = getattr(p, "main_grad", None)
            if g is None:
                g = p.grad
            if g is None:
                g = torch.zeros(p.shape, device=p.device, dtype=torch.float32)
                p.main_grad = g
            per = g[0].numel()
            buf = torch.zeros(len(groups), per, device=g.device, dtype=torch.float32)
            mine = []
            for gi, slots in enumerate(groups):
                for s in slots.tolist():
                    if lo <= s < lo + spr:
                        buf[gi].add_(g[s - lo].reshape(-1))
                        mine.append((gi, s - lo))
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
            for gi, j in mine:
                g[j].copy_(buf[gi].view_as(g[j]))
    return total


def redundant_slot_weights(blk, placement) -> list[float]:
    """Grad-norm weight per local slot: 1 for the owner copy, 0 for redundant copies and empty slots."""
    return [0.0 if placement.is_redundant_local_slot(j) else 1.0 for j in range(placement.slots_per_rank)]


class ParallelState:
    def __init__(self, world: int, rank: int, device, topology: PlaceMoETopology, placements: dict,
                 ep: ExpertParallel | None, dense_bucket: DenseGradBucket | None):
        self.world = world
        self.rank = rank
        self.device = device
        self.topology = topology
        self.placements = placements
        self.ep = ep
        self.dense_bucket = dense_bucket


def expert_topology(num_experts: int, ep_size: int, redundant_slots_per_rank: int = 0) -> PlaceMoETopology:
    primary = -(-num_experts // ep_size)
    return PlaceMoETopology(ep_size, ep_size, num_experts, primary + redundant_slots_per_rank)


def parallelize_model(model, *, plans=None, topology: PlaceMoETopology | None = None, group=None, device=None,
                      capture_routes: bool = False, transport: str = "auto") -> ParallelState:
    """Attach EP placement + dispatch to every MoE block and back dense grads with one bucket.

    ``transport``: "auto" (peer-memory kernels on CUDA, all-to-all otherwise), "p2p" or "nccl"
    (all-to-all with exchanged split sizes, the baseline).
    The model must already hold the local expert slots (built with
    ``num_local_slots = topology.slots_per_rank`` and filled through
    :func:`placement.slice_expert_weights` or an expert_init callback).
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    cfg = model.config
    if topology is None:
        topology = expert_topology(cfg.num_experts or world, world)
    if topology.ep_size != world:
        raise ValueError("expert parallel size must equal the process-group size")
    keys = [blk.layer_key for blk in model.moe_blocks()]
    placements = build_placements(plans, topology, rank, keys)
    ep = None
    if world > 1 and keys:
        dev0 = device or next(model.parameters()).device
        # "auto": peer-memory kernels on CUDA (no host synchronisation), all-to-all on CPU / gloo
        use_p2p = transport == "p2p" or (transport == "auto" and dev0.type == "cuda")
        if use_p2p:
            from .p2p_ep import P2PExpertParallel

            ep = P2PExpertParallel(group, capture_routes=capture_routes)
        else:
            ep = ExpertParallel(group, capture_routes=capture_routes)
    if ep is not None and hasattr(ep, "num_layers"):
        ep.num_layers = len(keys)  # one receive slab per MoE layer in the peer-memory arena
    for i, blk in enumerate(model.moe_blocks()):
        blk.ep_slab = i
        if blk.num_local_slots != topology.slots_per_rank:
            raise ValueError(f"{blk.layer_key} holds {blk.num_local_slots} slots, topology needs "
                             f"{topology.slots_per_rank}")
        blk.placement = placements[blk.layer_key]
        blk.ep = ep
    dev = device or next(model.parameters()).device
    bucket = None
    if dev.type == "cuda":
        dense = [p for n, p in model.named_parameters() if not is_expert_param(n)]
        bucket = DenseGradBucket(dense, dev)
    return ParallelState(world, rank, dev, topology, placements, ep, bucket)


def expert_init_from_full(model_cfg, topology: PlaceMoETopology, plans, rank: int, seed: int = 0, device="cpu"):
    """expert_init callback: draw the FULL logical expert tensors with a fixed seed and slice this rank's slots.

    Every rank draws the same logical experts, so copies are identical and a
    placement change never alters the function the model computes.
    """
    from ..placemoe.types import identity_plan
    from .placement import LayerPlacement

    std = model_cfg.initializer_range
    h, i, e = model_cfg.hidden_size, model_cfg.moe_intermediate_size, model_cfg.num_experts

    def init(layer_idx: int, name: str, tensor: torch.Tensor):
        key = f"model.layers.{layer_idx}.mlp.experts"
        plan = plans[key] if plans and key in plans else identity_plan(topology)
        pl = LayerPlacement(plan, topology, rank)
        g = torch.Generator(device="cpu").manual_seed(seed * 1000003 + layer_idx * 2 + (0 if name == "gate_up_proj" else 1))
        shape = (e, 2 * i, h) if name == "gate_up_proj" else (e, h, i)
        for j, x in enumerate(pl.local_logical.tolist()):
            if x < 0:
                tensor[j].zero_()
                continue
            # draw expert x deterministically (independent of how many experts precede it)
            gx = torch.Generator(device=tensor.device)
            gx.manual_seed(int(g.initial_seed()) + 7919 * (x + 1))
            tensor[j].normal_(0.0, std, generator=gx)

    return init


def flatten_mask(weights: list[float]) -> np.ndarray:
    return np.asarray(weights, dtype=np.float64)
