"""Deterministic feasible plans used as seeds and baselines.

* ``mirrored_r2_plan``: exactly two copies of every expert, the second copy in
  the mirrored half of the EP group; sources of each half use their half's copy.
* ``eplb_plan``: EPLB-style replication -- replica counts from the greedy
  max-per-copy-load allocation, copies packed onto GPUs longest-processing-time
  first (no GPU holds two copies of one expert), sources use the least-loaded
  copy (local copy first).
* ``fixed_ep_plan``: plain expert parallelism (identity layout, no replicas).

Reference parity: veomni/distributed/moe/hiermoe/placemoe/seeds.py:24-48 and the
EPLB layout builder scripts/profile/build_hiermoe_eplb_layout.py.
"""

from __future__ import annotations

import numpy as np

from .allocation import greedy_allocation, instances_from_allocation
from .mapping import initialize_mapping
from .materialize import layout_from_ranks, materialize_plan
from .partition import PartitionConfig, _lpt_seed, repair_duplicates
from .types import LayerPlan, PlaceMoETopology, identity_plan


def mirrored_r2_plan(topology: PlaceMoETopology) -> LayerPlan:
    if topology.ep_size % 2 or topology.total_slots != 2 * topology.num_experts:
        raise ValueError("Mirrored R2 requires an even EP size and exactly two copies per expert.")
    n, e = topology.total_slots, topology.num_experts
    layout = np.full(n, -1, dtype=np.int64)
    owners = np.zeros(e, dtype=np.int64)
    mapping = np.zeros((topology.ep_size, e), dtype=np.int64)
    half = topology.ep_size // 2
    for x in range(e):
        r, j = divmod(x, topology.slots_per_rank)
        a = r * topology.slots_per_rank + j
        b = (half + r) * topology.slots_per_rank + j
        layout[a] = layout[b] = x
        owners[x] = a
        mapping[:half, x] = a
        mapping[half:, x] = b
    plan = LayerPlan(layout, mapping, owners)
    plan.validate(topology, additional_copies=e)
    return plan


def fixed_ep_plan(topology: PlaceMoETopology) -> LayerPlan:
    return identity_plan(topology)


def eplb_plan(topology: PlaceMoETopology, demand: np.ndarray) -> LayerPlan:
    """demand: [S, E] source-conditioned demand (or [E])."""
    d2 = np.atleast_2d(np.asarray(demand, dtype=np.float64))
    if d2.shape[0] != topology.ep_size:
        d2 = np.broadcast_to(d2.sum(0) / topology.ep_size, (topology.ep_size, topology.num_experts))
    tot = d2.sum(0)
    extra = greedy_allocation(tot, topology.extra_copies, max_copies=topology.ep_size)
    inst = instances_from_allocation(topology.num_experts, extra)
    copies = np.bincount(inst, minlength=topology.num_experts)
    inst_demand = tot[inst] / copies[inst]
    cfg = PartitionConfig(capacities=(topology.slots_per_rank,) * topology.ep_size,
                          ranks_per_group=(1,) * topology.ep_size, omega=0.0, gamma=1.0)
    ranks = repair_duplicates(_lpt_seed(inst_demand, inst, cfg), inst, inst_demand)
    layout, _ = layout_from_ranks(inst, ranks, topology)
    mapping = initialize_mapping(d2, layout, topology.slot_ranks(), topology.ep_size)
    return materialize_plan(layout, mapping, d2, topology)
