"""Turn (instances, instance ranks, instance mapping) into a physical LayerPlan.

Instances of each rank are laid out in its ``slots_per_rank`` physical slots
(base copies before replicas, then by expert id, so an identity-like placement
keeps experts in ascending slot order).  The runtime owner of each logical
expert is the copy that serves the most demand under M (ties -> lowest slot);
M is rewritten from instance indices to physical slots.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/materialize.py:26-139.
"""

from __future__ import annotations

import numpy as np

from .types import LayerPlan, PlaceMoETopology


def layout_from_ranks(instance_expert: np.ndarray, instance_ranks: np.ndarray,
                      topology: PlaceMoETopology) -> tuple[np.ndarray, np.ndarray]:
    """Returns (slot_to_logical [N], slot_of_instance [I])."""
    n = topology.total_slots
    layout = np.full(n, -1, dtype=np.int64)
    slot_of = np.zeros(len(instance_expert), dtype=np.int64)
    base = np.zeros(len(instance_expert), dtype=bool)
    seen = set()
    for i, e in enumerate(instance_expert.tolist()):
        if e not in seen:
            base[i] = True
            seen.add(e)
    for r in range(topology.ep_size):
        members = np.flatnonzero(instance_ranks == r)
        if len(members) > topology.slots_per_rank:
            raise ValueError(f"rank {r} receives more instances than slots")
        members = members[np.lexsort((instance_expert[members], ~base[members]))]
        for j, i in enumerate(members.tolist()):
            slot = r * topology.slots_per_rank + j
            layout[slot] = instance_expert[i]
            slot_of[i] = slot
    return layout, slot_of


def select_owners(layout: np.ndarray, mapping: np.ndarray, demand: np.ndarray, num_experts: int) -> np.ndarray:
    served = np.zeros(len(layout))
    for s in range(mapping.shape[0]):
        np.add.at(served, mapping[s], demand[s])
    owners = np.zeros(num_experts, dtype=np.int64)
    for e in range(num_experts):
        cps = np.flatnonzero(layout == e)
        owners[e] = int(cps[np.lexsort((cps, -served[cps]))[0]])
    return owners


def materialize_plan(layout: np.ndarray, mapping_slots: np.ndarray, demand: np.ndarray,
                     topology: PlaceMoETopology) -> LayerPlan:
    owners = select_owners(layout, mapping_slots, demand, topology.num_experts)
    plan = LayerPlan(slot_to_logical=layout, source_logical_to_physical=mapping_slots, owner_slots=owners)
    plan.validate(topology)
    return plan
