"""Runtime expert placement state of one MoE layer (layout L, owners, mapping M).

``LayerPlacement`` keeps the plan of one layer as numpy arrays plus device
lookup tables:

* ``lut_global(rank)``  -- M[rank]: logical expert -> global physical slot;
* ``dest_rank`` / ``local_slot`` of every global slot;
* ``local_logical``     -- logical expert held by each local slot;
* ``replica_groups``    -- the global slots of every logical expert.

``version`` increases on every install (static load, mapping-only update,
full migration) so stale planner results can be rejected.

Static preload: ``slice_expert_weights`` fills a rank's slots from full
logical expert tensors according to the layout (each rank takes the logical
experts of its slots), the equivalent of the reference's artifact-driven EP
slicing.

Reference parity: ExpertLayerState and map_logical_to_physical
(veomni/distributed/moe/hiermoe/expert_swap.py:357-587, :5831-5979), static
preload veomni/distributed/parallel_plan.py:35-142, mapping-only install
expert_swap.py:10920-10973.
"""

from __future__ import annotations

import numpy as np
import torch

from ..placemoe.types import EMPTY_EXPERT, LayerPlan, PlaceMoETopology, identity_plan


class LayerPlacement:
    def __init__(self, plan: LayerPlan, topology: PlaceMoETopology, rank: int):
        plan.validate(topology)
        self.topology = topology
        self.rank = rank
        self.version = 0
        self._set(plan)

    def _set(self, plan: LayerPlan) -> None:
        t = self.topology
        self.plan = plan
        self.slot_to_logical = np.asarray(plan.slot_to_logical, dtype=np.int64)
        self.mapping = np.asarray(plan.source_logical_to_physical, dtype=np.int64)
        self.owner_slots = np.asarray(plan.owner_slots, dtype=np.int64)
        self.slot_rank = t.slot_ranks()
        self.local_slot = np.arange(t.total_slots) % t.slots_per_rank
        lo = self.rank * t.slots_per_rank
        self.local_logical = self.slot_to_logical[lo: lo + t.slots_per_rank].copy()
        self._dev_cache: dict = {}

    # -------------------------------------------------------------- queries
    @property
    def slots_per_rank(self) -> int:
        return self.topology.slots_per_rank

    def lut_global(self, src_rank: int | None = None) -> np.ndarray:
        return self.mapping[self.rank if src_rank is None else src_rank]

    def local_lut_cpu(self) -> torch.Tensor:
        """Single-device LUT: logical expert -> local slot (valid when every slot is on this rank)."""
        return torch.from_numpy(self.local_slot[self.lut_global()].copy())

    def local_lut_device(self, device) -> torch.Tensor:
        key = ("local", str(device))
        if key not in self._dev_cache:
            self._dev_cache[key] = self.local_lut_cpu().to(device=device, dtype=torch.int32)
        return self._dev_cache[key]

    def route_tables(self, device):
        """(dest_rank[E], local_slot[E]) of this rank's mapping as device int32 tensors."""
        key = ("route", str(device))
        if key not in self._dev_cache:
            g = self.lut_global()
            self._dev_cache[key] = (
                torch.from_numpy(self.slot_rank[g].copy()).to(device=device, dtype=torch.int32),
                torch.from_numpy(self.local_slot[g].copy()).to(device=device, dtype=torch.int32),
            )
        return self._dev_cache[key]

    def replica_groups(self) -> list[np.ndarray]:
        return [g for g in self.plan.replica_groups() if len(g) > 1]

    def is_redundant_local_slot(self, j: int) -> bool:
        """True when local slot j holds a copy that is not its expert's owner (excluded from grad norms)."""
        gslot = self.rank * self.slots_per_rank + j
        e = self.slot_to_logical[gslot]
        return e == EMPTY_EXPERT or self.owner_slots[e] != gslot

    # -------------------------------------------------------------- updates
    def install_mapping(self, plan: LayerPlan) -> None:
        """Mapping-only update: layout and owners must be unchanged."""
        plan.validate(self.topology)
        if not np.array_equal(plan.slot_to_logical, self.slot_to_logical):
            raise ValueError("mapping-only update changes the layout")
        if not np.array_equal(plan.owner_slots, self.owner_slots):
            raise ValueError("mapping-only update changes the runtime owners")
        self._set(plan)
        self.version += 1

    def install_layout(self, plan: LayerPlan) -> None:
        """Full (L, M) install; parameter migration must have been done by the caller."""
        plan.validate(self.topology)
        self._set(plan)
        self.version += 1


def build_placements(plans: dict[str, LayerPlan] | None, topology: PlaceMoETopology, rank: int,
                     layer_keys: list[str]) -> dict[str, LayerPlacement]:
    out = {}
    for key in layer_keys:
        plan = plans[key] if plans is not None and key in plans else identity_plan(topology)
        out[key] = LayerPlacement(plan, topology, rank)
    return out


@torch.no_grad()
def slice_expert_weights(full: torch.Tensor, placement: LayerPlacement) -> torch.Tensor:
    """Local slot tensor [spr, ...] from a full logical tensor [E, ...] (empty slots are zero)."""
    out = torch.zeros((placement.slots_per_rank, *full.shape[1:]), dtype=full.dtype, device=full.device)
    for j, e in enumerate(placement.local_logical.tolist()):
        if e != EMPTY_EXPERT:
            out[j].copy_(full[e])
    return out
