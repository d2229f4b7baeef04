"""PlaceMoE data model: topology, profile statistics and a per-layer plan (L, M).

* ``Topology(ep_size, ranks_per_node, num_experts, slots_per_rank)`` -- the
  physical slot capacity of one expert-parallel MoE layer.  On one NVSwitch
  domain (8xB200) ``ranks_per_node == ep_size``: one level.
* ``ProfileStatistics(demand[S, E], affinity[S, E, E])`` -- source-conditioned
  assignment demand and symmetric, zero-diagonal co-selection affinity.
* ``LayerPlan(slot_to_logical, source_logical_to_physical, owner_slots)`` --
  layout ``L`` (logical expert of every physical slot, -1 = empty), mapping
  ``M`` (copy that source rank r uses for logical expert e) and the runtime
  owner copy of every expert.  ``validate`` enforces: >= 1 copy per expert,
  optional exact extra-copy budget, M points at a copy of the right expert,
  owners hold their expert.

Semantics and the JSON payload keys are the same as
veomni/distributed/moe/hiermoe/placemoe/types.py:25-177 so that artifacts are
interchangeable.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np

EMPTY_EXPERT = -1


def _frozen(a, dtype) -> np.ndarray:
    out = np.array(a, dtype=dtype, copy=True)
    out.setflags(write=False)
    return out


@dataclass(frozen=True)
class PlaceMoETopology:
    ep_size: int
    ranks_per_node: int
    num_experts: int
    slots_per_rank: int

    def __post_init__(self) -> None:
        for k in ("ep_size", "ranks_per_node", "num_experts", "slots_per_rank"):
            if int(getattr(self, k)) <= 0:
                raise ValueError(f"{k} must be positive.")
        if self.ep_size % self.ranks_per_node != 0:
            raise ValueError("ep_size must be divisible by ranks_per_node.")
        if self.total_slots < self.num_experts:
            raise ValueError("Physical capacity cannot hold one copy of every expert.")

    @property
    def num_nodes(self) -> int:
        return self.ep_size // self.ranks_per_node

    @property
    def total_slots(self) -> int:
        return self.ep_size * self.slots_per_rank

    @property
    def extra_copies(self) -> int:
        return self.total_slots - self.num_experts

    def rank_of_slot(self, slot: int) -> int:
        if slot < 0 or slot >= self.total_slots:
            raise ValueError(f"Physical slot {slot} is outside the topology.")
        return slot // self.slots_per_rank

    def slot_ranks(self) -> np.ndarray:
        return np.arange(self.total_slots, dtype=np.int64) // self.slots_per_rank


@dataclass(frozen=True)
class ProfileStatistics:
    demand: np.ndarray
    affinity: np.ndarray

    def __post_init__(self) -> None:
        d = _frozen(self.demand, np.float64)
        a = _frozen(self.affinity, np.float64)
        if d.ndim != 2:
            raise ValueError("demand must have shape [source_rank, expert].")
        s, e = d.shape
        if a.shape != (s, e, e):
            raise ValueError("affinity must have shape [source_rank, expert, expert].")
        if (d < 0).any() or (a < 0).any():
            raise ValueError("Profile statistics must be non-negative.")
        if not np.allclose(a, np.swapaxes(a, 1, 2)):
            raise ValueError("Expert affinity must be symmetric for every source rank.")
        if not np.allclose(np.diagonal(a, axis1=1, axis2=2), 0.0):
            raise ValueError("Expert affinity diagonal must be zero.")
        object.__setattr__(self, "demand", d)
        object.__setattr__(self, "affinity", a)

    @property
    def ep_size(self) -> int:
        return self.demand.shape[0]

    @property
    def num_experts(self) -> int:
        return self.demand.shape[1]

    @property
    def expert_demand(self) -> np.ndarray:
        return self.demand.sum(0)

    @property
    def expert_affinity(self) -> np.ndarray:
        return self.affinity.sum(0)


@dataclass(frozen=True)
class LayerPlan:
    slot_to_logical: np.ndarray
    source_logical_to_physical: np.ndarray
    owner_slots: np.ndarray

    def __post_init__(self) -> None:
        object.__setattr__(self, "slot_to_logical", _frozen(self.slot_to_logical, np.int64))
        object.__setattr__(self, "source_logical_to_physical", _frozen(self.source_logical_to_physical, np.int64))
        object.__setattr__(self, "owner_slots", _frozen(self.owner_slots, np.int64))

    @property
    def copy_counts(self) -> np.ndarray:
        used = self.slot_to_logical[self.slot_to_logical != EMPTY_EXPERT]
        return np.bincount(used, minlength=len(self.owner_slots))

    def validate(self, topology: PlaceMoETopology, *, additional_copies: int | None = None) -> None:
        e, n = topology.num_experts, topology.total_slots
        layout, mapping, owners = self.slot_to_logical, self.source_logical_to_physical, self.owner_slots
        if layout.shape != (n,):
            raise ValueError("Layout length does not match the physical slot capacity.")
        if mapping.shape != (topology.ep_size, e):
            raise ValueError("Mapping shape does not match [source_rank, logical_expert].")
        if owners.shape != (e,):
            raise ValueError("owner_slots must contain one runtime owner per logical expert.")
        if (layout < EMPTY_EXPERT).any() or (layout >= e).any():
            raise ValueError("Layout contains an invalid logical expert ID.")
        counts = self.copy_counts
        if (counts[:e] < 1).any():
            raise ValueError("Every logical expert must retain at least one physical copy.")
        if additional_copies is not None and int(counts.sum()) - e != additional_copies:
            raise ValueError("Layout does not use the requested additional-copy budget.")
        if (mapping < 0).any() or (mapping >= n).any():
            raise ValueError("Mapping references a slot outside the topology.")
        if not np.array_equal(layout[mapping], np.broadcast_to(np.arange(e), mapping.shape)):
            raise ValueError("Mapping references a copy of the wrong logical expert.")
        if (owners < 0).any() or (owners >= n).any():
            raise ValueError("Runtime owner references a slot outside the topology.")
        if not np.array_equal(layout[owners], np.arange(e)):
            raise ValueError("Runtime owner slots do not match their logical experts.")

    def to_runtime_payload(self) -> dict[str, Any]:
        return {
            "slot_to_logical": self.slot_to_logical.tolist(),
            "owner_slots": self.owner_slots.tolist(),
            "source_logical_to_physical": self.source_logical_to_physical.tolist(),
        }

    @classmethod
    def from_runtime_payload(cls, payload: dict[str, Any]) -> "LayerPlan":
        return cls(
            slot_to_logical=payload["slot_to_logical"],
            owner_slots=payload["owner_slots"],
            source_logical_to_physical=payload["source_logical_to_physical"],
        )

    def replica_groups(self) -> list[np.ndarray]:
        """Physical slots of every logical expert (owner first)."""
        groups = []
        for e, owner in enumerate(self.owner_slots.tolist()):
            slots = np.flatnonzero(self.slot_to_logical == e)
            groups.append(np.concatenate([[owner], slots[slots != owner]]).astype(np.int64))
        return groups


def identity_plan(topology: PlaceMoETopology) -> LayerPlan:
    """Fixed expert parallelism: expert e on slot e (contiguous blocks per rank), no replicas.

    Extra slots (if any) are left empty.
    """
    n, e = topology.total_slots, topology.num_experts
    per_rank = -(-e // topology.ep_size)
    if per_rank > topology.slots_per_rank:
        raise ValueError("identity plan needs ceil(E / ep) <= slots_per_rank")
    layout = np.full(n, EMPTY_EXPERT, dtype=np.int64)
    owners = np.zeros(e, dtype=np.int64)
    for x in range(e):
        r, j = divmod(x, per_rank)
        slot = r * topology.slots_per_rank + j
        layout[slot] = x
        owners[x] = slot
    mapping = np.broadcast_to(owners, (topology.ep_size, e)).copy()
    plan = LayerPlan(layout, mapping, owners)
    plan.validate(topology)
    return plan
