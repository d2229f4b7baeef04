"""PlaceMoE data model: the slot topology, profile statistics and a per-layer plan (L, M).

A placement problem lives on ``PlaceMoETopology``: ``ep_size`` GPUs grouped
into nodes of ``ranks_per_node``, each GPU holding ``slots_per_rank`` physical
expert slots, for ``num_experts`` logical experts.  Slot ``s`` sits on GPU
``s // slots_per_rank``.  On one NVSwitch domain (8xB200) there is one node.

``LayerPlan`` is the answer for one MoE layer:

* ``slot_to_logical`` (layout L): the logical expert held by every slot, or
  ``EMPTY_EXPERT`` (-1);
* ``source_logical_to_physical`` (mapping M): ``M[r, e]`` is the slot whose
  copy of expert ``e`` serves tokens routed on GPU ``r``;
* ``owner_slots``: the copy of every expert that owns its optimizer state and
  counts it once in the gradient norm.

A plan is consistent when every expert has a copy, every ``M[r, e]`` and
``owner_slots[e]`` points at a slot holding ``e``, and (optionally) the layout
spends exactly the requested number of extra copies.  ``LayerPlan.problems``
lists every violated rule; ``validate`` raises on the first.

``ProfileStatistics`` carries what the planner optimises against: the
source-conditioned demand ``demand[r, e]`` (assignments of expert ``e`` made
on GPU ``r``) and the co-selection ``affinity[r, e, f]`` (tokens of GPU ``r``
that chose both ``e`` and ``f``; symmetric, zero diagonal).

The three arrays of a plan and their JSON keys are the interchange format of
the schema-v2 artifact; their meaning matches
veomni/distributed/moe/hiermoe/placemoe/types.py:25-177, so artifacts written
by either implementation load in the other.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np

EMPTY_EXPERT = -1

_PLAN_KEYS = ("slot_to_logical", "owner_slots", "source_logical_to_physical")


def _readonly(values, dtype) -> np.ndarray:
    arr = np.array(values, dtype=dtype, copy=True)
    arr.flags.writeable = False
    return arr


@dataclass(frozen=True)
class PlaceMoETopology:
    ep_size: int
    ranks_per_node: int
    num_experts: int
    slots_per_rank: int

    def __post_init__(self) -> None:
        bad = [name for name in ("ep_size", "ranks_per_node", "num_experts", "slots_per_rank")
               if int(getattr(self, name)) < 1]
        if bad:
            raise ValueError(f"topology sizes must be >= 1: {', '.join(bad)}")
        if self.ep_size % self.ranks_per_node:
            raise ValueError(f"{self.ep_size} GPUs do not split into nodes of {self.ranks_per_node}")
        if self.total_slots < self.num_experts:
            raise ValueError(f"{self.total_slots} slots cannot hold {self.num_experts} experts once each")

    @property
    def num_nodes(self) -> int:
        return self.ep_size // self.ranks_per_node

    @property
    def total_slots(self) -> int:
        return self.ep_size * self.slots_per_rank

    @property
    def extra_copies(self) -> int:
        """Slots beyond one copy per expert: the replica budget."""
        return self.total_slots - self.num_experts

    def rank_of_slot(self, slot: int) -> int:
        if not 0 <= slot < self.total_slots:
            raise ValueError(f"slot {slot} is not in [0, {self.total_slots})")
        return slot // self.slots_per_rank

    def slot_ranks(self) -> np.ndarray:
        """GPU of every slot, [total_slots]."""
        return np.repeat(np.arange(self.ep_size, dtype=np.int64), self.slots_per_rank)


@dataclass(frozen=True)
class ProfileStatistics:
    demand: np.ndarray
    affinity: np.ndarray

    def __post_init__(self) -> None:
        demand = _readonly(self.demand, np.float64)
        affinity = _readonly(self.affinity, np.float64)
        if demand.ndim != 2:
            raise ValueError(f"demand is [gpu, expert]; got shape {demand.shape}")
        gpus, experts = demand.shape
        if affinity.shape != (gpus, experts, experts):
            raise ValueError(f"affinity is [gpu, expert, expert] = {(gpus, experts, experts)}; got {affinity.shape}")
        if min(demand.min(initial=0.0), affinity.min(initial=0.0)) < 0:
            raise ValueError("demand and affinity are counts: no negative entries")
        if not np.allclose(affinity, affinity.transpose(0, 2, 1)):
            raise ValueError("affinity[r] must be a symmetric matrix for every GPU r")
        if np.abs(np.einsum("rii->ri", affinity)).max(initial=0.0) > 1e-9:
            raise ValueError("affinity[r, e, e] must be 0 (an expert is not co-selected with itself)")
        object.__setattr__(self, "demand", demand)
        object.__setattr__(self, "affinity", affinity)

    @property
    def ep_size(self) -> int:
        return int(self.demand.shape[0])

    @property
    def num_experts(self) -> int:
        return int(self.demand.shape[1])

    @property
    def expert_demand(self) -> np.ndarray:
        """Demand per expert over all source GPUs, [E]."""
        return self.demand.sum(axis=0)

    @property
    def expert_affinity(self) -> np.ndarray:
        """Co-selection over all source GPUs, [E, E]."""
        return self.affinity.sum(axis=0)


@dataclass(frozen=True)
class LayerPlan:
    slot_to_logical: np.ndarray
    source_logical_to_physical: np.ndarray
    owner_slots: np.ndarray

    def __post_init__(self) -> None:
        for name in _PLAN_KEYS:
            object.__setattr__(self, name, _readonly(getattr(self, name), np.int64))

    @property
    def copy_counts(self) -> np.ndarray:
        """Copies of every logical expert in the layout, [E]."""
        held = self.slot_to_logical[self.slot_to_logical >= 0]
        return np.bincount(held, minlength=len(self.owner_slots))

    def problems(self, topology: PlaceMoETopology, additional_copies: int | None = None) -> list[str]:
        """Every rule of a consistent plan that this plan breaks (empty when it is consistent)."""
        e, n, r = topology.num_experts, topology.total_slots, topology.ep_size
        layout, mapping, owners = self.slot_to_logical, self.source_logical_to_physical, self.owner_slots
        shapes = [("layout", layout.shape, (n,)), ("mapping", mapping.shape, (r, e)), ("owners", owners.shape, (e,))]
        found = [f"{what} has shape {got}, the topology needs {want}" for what, got, want in shapes if got != want]
        if found:
            return found  # the element checks below need the right shapes
        if ((layout < EMPTY_EXPERT) | (layout >= e)).any():
            found.append(f"layout entries must be -1 (empty) or an expert id below {e}")
            return found
        copies = self.copy_counts
        missing = np.flatnonzero(copies[:e] == 0)
        if missing.size:
            found.append(f"experts without any copy: {missing[:8].tolist()}")
        if additional_copies is not None and int(copies.sum()) - e != additional_copies:
            found.append(f"layout spends {int(copies.sum()) - e} extra copies, the budget is {additional_copies}")
        for what, slots, expect in (("mapping", mapping, np.broadcast_to(np.arange(e), mapping.shape)),
                                    ("owner", owners, np.arange(e))):
            if ((slots < 0) | (slots >= n)).any():
                found.append(f"{what} points outside the {n} slots")
            elif not np.array_equal(layout[slots], expect):
                found.append(f"{what} points at a slot that holds another expert")
        return found

    def validate(self, topology: PlaceMoETopology, *, additional_copies: int | None = None) -> None:
        found = self.problems(topology, additional_copies)
        if found:
            raise ValueError("inconsistent layer plan: " + "; ".join(found))

    def to_runtime_payload(self) -> dict[str, Any]:
        """The artifact's per-layer JSON object."""
        return {name: getattr(self, name).tolist() for name in _PLAN_KEYS}

    @classmethod
    def from_runtime_payload(cls, payload: dict[str, Any]) -> "LayerPlan":
        return cls(**{name: payload[name] for name in _PLAN_KEYS})

    def replica_groups(self) -> list[np.ndarray]:
        """Slots of every logical expert, owner first (one group per expert)."""
        order = np.argsort(self.slot_to_logical, kind="stable")
        held = self.slot_to_logical[order]
        groups = []
        for e, owner in enumerate(self.owner_slots.tolist()):
            lo, hi = np.searchsorted(held, [e, e + 1])
            others = order[lo:hi]
            groups.append(np.concatenate(([owner], others[others != owner])).astype(np.int64))
        return groups


def identity_plan(topology: PlaceMoETopology) -> LayerPlan:
    """Fixed expert parallelism: expert e on slot e (contiguous blocks per rank), no replicas.

    Extra slots (if any) are left empty.
    """
    e, spr = topology.num_experts, topology.slots_per_rank
    per_rank = -(-e // topology.ep_size)
    if per_rank > spr:
        raise ValueError(f"fixed EP needs ceil({e} / {topology.ep_size}) = {per_rank} slots per GPU, have {spr}")
    experts = np.arange(e)
    owners = (experts // per_rank) * spr + experts % per_rank
    layout = np.full(topology.total_slots, EMPTY_EXPERT, dtype=np.int64)
    layout[owners] = experts
    plan = LayerPlan(layout, np.tile(owners, (topology.ep_size, 1)), owners)
    plan.validate(topology)
    return plan
