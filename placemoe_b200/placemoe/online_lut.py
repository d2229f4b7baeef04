"""Online mapping correction: re-point a few entries of M for a fixed layout L.

Between planner runs, the source-aware mapping ``M[s, e]`` (which copy of
expert ``e`` serves tokens of source rank ``s``) can drift out of balance.
This greedy corrector evaluates every single-entry change (s, e -> another
copy of e) against the recent source-conditioned demand and applies the best
``max_changes`` ones, each only if it lowers the objective

    max_r load_r  +  remote_weight * remote assignments

where ``load_r`` is the assignments served by rank r.  The layout (which
expert sits in which slot) is untouched, so the result installs as a
mapping-only update.

Reference parity: veomni/distributed/moe/hiermoe/online_lut_planner.py
(one-entry LUT correction for a fixed layout).
"""

from __future__ import annotations

import numpy as np

from .types import LayerPlan, PlaceMoETopology


def _objective(mapping: np.ndarray, demand: np.ndarray, slot_rank: np.ndarray, world: int,
               remote_weight: float) -> float:
    load = np.zeros(world)
    remote = 0.0
    for s in range(demand.shape[0]):
        ranks = slot_rank[mapping[s]]
        np.add.at(load, ranks, demand[s])
        remote += float(demand[s][ranks != s].sum())
    return float(load.max()) + remote_weight * remote


def online_lut_update(plan: LayerPlan, topology: PlaceMoETopology, demand: np.ndarray, *, max_changes: int = 1,
                      remote_weight: float = 0.1) -> tuple[LayerPlan, list[tuple[int, int, int, int]]]:
    """Return (new plan, [(source, expert, old slot, new slot)]) with at most ``max_changes`` edits."""
    demand = np.asarray(demand, dtype=np.float64)
    layout = np.asarray(plan.slot_to_logical)
    mapping = np.asarray(plan.source_logical_to_physical).copy()
    slot_rank = np.arange(len(layout)) // topology.slots_per_rank
    copies = {e: np.flatnonzero(layout == e) for e in range(topology.num_experts)}
    changes = []
    cur = _objective(mapping, demand, slot_rank, topology.ep_size, remote_weight)
    for _ in range(max_changes):
        best = None
        for s in range(topology.ep_size):
            for e in range(topology.num_experts):
                if demand[s, e] <= 0 or len(copies[e]) < 2:
                    continue
                old = mapping[s, e]
                for c in copies[e]:
                    if c == old:
                        continue
                    mapping[s, e] = c
                    val = _objective(mapping, demand, slot_rank, topology.ep_size, remote_weight)
                    if val < cur - 1e-12 and (best is None or val < best[0]):
                        best = (val, s, e, int(old), int(c))
                mapping[s, e] = old
        if best is None:
            break
        cur, s, e, old, new = best
        mapping[s, e] = new
        changes.append((s, e, old, new))
    new_plan = LayerPlan(layout.copy(), mapping, np.asarray(plan.owner_slots).copy())
    new_plan.validate(topology, additional_copies=topology.total_slots - topology.num_experts
                      - int((layout < 0).sum()))
    return new_plan, changes
