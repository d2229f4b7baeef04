"""Source-aware token-to-copy mapping M[source_rank, logical_expert] -> physical slot.

``initialize_mapping``: demand-ordered greedy -- a source uses its own GPU's
copy when it has one, otherwise the copy whose rank currently carries the
least projected load.
``optimize_mapping``: coordinate descent in the C++ core with the objective
-omega*co-selection reuse - lambda*on-GPU demand + gamma*peak rank load.
``optimize_mapping_normalized``: scale-free proposals spanning communication-only
to compute-balanced mappings.
``optimize_community_mapping``: block mapping of (source unit, expert community)
to destination units, scored with exact per-destination row counts from the
community-mask histogram (``community_intersection_hits``).

Reference parity: veomni/distributed/moe/hiermoe/placemoe/mapping.py:181-810.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .._build import load_planner


def copies_of(slot_to_logical: np.ndarray, num_experts: int) -> list[np.ndarray]:
    return [np.flatnonzero(slot_to_logical == e) for e in range(num_experts)]


def mapping_rank_loads(demand: np.ndarray, mapping: np.ndarray, slot_rank: np.ndarray, ep_size: int) -> np.ndarray:
    loads = np.zeros(ep_size)
    for s in range(demand.shape[0]):
        np.add.at(loads, slot_rank[mapping[s]], demand[s])
    return loads


def validate_instance_mapping(mapping: np.ndarray, slot_to_logical: np.ndarray, num_experts: int) -> None:
    if mapping.shape[1] != num_experts:
        raise ValueError("mapping must be [source_rank, logical_expert]")
    if not np.array_equal(slot_to_logical[mapping], np.broadcast_to(np.arange(num_experts), mapping.shape)):
        raise ValueError("mapping references a copy of the wrong logical expert")


def initialize_mapping(demand: np.ndarray, slot_to_logical: np.ndarray, slot_rank: np.ndarray,
                       ep_size: int) -> np.ndarray:
    s_count, e = demand.shape
    cps = copies_of(slot_to_logical, e)
    mapping = np.zeros((s_count, e), dtype=np.int64)
    loads = np.zeros(ep_size)
    order = np.dstack(np.unravel_index(np.argsort(-demand, axis=None, kind="stable"), demand.shape))[0]
    for s, x in order:
        c = cps[x]
        local = c[slot_rank[c] == s]
        if len(local):
            pick = int(local[0])
        else:
            pick = int(c[np.lexsort((c, loads[slot_rank[c]]))[0]])
        mapping[s, x] = pick
        loads[slot_rank[pick]] += demand[s, x]
    return mapping


def optimize_mapping(demand: np.ndarray, affinity: np.ndarray, slot_to_logical: np.ndarray, slot_rank: np.ndarray,
                     mapping: np.ndarray, *, omega: float, gamma: float, local_weight: float,
                     sweeps: int = 8) -> tuple[np.ndarray, float]:
    m = torch.from_numpy(np.ascontiguousarray(mapping, dtype=np.int64).copy())
    obj = load_planner().optimize_mapping(torch.from_numpy(np.array(demand, dtype=np.float64, copy=True)),
                                          torch.from_numpy(np.array(affinity, dtype=np.float64, copy=True)),
                                          torch.from_numpy(np.array(slot_to_logical, dtype=np.int64, copy=True)),
                                          torch.from_numpy(np.array(slot_rank, dtype=np.int64, copy=True)), m,
                                          float(omega), float(local_weight), float(gamma), int(sweeps))
    return m.numpy().copy(), float(obj)


# ------------------------------------------------------------------ proposals beyond coordinate descent
def optimize_mapping_normalized(demand: np.ndarray, affinity: np.ndarray, slot_to_logical: np.ndarray,
                                slot_rank: np.ndarray, mapping: np.ndarray, *, ranks_per_node: int,
                                assignment_weight: float, node_weight: float = 1.0, rank_weight: float = 0.15,
                                sweeps: int = 6) -> tuple[np.ndarray, float]:
    """Scale-normalised mapping proposal (C++ core): co-selection reward on the candidate's node / GPU over the
    total co-selection mass, minus ``assignment_weight`` x projected peak GPU load over the total demand.

    Returns (mapping, peak GPU load).  A proposal only: the exact route replay decides whether it is kept.
    """
    m = torch.from_numpy(np.ascontiguousarray(mapping, dtype=np.int64).copy())
    peak, _, _ = load_planner().optimize_mapping_normalized(
        torch.from_numpy(np.array(demand, dtype=np.float64, copy=True)),
        torch.from_numpy(np.array(affinity, dtype=np.float64, copy=True)),
        torch.from_numpy(np.array(slot_to_logical, dtype=np.int64, copy=True)),
        torch.from_numpy(np.array(slot_rank, dtype=np.int64, copy=True)), m, int(ranks_per_node),
        float(assignment_weight), float(node_weight), float(rank_weight), int(sweeps))
    return m.numpy().copy(), float(peak)


def community_intersection_hits(mask_histogram: np.ndarray) -> np.ndarray:
    """hits[u, X] = tokens of source unit u whose community mask shares a community with X."""
    h = torch.from_numpy(np.ascontiguousarray(mask_histogram, dtype=np.int64))
    return load_planner().community_intersection_hits(h).numpy()


def community_mask_histogram(routes_by_source, communities: np.ndarray, *, ranks_per_unit: int,
                             num_communities: int, sources_per_step: int = 0) -> np.ndarray:
    """Tokens per (source unit, set of communities the token's experts belong to); sources are grouped
    ``ranks_per_unit`` at a time.  routes_by_source: one [tokens, k] logical-route tensor per source GPU,
    or several steps of them back to back (``sources_per_step`` each), summed over the steps."""
    rs = [torch.as_tensor(r) for r in routes_by_source]  # int32 or int64; the core converts anything else
    c = torch.from_numpy(np.ascontiguousarray(communities, dtype=np.int64))
    return load_planner().community_mask_histogram(rs, c, int(ranks_per_unit), int(num_communities),
                                                   int(sources_per_step)).numpy()


@dataclass(frozen=True)
class CommunityMappingResult:
    mapping: np.ndarray  # [source GPU, expert] -> slot
    destination_units: np.ndarray  # [source unit, community] -> destination unit
    proxy_cost: float
    sweeps: int
    changes: int


def optimize_community_mapping(slot_to_logical: np.ndarray, slot_unit: np.ndarray, communities: np.ndarray,
                               assignments_by_community: np.ndarray, mask_histogram: np.ndarray, *,
                               ranks_per_unit: int, comm_ms_per_token: float, ms_per_assignment: float,
                               row_limit: int = 64, beam_width: int = 64, sweeps: int = 4,
                               intersection_hits: np.ndarray | None = None) -> CommunityMappingResult:
    """Map every (source unit, expert community) block to one destination unit (C++ core).

    slot_to_logical [N]: layout; slot_unit [N]: unit (node, or GPU on one level) of every slot;
    communities [E]: community label of every expert (0..C-1); assignments_by_community [U, C];
    mask_histogram [U, 2^C].  A unit can serve a community only when it holds a copy of every expert of
    the community; an expert may hold at most one copy per unit.
    """
    layout = np.asarray(slot_to_logical, dtype=np.int64)
    unit = np.asarray(slot_unit, dtype=np.int64)
    comm = np.asarray(communities, dtype=np.int64)
    e, c = len(comm), int(comm.max(initial=-1)) + 1
    if c == 0 or (comm < 0).any() or not np.array_equal(np.unique(comm), np.arange(c)):
        raise ValueError("community labels must cover 0..C-1 with every expert labelled")
    asg = np.asarray(assignments_by_community, dtype=np.float64)
    units = asg.shape[0]
    copy_at = np.full((e, units), -1, dtype=np.int64)  # slot of expert x on unit u
    for slot, x in enumerate(layout.tolist()):
        if x < 0:
            continue
        if copy_at[x, unit[slot]] >= 0:
            raise ValueError(f"expert {x} has two copies on unit {int(unit[slot])}")
        copy_at[x, unit[slot]] = slot
    allowed = np.stack([(copy_at[comm == k] >= 0).all(axis=0) for k in range(c)]).astype(np.int64)  # [C, U]
    hits = community_intersection_hits(mask_histogram) if intersection_hits is None else intersection_hits
    dest, cost, done, changes = load_planner().optimize_community_mapping(
        torch.from_numpy(allowed), torch.from_numpy(np.ascontiguousarray(asg)),
        torch.from_numpy(np.ascontiguousarray(hits, dtype=np.int64)), float(comm_ms_per_token),
        float(ms_per_assignment), int(ranks_per_unit), int(row_limit), int(beam_width), int(sweeps))
    dest = dest.numpy()
    mapping = np.empty((units * ranks_per_unit, e), dtype=np.int64)
    for u in range(units):
        mapping[u * ranks_per_unit:(u + 1) * ranks_per_unit] = copy_at[np.arange(e), dest[u, comm]][None, :]
    return CommunityMappingResult(mapping, dest, float(cost), int(done), int(changes))


def copy_set_communities(slot_to_logical: np.ndarray, slot_rank: np.ndarray, num_experts: int,
                         max_communities: int = 16) -> np.ndarray | None:
    """One-level communities: experts whose copies sit on exactly the same set of GPUs form one community
    (so every GPU of the set serves the whole community).  None when there are more than
    ``max_communities`` distinct sets (the mask histogram would be too large)."""
    layout = np.asarray(slot_to_logical, dtype=np.int64)
    sets = [tuple(sorted(set(slot_rank[layout == x].tolist()))) for x in range(num_experts)]
    index: dict = {}
    labels = np.array([index.setdefault(s, len(index)) for s in sets], dtype=np.int64)
    return labels if len(index) <= max_communities else None
