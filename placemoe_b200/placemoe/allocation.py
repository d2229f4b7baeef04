"""Exact-budget replica allocation: how many physical copies each expert gets.

``additional = full_rounds * E + residual`` extra copies: every expert gets
``full_rounds`` extra copies and ``residual`` more go to selected experts.
Candidates (all with exactly the budget, each expert at most once per round):

* ``grouped``  -- the reference's construction: experts are split into
  equal-size affinity groups of size gcd(E, residual) (from a partition), and
  the bounded DP keeps the highest-demand fixed-cardinality group subsets;
* ``greedy``   -- classic max-load-per-copy greedy (an expert with demand d and
  c copies has per-copy load d/c; the next copy goes to the largest);
* ``top``      -- the ``residual`` highest-demand experts.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/allocation.py:24-109.
"""

from __future__ import annotations

import heapq
from collections.abc import Sequence

import numpy as np


def bounded_group_shortlist(groups: Sequence[np.ndarray], demand: np.ndarray, *, selected_groups: int,
                            candidate_limit: int) -> list[tuple[int, ...]]:
    """Best ``candidate_limit`` subsets of exactly ``selected_groups`` groups by total demand (DP over groups)."""
    if candidate_limit <= 0:
        raise ValueError("candidate_limit must be positive.")
    if not 0 <= selected_groups <= len(groups):
        raise ValueError("selected_groups is outside the available group range.")
    demand = np.asarray(demand, dtype=np.float64)
    scores = []
    for g in groups:
        g = np.asarray(g, dtype=np.int64)
        if g.ndim != 1 or (g < 0).any() or (g >= len(demand)).any():
            raise ValueError("Replica group contains an invalid logical expert ID.")
        scores.append(float(demand[g].sum()))
    # table[c] = best (score, subset) lists with c groups chosen so far
    table: list[list[tuple[float, tuple[int, ...]]]] = [[(0.0, ())]] + [[] for _ in range(selected_groups)]
    for gi, sc in enumerate(scores):
        for c in range(min(selected_groups, gi + 1), 0, -1):
            merged = table[c] + [(v + sc, sub + (gi,)) for v, sub in table[c - 1]]
            merged.sort(key=lambda row: (-row[0], row[1]))
            table[c] = merged[:candidate_limit]
    return [sub for _, sub in table[selected_groups]]


def grouped_allocations(partitions: Sequence[np.ndarray], demand: np.ndarray, *, additional_copies: int,
                        candidate_limit: int) -> list[np.ndarray]:
    demand = np.asarray(demand, dtype=np.float64)
    e = len(demand)
    if e == 0:
        raise ValueError("demand must contain one value per logical expert.")
    if additional_copies < 0:
        raise ValueError("additional_copies must be non-negative.")
    rounds, residual = divmod(additional_copies, e)
    full = np.tile(np.arange(e, dtype=np.int64), rounds)
    if residual == 0:
        return [full]
    gsize = int(np.gcd(e, residual))
    ngroups = e // gsize
    pick = residual // gsize
    out, seen = [], set()
    for part in partitions:
        part = np.asarray(part, dtype=np.int64)
        if part.shape != (e,):
            raise ValueError("Each partition must contain one label per logical expert.")
        if not np.array_equal(np.unique(part), np.arange(ngroups)):
            raise ValueError("Partition labels must be consecutive and match the required group count.")
        groups = [np.flatnonzero(part == g) for g in range(ngroups)]
        if any(len(g) != gsize for g in groups):
            raise ValueError("Replica allocation requires equal-capacity expert groups.")
        for combo in bounded_group_shortlist(groups, demand, selected_groups=pick, candidate_limit=candidate_limit):
            extra = np.sort(np.concatenate([groups[i] for i in combo]))
            alloc = np.concatenate([full, extra]).astype(np.int64)
            key = alloc.tobytes()
            if key not in seen:
                seen.add(key)
                out.append((-float(demand[extra].sum()), key, alloc))
    out.sort(key=lambda r: (r[0], r[1]))
    return [a for _, _, a in out[:candidate_limit]]


def greedy_allocation(demand: np.ndarray, additional_copies: int, max_copies: int | None = None) -> np.ndarray:
    """Extra-copy list by largest per-copy load first (ties -> lower expert id)."""
    demand = np.asarray(demand, dtype=np.float64)
    e = len(demand)
    copies = np.ones(e, dtype=np.int64)
    heap = [(-demand[x], x) for x in range(e)]
    heapq.heapify(heap)
    extra = []
    cap = max_copies if max_copies is not None else e + additional_copies
    while len(extra) < additional_copies and heap:
        neg, x = heapq.heappop(heap)
        if copies[x] >= cap:
            continue
        copies[x] += 1
        extra.append(x)
        heapq.heappush(heap, (-demand[x] / copies[x], x))
    if len(extra) != additional_copies:
        raise ValueError("copy cap too small for the additional-copy budget")
    return np.sort(np.asarray(extra, dtype=np.int64))


def top_demand_allocation(demand: np.ndarray, additional_copies: int) -> np.ndarray:
    demand = np.asarray(demand, dtype=np.float64)
    e = len(demand)
    rounds, residual = divmod(additional_copies, e)
    order = np.lexsort((np.arange(e), -demand))
    return np.sort(np.concatenate([np.tile(np.arange(e), rounds), order[:residual]]).astype(np.int64))


def candidate_allocations(demand: np.ndarray, additional_copies: int, *, partitions: Sequence[np.ndarray] = (),
                          candidate_limit: int = 4, max_copies: int | None = None) -> list[np.ndarray]:
    """Deduplicated union of grouped, greedy and top-demand allocations."""
    rows: list[np.ndarray] = []
    if partitions:
        rows += grouped_allocations(partitions, demand, additional_copies=additional_copies,
                                    candidate_limit=candidate_limit)
    rows.append(greedy_allocation(demand, additional_copies, max_copies))
    rows.append(top_demand_allocation(demand, additional_copies))
    seen, out = set(), []
    for r in rows:
        k = np.sort(r).tobytes()
        if k not in seen:
            seen.add(k)
            out.append(np.sort(r))
    return out


def instances_from_allocation(num_experts: int, extra: np.ndarray) -> np.ndarray:
    """Logical expert of every instance: one base copy per expert followed by the extra copies."""
    return np.concatenate([np.arange(num_experts, dtype=np.int64), np.asarray(extra, dtype=np.int64)])
