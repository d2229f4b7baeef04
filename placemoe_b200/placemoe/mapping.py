"""Source-aware token-to-copy mapping M[source_rank, logical_expert] -> physical slot.

``initialize_mapping``: demand-ordered greedy -- a source uses its own GPU's
copy when it has one, otherwise the copy whose rank currently carries the
least projected load.
``optimize_mapping``: coordinate descent in the C++ core with the objective
-omega*co-selection reuse - lambda*on-GPU demand + gamma*peak rank load.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/mapping.py:181-442.
"""

from __future__ import annotations

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
