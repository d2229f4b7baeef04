"""Placement of expert instances onto GPUs.

``place_instances`` assigns each instance (a copy of a logical expert) to an
EP rank with exactly ``slots_per_rank`` instances per rank and no rank holding
two copies of the same expert.  With ``ranks_per_node < ep_size`` (several
nodes) it partitions instances over nodes first and then over the ranks of
each node; on one NVSwitch domain (``ranks_per_node == ep_size``) the node
level is trivial and only the rank-level partition runs.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/placement.py:29-513
(hierarchical placement, duplicate repair :255-326).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .partition import PartitionConfig, partition_items, repair_duplicates


@dataclass(frozen=True)
class PlacementConfig:
    ep_size: int
    ranks_per_node: int
    slots_per_rank: int
    omega: float
    gamma: float
    restarts: int = 2
    exchange_limit: int = 256
    seed: int = 0

    @property
    def num_nodes(self) -> int:
        return self.ep_size // self.ranks_per_node


@dataclass(frozen=True)
class PlacementResult:
    instance_ranks: np.ndarray  # [instances] rank of each instance
    objective: float
    seed_name: str


def rank_placement_is_unique(instance_ranks: np.ndarray, instance_expert: np.ndarray) -> bool:
    pairs = set()
    for r, e in zip(instance_ranks.tolist(), instance_expert.tolist()):
        if (r, e) in pairs:
            return False
        pairs.add((r, e))
    return True


def place_instances(instance_expert: np.ndarray, inst_demand: np.ndarray, inst_affinity: np.ndarray,
                    cfg: PlacementConfig, max_candidates: int = 3) -> list[PlacementResult]:
    inst_expert = np.asarray(instance_expert, dtype=np.int64)
    n = len(inst_expert)
    if n != cfg.ep_size * cfg.slots_per_rank:
        raise ValueError("instances must fill every physical slot exactly")
    results: list[PlacementResult] = []
    if cfg.num_nodes == 1:
        pcfg = PartitionConfig(capacities=(cfg.slots_per_rank,) * cfg.ep_size, ranks_per_group=(1,) * cfg.ep_size,
                               omega=cfg.omega, gamma=cfg.gamma, restarts=cfg.restarts,
                               exchange_limit=cfg.exchange_limit, seed=cfg.seed)
        for r in partition_items(inst_affinity, inst_demand, inst_expert, pcfg)[:max_candidates]:
            if rank_placement_is_unique(r.labels, inst_expert):
                results.append(PlacementResult(r.labels.copy(), r.objective, r.seed_name))
        return results
    # two levels: nodes, then ranks inside every node
    ncfg = PartitionConfig(capacities=(cfg.ranks_per_node * cfg.slots_per_rank,) * cfg.num_nodes,
                           ranks_per_group=(cfg.ranks_per_node,) * cfg.num_nodes, omega=cfg.omega, gamma=cfg.gamma,
                           restarts=cfg.restarts, exchange_limit=cfg.exchange_limit, seed=cfg.seed)
    for nres in partition_items(inst_affinity, inst_demand, np.full(n, -1), ncfg)[:max_candidates]:
        ranks = np.zeros(n, dtype=np.int64)
        total = nres.objective
        for node in range(cfg.num_nodes):
            members = np.flatnonzero(nres.labels == node)
            rcfg = PartitionConfig(capacities=(cfg.slots_per_rank,) * cfg.ranks_per_node,
                                   ranks_per_group=(1,) * cfg.ranks_per_node, omega=cfg.omega, gamma=cfg.gamma,
                                   restarts=cfg.restarts, exchange_limit=cfg.exchange_limit, seed=cfg.seed)
            sub = partition_items(inst_affinity[np.ix_(members, members)], inst_demand[members],
                                  inst_expert[members], rcfg)[0]
            ranks[members] = node * cfg.ranks_per_node + sub.labels
        ranks = repair_duplicates(ranks, inst_expert, inst_demand)
        if rank_placement_is_unique(ranks, inst_expert):
            results.append(PlacementResult(ranks, total, f"hier-{nres.seed_name}"))
    return results
