"""Capacity-constrained partition of expert instances into groups (GPUs).

Objective (same calibrated form as the reference):
    -omega * (affinity inside groups) + gamma * max_g load_g / ranks_g
Seeds: spectral embedding of the normalised affinity -> KMeans centres ->
capacity-exact assignment (Hungarian on distances to capacity-repeated
centres), a longest-processing-time load-balanced seed and a round-robin seed.
Every seed is repaired so that no group holds two copies of one expert, then
refined by pairwise exchanges in the C++ core (``refine_partition``).

Reference parity: veomni/distributed/moe/hiermoe/placemoe/partition.py:27-426
(spectral seed :131, capacity assignment :140, exchange refinement :160).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .._build import load_planner


@dataclass(frozen=True)
class PartitionConfig:
    capacities: tuple[int, ...]
    ranks_per_group: tuple[int, ...]
    omega: float
    gamma: float
    restarts: int = 3
    assignment_iterations: int = 12
    exchange_limit: int = 256
    seed: int = 0

    def __post_init__(self):
        if not self.capacities or any(c <= 0 for c in self.capacities):
            raise ValueError("Partition capacities must be positive.")
        if len(self.ranks_per_group) != len(self.capacities):
            raise ValueError("Each partition group must define its rank count.")
        if any(r <= 0 for r in self.ranks_per_group):
            raise ValueError("Ranks per partition group must be positive.")
        if self.omega < 0 or self.gamma < 0:
            raise ValueError("Calibrated partition coefficients must be non-negative.")


@dataclass(frozen=True)
class PartitionResult:
    labels: np.ndarray
    objective: float
    within_affinity: float
    peak_load_per_rank: float
    exchanges: int
    seed_name: str


def partition_objective(affinity, demand, labels, cfg: PartitionConfig) -> tuple[float, float, float]:
    labels = np.asarray(labels, dtype=np.int64)
    g = len(cfg.capacities)
    if not np.array_equal(np.bincount(labels, minlength=g), np.asarray(cfg.capacities)):
        raise ValueError("Partition labels do not satisfy the configured capacities.")
    same = labels[:, None] == labels[None, :]
    within = float(np.triu(np.where(same, affinity, 0.0), 1).sum())
    loads = np.bincount(labels, weights=demand, minlength=g) / np.asarray(cfg.ranks_per_group, dtype=np.float64)
    peak = float(loads.max(initial=0.0))
    return -cfg.omega * within + cfg.gamma * peak, within, peak


def spectral_embedding(affinity: np.ndarray, dims: int) -> np.ndarray:
    deg = np.maximum(affinity.sum(1), 1.0)
    norm = affinity / np.sqrt(deg[:, None] * deg[None, :])
    vals, vecs = np.linalg.eigh(norm)
    emb = vecs[:, np.argsort(vals)[-dims:]]
    return emb / np.maximum(np.linalg.norm(emb, axis=1, keepdims=True), 1e-12)


def _kmeans_centers(x: np.ndarray, k: int, seed: int, iters: int = 100) -> np.ndarray:
    """Lloyd's k-means with k-means++ seeding (Arthur & Vassilvitskii, 2007) on a few hundred points:
    small enough for numpy, and it keeps the planner processes free of a heavyweight import."""
    rng = np.random.default_rng(seed)
    n = x.shape[0]
    centers = np.empty((k, x.shape[1]), dtype=np.float64)
    centers[0] = x[rng.integers(n)]
    d2 = ((x - centers[0]) ** 2).sum(1)
    for c in range(1, k):
        total = d2.sum()
        i = int(rng.choice(n, p=d2 / total)) if total > 0 else int(rng.integers(n))
        centers[c] = x[i]
        d2 = np.minimum(d2, ((x - centers[c]) ** 2).sum(1))
    for _ in range(iters):
        lab = ((x[:, None, :] - centers[None, :, :]) ** 2).sum(-1).argmin(1)
        new = np.stack([x[lab == c].mean(0) if (lab == c).any() else centers[c] for c in range(k)])
        if np.allclose(new, centers):
            break
        centers = new
    return centers


def _capacity_assign(emb: np.ndarray, cfg: PartitionConfig, seed: int) -> np.ndarray:
    from scipy.optimize import linear_sum_assignment

    g = len(cfg.capacities)
    centers = _kmeans_centers(np.asarray(emb, dtype=np.float64), g, seed)
    slot_group = np.repeat(np.arange(g), cfg.capacities)
    labels = np.zeros(emb.shape[0], dtype=np.int64)
    for _ in range(cfg.assignment_iterations):
        dist = ((emb[:, None, :] - centers[slot_group][None, :, :]) ** 2).sum(-1)
        rows, cols = linear_sum_assignment(dist)
        labels[rows] = slot_group[cols]
        new = np.stack([emb[labels == k].mean(0) if (labels == k).any() else centers[k] for k in range(g)])
        if np.allclose(new, centers):
            break
        centers = new
    return labels


def _lpt_seed(demand: np.ndarray, item_expert: np.ndarray, cfg: PartitionConfig) -> np.ndarray:
    g = len(cfg.capacities)
    cap = np.asarray(cfg.capacities).copy()
    load = np.zeros(g)
    labels = np.full(len(demand), -1, dtype=np.int64)
    held: list[set] = [set() for _ in range(g)]
    for i in np.lexsort((np.arange(len(demand)), -demand)):
        order = np.lexsort((np.arange(g), load / np.asarray(cfg.ranks_per_group)))
        choice = next((k for k in order if cap[k] > 0 and item_expert[i] not in held[k]), None)
        if choice is None:
            choice = next(k for k in order if cap[k] > 0)
        labels[i] = choice
        cap[choice] -= 1
        load[choice] += demand[i]
        held[choice].add(int(item_expert[i]))
    return labels


def _round_robin_seed(n: int, cfg: PartitionConfig) -> np.ndarray:
    return np.repeat(np.arange(len(cfg.capacities)), cfg.capacities)[:n].astype(np.int64)


def repair_duplicates(labels: np.ndarray, item_expert: np.ndarray, demand: np.ndarray) -> np.ndarray:
    """Swap items until no group holds two copies of the same expert (keeps capacities)."""
    labels = labels.copy()
    n = len(labels)
    for _ in range(4 * n):
        bad = None
        seen = {}
        for i in range(n):
            key = (int(labels[i]), int(item_expert[i]))
            if key in seen:
                bad = i
                break
            seen[key] = i
        if bad is None:
            return labels
        gi, ei = labels[bad], item_expert[bad]
        fixed = False
        for j in np.argsort(demand):
            gj = labels[j]
            if gj == gi:
                continue
            if (labels[item_expert == ei] == gj).any():
                continue
            if (labels[item_expert == item_expert[j]] == gi).any() and item_expert[j] != ei:
                continue
            labels[bad], labels[j] = gj, gi
            fixed = True
            break
        if not fixed:
            break
    return labels


def partition_items(affinity: np.ndarray, demand: np.ndarray, item_expert: np.ndarray,
                    cfg: PartitionConfig) -> list[PartitionResult]:
    """All refined seeds, best first."""
    affinity = np.asarray(affinity, dtype=np.float64)
    demand = np.asarray(demand, dtype=np.float64)
    item_expert = np.asarray(item_expert, dtype=np.int64)
    n = len(demand)
    if n != sum(cfg.capacities):
        raise ValueError("Demand length must equal the total partition capacity.")
    if affinity.shape != (n, n):
        raise ValueError("Affinity must be a square matrix matching the demand length.")
    seeds: list[tuple[str, np.ndarray]] = [("lpt", _lpt_seed(demand, item_expert, cfg)),
                                           ("round_robin", _round_robin_seed(n, cfg))]
    g = len(cfg.capacities)
    if g > 1 and affinity.sum() > 0:
        emb = spectral_embedding(affinity, min(g, n - 1))
        for r in range(cfg.restarts):
            seeds.append((f"spectral{r}", _capacity_assign(emb, cfg, cfg.seed + r)))
    core = load_planner()
    out, seen = [], set()
    ranks = torch.tensor(cfg.ranks_per_group, dtype=torch.float64)
    for name, lab in seeds:
        lab = repair_duplicates(lab, item_expert, demand)
        lt = torch.from_numpy(lab.copy())
        ex = core.refine_partition(torch.from_numpy(affinity), torch.from_numpy(demand), lt,
                                   torch.from_numpy(item_expert), ranks, float(cfg.omega), float(cfg.gamma),
                                   int(cfg.exchange_limit))
        lab = lt.numpy().copy()
        key = lab.tobytes()
        if key in seen:
            continue
        seen.add(key)
        obj, within, peak = partition_objective(affinity, demand, lab, cfg)
        out.append(PartitionResult(lab, obj, within, peak, int(ex), name))
    out.sort(key=lambda r: (r.objective, r.seed_name))
    return out


def expert_groups_for_allocation(affinity: np.ndarray, demand: np.ndarray, group_size: int, seed: int = 0,
                                 restarts: int = 2) -> list[np.ndarray]:
    """Equal-size affinity groups of logical experts (inputs of the grouped allocation)."""
    e = len(demand)
    if e % group_size:
        raise ValueError("group size must divide the number of experts")
    ng = e // group_size
    if ng == 1:
        return [np.zeros(e, dtype=np.int64)]
    cfg = PartitionConfig(capacities=(group_size,) * ng, ranks_per_group=(1,) * ng, omega=1.0, gamma=0.0,
                          restarts=restarts, seed=seed, exchange_limit=64)
    res = partition_items(affinity, demand, np.full(e, -1, dtype=np.int64), cfg)
    return [r.labels for r in res[:restarts + 1]]
