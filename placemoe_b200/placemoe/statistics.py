"""Route statistics for the planner.

``profile_route_statistics(samples, num_experts)``: samples is a sequence of
steps, each a sequence (one per source rank) of ``[tokens, top_k]`` logical
routes.  Returns demand[s, e] (assignments from s to e) and the co-selection
affinity[s, i, j] (tokens on s choosing both i and j).  The per-token pair
accumulation runs in the C++ core (``csrc/planner/route_stats.cpp``).

``uniform_copy_statistics`` splits logical statistics evenly over copies (used
before a mapping exists); ``project_statistics_to_copies`` routes them through
a mapping M.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/statistics.py:30-140.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from .._build import load_planner
from .types import EMPTY_EXPERT, ProfileStatistics


def profile_route_statistics(samples: Sequence[Sequence], *, num_experts: int) -> ProfileStatistics:
    if not samples or not samples[0]:
        raise ValueError("At least one routing sample and source rank are required.")
    if num_experts <= 0:
        raise ValueError("num_experts must be positive.")
    ep = len(samples[0])
    demand = torch.zeros(ep, num_experts, dtype=torch.float64)
    affinity = torch.zeros(ep, num_experts, num_experts, dtype=torch.float64)
    core = load_planner()
    for sample in samples:
        if len(sample) != ep:
            raise ValueError("All routing samples must contain the same source ranks.")
        for s, route in enumerate(sample):
            r = torch.as_tensor(route)
            if r.ndim != 2 or r.shape[1] <= 0:
                raise ValueError("Each route tensor must have shape [tokens, top_k].")
            core.accumulate_route_stats(r.detach().cpu().to(torch.int64).contiguous(), s, demand, affinity)
    return ProfileStatistics(demand=demand.numpy(), affinity=affinity.numpy())


def _copy_counts(copy_to_expert: np.ndarray, num_experts: int) -> np.ndarray:
    if (copy_to_expert < EMPTY_EXPERT).any() or (copy_to_expert >= num_experts).any():
        raise ValueError("copy_to_expert contains an invalid logical expert ID.")
    counts = np.bincount(copy_to_expert[copy_to_expert >= 0], minlength=num_experts)
    if (counts < 1).any():
        raise ValueError("Every logical expert must retain at least one physical copy.")
    return counts


def uniform_copy_statistics(stats: ProfileStatistics, copy_to_expert) -> tuple[np.ndarray, np.ndarray]:
    c2e = np.asarray(copy_to_expert, dtype=np.int64)
    counts = _copy_counts(c2e, stats.num_experts)
    n = len(c2e)
    act = np.flatnonzero(c2e >= 0)
    demand = np.zeros((stats.ep_size, n))
    demand[:, act] = stats.demand[:, c2e[act]] / counts[c2e[act]][None, :]
    affinity = np.zeros((stats.ep_size, n, n))
    ea = c2e[act]
    sub = stats.affinity[:, ea][:, :, ea] / (counts[ea][:, None] * counts[ea][None, :])[None]
    same = ea[:, None] == ea[None, :]
    sub[:, same] = 0.0
    affinity[np.ix_(np.arange(stats.ep_size), act, act)] = sub
    return demand, affinity


def project_statistics_to_copies(stats: ProfileStatistics, copy_to_expert, mapping) -> tuple[np.ndarray, np.ndarray]:
    c2e = np.asarray(copy_to_expert, dtype=np.int64)
    m = np.asarray(mapping, dtype=np.int64)
    _copy_counts(c2e, stats.num_experts)
    if m.shape != (stats.ep_size, stats.num_experts):
        raise ValueError("mapping must have shape [source_rank, logical_expert].")
    if (m < 0).any() or (m >= len(c2e)).any():
        raise ValueError("mapping references an unavailable physical copy.")
    if not np.array_equal(c2e[m], np.broadcast_to(np.arange(stats.num_experts), m.shape)):
        raise ValueError("mapping references a copy of the wrong logical expert.")
    n = len(c2e)
    demand = np.zeros((stats.ep_size, n))
    affinity = np.zeros((stats.ep_size, n, n))
    for s in range(stats.ep_size):
        sel = m[s]
        np.add.at(demand[s], sel, stats.demand[s])
        # affinity between the copies chosen for (i, j); P^T A P with P the selection matrix
        p = np.zeros((stats.num_experts, n))
        p[np.arange(stats.num_experts), sel] = 1.0
        affinity[s] = p.T @ stats.affinity[s] @ p
        np.fill_diagonal(affinity[s], 0.0)
    return demand, affinity
