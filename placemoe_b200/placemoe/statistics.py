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
    if num_experts < 1:
        raise ValueError(f"num_experts must be >= 1, got {num_experts}")
    if len(samples) == 0 or len(samples[0]) == 0:
        raise ValueError("route statistics need at least one step with at least one source GPU")
    gpus = len(samples[0])
    demand = torch.zeros(gpus, num_experts, dtype=torch.float64)
    affinity = torch.zeros(gpus, num_experts, num_experts, dtype=torch.float64)
    core = load_planner()
    for step, sample in enumerate(samples):
        if len(sample) != gpus:
            raise ValueError(f"step {step} has routes of {len(sample)} GPUs, step 0 of {gpus}")
        for src, route in enumerate(sample):
            ids = torch.as_tensor(route)
            if ids.dim() != 2 or ids.shape[1] == 0:
                raise ValueError(f"step {step}, GPU {src}: routes are [tokens, top_k], got {tuple(ids.shape)}")
            core.accumulate_route_stats(ids.detach().to("cpu", torch.int64).contiguous(), src, demand, affinity)
    return ProfileStatistics(demand=demand.numpy(), affinity=affinity.numpy())


def _copies_per_expert(copy_to_expert: np.ndarray, num_experts: int) -> np.ndarray:
    """Copies of each expert in a copy -> expert table (-1 = empty copy); every expert needs one."""
    bad = (copy_to_expert < EMPTY_EXPERT) | (copy_to_expert >= num_experts)
    if bad.any():
        raise ValueError(f"copy table holds ids outside [-1, {num_experts}): {copy_to_expert[bad][:4].tolist()}")
    counts = np.bincount(copy_to_expert[copy_to_expert != EMPTY_EXPERT], minlength=num_experts)
    if counts.min(initial=1) == 0:
        raise ValueError(f"experts without a copy: {np.flatnonzero(counts == 0)[:8].tolist()}")
    return counts


def uniform_copy_statistics(stats: ProfileStatistics, copy_to_expert) -> tuple[np.ndarray, np.ndarray]:
    """Statistics per copy when every copy of an expert takes an equal share (no mapping yet)."""
    c2e = np.asarray(copy_to_expert, dtype=np.int64)
    counts = _copies_per_expert(c2e, stats.num_experts)
    live = np.flatnonzero(c2e != EMPTY_EXPERT)
    experts = c2e[live]
    share = 1.0 / counts[experts]
    demand = np.zeros((stats.ep_size, len(c2e)))
    demand[:, live] = stats.demand[:, experts] * share[None, :]
    pair = stats.affinity[:, experts[:, None], experts[None, :]] * np.outer(share, share)[None]
    pair[:, experts[:, None] == experts[None, :]] = 0.0  # copies of one expert are never co-selected
    affinity = np.zeros((stats.ep_size, len(c2e), len(c2e)))
    affinity[:, live[:, None], live[None, :]] = pair
    return demand, affinity


def project_statistics_to_copies(stats: ProfileStatistics, copy_to_expert, mapping) -> tuple[np.ndarray, np.ndarray]:
    """Statistics per copy when GPU r sends expert e's tokens to copy ``mapping[r, e]``."""
    c2e = np.asarray(copy_to_expert, dtype=np.int64)
    m = np.asarray(mapping, dtype=np.int64)
    _copies_per_expert(c2e, stats.num_experts)
    if m.shape != (stats.ep_size, stats.num_experts):
        raise ValueError(f"mapping is [gpu, expert] = {(stats.ep_size, stats.num_experts)}, got {m.shape}")
    if ((m < 0) | (m >= len(c2e))).any() or not (c2e[m] == np.arange(stats.num_experts)[None, :]).all():
        raise ValueError("mapping must point every (gpu, expert) at a copy of that expert")
    n = len(c2e)
    demand = np.zeros((stats.ep_size, n))
    affinity = np.zeros((stats.ep_size, n, n))
    for src in range(stats.ep_size):
        chosen = m[src]
        np.add.at(demand[src], chosen, stats.demand[src])
        # co-selection moves with the chosen copies: scatter-add the expert pair matrix onto copy pairs
        np.add.at(affinity[src], (chosen[:, None], chosen[None, :]), stats.affinity[src])
        np.fill_diagonal(affinity[src], 0.0)
    return demand, affinity
