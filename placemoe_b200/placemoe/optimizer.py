"""Layout / mapping alternation of the PlaceMoE optimizer.

``optimize_replica_allocation`` -- full (L, M) planning for one layer:

    for every replica-allocation candidate (grouped / greedy / top-demand):
        instance statistics <- uniform split of the logical statistics
        for each layout/mapping alternation:
            placement candidates (partition of instances onto GPUs)
            for each placement: fresh mapping (greedy init) and, from the second alternation on,
                the carried mapping of the incumbent, each refined by the
                coordinate-descent core
            plus proposals from the fresh seed: scale-normalised mappings (one
                per assignment weight) and a community block mapping (experts with
                the same copy GPUs move as one block, rows counted exactly from
                the token community masks)
            every candidate is scored by the exact route-replay evaluator;
            the incumbent only changes on strict improvement (monotone)
            instance statistics <- projection through the incumbent mapping

``optimize_fixed_layout_mapping`` -- mapping-only update for a fixed layout L
(hot updates between full re-plans).

Reference parity: veomni/distributed/moe/hiermoe/placemoe/optimizer.py:32-383.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .allocation import candidate_allocations, instances_from_allocation
from .evaluator import PlanCost, RouteReplayEvaluator
from .mapping import (community_mask_histogram, copy_set_communities, initialize_mapping, optimize_community_mapping,
                      optimize_mapping, optimize_mapping_normalized)
from .materialize import layout_from_ranks, materialize_plan
from .partition import expert_groups_for_allocation
from .placement import PlacementConfig, place_instances
from .seeds import eplb_plan, fixed_ep_plan
from .statistics import project_statistics_to_copies
from .types import LayerPlan, PlaceMoETopology, ProfileStatistics


@dataclass(frozen=True)
class OptimizerConfig:
    rounds: int = 2
    placement_candidates: int = 2
    allocation_candidates: int = 3
    mapping_sweeps: int = 8
    partition_restarts: int = 2
    exchange_limit: int = 256
    seed: int = 0
    include_baselines: bool = True
    # scale-normalised mapping proposals (one per assignment weight) and the community block proposal
    normalized_weights: tuple = (0.5, 2.0)
    community_mapping: bool = True

    def __post_init__(self):
        if self.rounds <= 0 or self.placement_candidates <= 0 or self.allocation_candidates <= 0:
            raise ValueError("optimizer counts must be positive")


@dataclass(frozen=True)
class OptimizerCandidate:
    plan: LayerPlan
    cost: PlanCost
    label: str


@dataclass
class OptimizationResult:
    candidates: list[OptimizerCandidate] = field(default_factory=list)
    history: list[float] = field(default_factory=list)

    @property
    def best(self) -> OptimizerCandidate:
        return min(self.candidates, key=lambda c: (c.cost.total_ms, c.label))


def _instance_stats(stats: ProfileStatistics, inst: np.ndarray, mapping_inst: np.ndarray | None):
    """Per-instance demand [I] and affinity [I, I] (summed over sources)."""
    if mapping_inst is None:
        from .statistics import uniform_copy_statistics

        d, a = uniform_copy_statistics(stats, inst)
    else:
        d, a = project_statistics_to_copies(stats, inst, mapping_inst)
    return d.sum(0), a.sum(0)


def _instance_mapping_from_slots(mapping_slots: np.ndarray, slot_of_inst: np.ndarray) -> np.ndarray:
    inv = np.full(slot_of_inst.max() + 1, -1, dtype=np.int64)
    inv[slot_of_inst] = np.arange(len(slot_of_inst))
    return inv[mapping_slots]


def optimize_replica_allocation(stats: ProfileStatistics, topology: PlaceMoETopology,
                                evaluator: RouteReplayEvaluator, cfg: OptimizerConfig = OptimizerConfig(),
                                log=None) -> OptimizationResult:
    e = topology.num_experts
    if stats.num_experts != e or stats.ep_size != topology.ep_size:
        raise ValueError("statistics do not match the topology")
    omega, gamma, local_w = evaluator.coefficients()
    slot_rank = topology.slot_ranks()
    res = OptimizationResult()
    incumbent: OptimizerCandidate | None = None

    def consider(plan: LayerPlan, label: str) -> OptimizerCandidate:
        nonlocal incumbent
        cand = OptimizerCandidate(plan, evaluator.evaluate(plan), label)
        res.candidates.append(cand)
        if incumbent is None or cand.cost.total_ms < incumbent.cost.total_ms - 1e-12:
            incumbent = cand
        res.history.append(incumbent.cost.total_ms)
        if log:
            log(f"  {label}: {cand.cost.total_ms:.4f} ms (best {incumbent.cost.total_ms:.4f})")
        return cand

    if cfg.include_baselines:
        if topology.slots_per_rank * topology.ep_size >= e and -(-e // topology.ep_size) <= topology.slots_per_rank:
            consider(fixed_ep_plan(topology), "fixed-ep")
        if topology.extra_copies > 0:
            consider(eplb_plan(topology, stats.demand), "eplb")

    extra = topology.extra_copies
    partitions = []
    residual = extra % e
    if residual:
        gsize = int(np.gcd(e, residual))
        partitions = expert_groups_for_allocation(stats.expert_affinity, stats.expert_demand, gsize, cfg.seed,
                                                  cfg.partition_restarts)
    allocations = candidate_allocations(stats.expert_demand, extra, partitions=partitions,
                                        candidate_limit=cfg.allocation_candidates,
                                        max_copies=topology.ep_size)[: cfg.allocation_candidates + 2]
    pcfg = PlacementConfig(topology.ep_size, topology.ranks_per_node, topology.slots_per_rank, omega, gamma,
                           restarts=cfg.partition_restarts, exchange_limit=cfg.exchange_limit, seed=cfg.seed)
    for ai, alloc in enumerate(allocations):
        inst = instances_from_allocation(e, alloc)
        if np.bincount(inst, minlength=e).max() > topology.ep_size:
            continue
        mapping_inst = None
        carried: np.ndarray | None = None
        for rnd in range(cfg.rounds):
            inst_d, inst_a = _instance_stats(stats, inst, mapping_inst)
            for pi, place in enumerate(place_instances(inst, inst_d, inst_a, pcfg, cfg.placement_candidates)):
                layout, slot_of = layout_from_ranks(inst, place.instance_ranks, topology)
                seeds = [initialize_mapping(stats.demand, layout, slot_rank, topology.ep_size)]
                if carried is not None and np.array_equal(layout[carried], np.broadcast_to(np.arange(e), carried.shape)):
                    seeds.append(carried)
                for si, m0 in enumerate(seeds):
                    m, _ = optimize_mapping(stats.demand, stats.affinity, layout, slot_rank, m0, omega=omega,
                                            gamma=gamma, local_weight=local_w, sweeps=cfg.mapping_sweeps)
                    plan = materialize_plan(layout, m, stats.demand, topology)
                    consider(plan, f"alloc{ai}/round{rnd}/place{pi}:{place.seed_name}/map{si}")
                tag = f"alloc{ai}/round{rnd}/place{pi}:{place.seed_name}"
                for label, m in _mapping_proposals(stats, layout, slot_rank, seeds[0], topology, evaluator, cfg):
                    consider(materialize_plan(layout, m, stats.demand, topology), f"{tag}/{label}")
            if incumbent is not None and incumbent.label.startswith(f"alloc{ai}/"):
                p = incumbent.plan
                carried = p.source_logical_to_physical.copy()
                inst_of_slot = np.full(topology.total_slots, -1, dtype=np.int64)
                # instance index of every slot of the incumbent layout (re-derived from its own layout)
                inst = np.array([x for x in p.slot_to_logical.tolist() if x >= 0], dtype=np.int64)
                order = np.flatnonzero(p.slot_to_logical >= 0)
                inst_of_slot[order] = np.arange(len(order))
                mapping_inst = inst_of_slot[carried]
    return res


def _mapping_proposals(stats: ProfileStatistics, layout: np.ndarray, slot_rank: np.ndarray, seed: np.ndarray,
                       topology: PlaceMoETopology, evaluator: RouteReplayEvaluator, cfg: OptimizerConfig):
    """(label, mapping) proposals beyond the calibrated descent, for the exact evaluator to judge."""
    out = []
    seen = set()
    for w in cfg.normalized_weights:
        m, _ = optimize_mapping_normalized(stats.demand, stats.affinity, layout, slot_rank, seed,
                                           ranks_per_node=topology.ranks_per_node, assignment_weight=w,
                                           sweeps=cfg.mapping_sweeps)
        if m.tobytes() not in seen:
            seen.add(m.tobytes())
            out.append((f"normalized{w:g}", m))
    if cfg.community_mapping and topology.extra_copies > 0:
        comm = copy_set_communities(layout, slot_rank, topology.num_experts)
        if comm is not None:
            c = int(comm.max()) + 1
            flat = [r for step in evaluator.samples for r in step]
            hist = community_mask_histogram(flat, comm, ranks_per_unit=1, num_communities=c,
                                            sources_per_step=topology.ep_size)
            asg = np.zeros((topology.ep_size, c))
            for k in range(c):
                asg[:, k] = stats.demand[:, comm == k].sum(axis=1)
            omega, gamma, _ = evaluator.coefficients()
            res = optimize_community_mapping(layout, slot_rank, comm, asg, hist, ranks_per_unit=1,
                                             comm_ms_per_token=omega, ms_per_assignment=gamma)
            if res.mapping.tobytes() not in seen:
                out.append(("community", res.mapping))
    return out


def optimize_fixed_layout_mapping(stats: ProfileStatistics, topology: PlaceMoETopology, layout_plan: LayerPlan,
                                  evaluator: RouteReplayEvaluator, cfg: OptimizerConfig = OptimizerConfig()
                                  ) -> OptimizationResult:
    """Mapping-only refresh: L and its owners stay, M is re-optimised (monotone vs. the current M)."""
    omega, gamma, local_w = evaluator.coefficients()
    slot_rank = topology.slot_ranks()
    layout = layout_plan.slot_to_logical
    res = OptimizationResult()
    best = OptimizerCandidate(layout_plan, evaluator.evaluate(layout_plan), "current")
    res.candidates.append(best)
    for si, m0 in enumerate([layout_plan.source_logical_to_physical,
                             initialize_mapping(stats.demand, layout, slot_rank, topology.ep_size)]):
        m, _ = optimize_mapping(stats.demand, stats.affinity, layout, slot_rank, m0, omega=omega, gamma=gamma,
                                local_weight=local_w, sweeps=cfg.mapping_sweeps)
        plan = LayerPlan(layout, m, layout_plan.owner_slots)
        plan.validate(topology)
        cand = OptimizerCandidate(plan, evaluator.evaluate(plan), f"mapping{si}")
        res.candidates.append(cand)
    seed = initialize_mapping(stats.demand, layout, slot_rank, topology.ep_size)
    for label, m in _mapping_proposals(stats, layout, slot_rank, seed, topology, evaluator, cfg):
        plan = LayerPlan(layout, m, layout_plan.owner_slots)
        plan.validate(topology)
        res.candidates.append(OptimizerCandidate(plan, evaluator.evaluate(plan), label))
    return res
