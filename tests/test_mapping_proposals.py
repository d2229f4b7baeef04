"""Mapping proposals beyond the calibrated coordinate descent: scale-normalised mappings and the community
block mapping (C++ cores), their invariants, and their place in the layout / mapping alternation.

The first four cases restate the invariant tests of the reference's
tests/distributed/test_placemoe_optimizer.py (community block moves, intersection hits, bounded row search,
the communication / compute trade-off of normalised proposals) against this implementation's API.
"""

import numpy as np
import torch

from placemoe_b200.placemoe.mapping import (community_intersection_hits, community_mask_histogram,
                                            copy_set_communities, initialize_mapping, optimize_community_mapping,
                                            optimize_mapping_normalized)
from placemoe_b200.placemoe.types import ProfileStatistics


def test_community_mapping_moves_co_selected_experts_as_one_block():
    layout = np.array([0, 0, 1, 1, 2, 2, 3, 3])
    slot_unit = np.array([0, 1, 0, 1, 1, 2, 1, 2])
    communities = np.array([0, 0, 1, 1])
    assignments = np.zeros((4, 2))
    assignments[3] = [20, 20]
    masks = np.zeros((4, 4), dtype=np.int64)
    masks[3, 3] = 10  # ten tokens of unit 3 use both communities
    res = optimize_community_mapping(layout, slot_unit, communities, assignments, masks, ranks_per_unit=1,
                                     comm_ms_per_token=1.0, ms_per_assignment=0.0)
    assert res.destination_units[3].tolist() == [1, 1]  # one destination: each token is sent once
    assert slot_unit[res.mapping[3]].tolist() == [1, 1, 1, 1]
    assert res.proxy_cost == 10


def test_community_intersection_hits_match_mask_unions():
    hist = np.array([[0, 2, 3, 5]], dtype=np.int64)
    assert community_intersection_hits(hist).tolist() == [[0, 7, 8, 10]]
    rng = np.random.default_rng(0)
    hist = rng.integers(0, 50, size=(3, 32))
    hits = community_intersection_hits(hist)
    masks = np.arange(32)
    for u in range(3):
        for x in range(32):
            assert hits[u, x] == hist[u, (masks & x) != 0].sum()


def test_community_mapping_bounds_large_source_row_search():
    c = 13
    layout = np.repeat(np.arange(c), 2)
    slot_unit = np.tile(np.arange(2), c)
    masks = np.zeros((2, 1 << c), dtype=np.int64)
    masks[:, -1] = 1
    res = optimize_community_mapping(layout, slot_unit, np.arange(c), np.ones((2, c)), masks, ranks_per_unit=1,
                                     comm_ms_per_token=1.0, ms_per_assignment=0.0, row_limit=4, beam_width=4)
    assert res.mapping.shape == (2, c) and res.destination_units.shape == (2, c)
    # every token of a unit uses all communities: one destination unit for all of them is optimal
    for u in range(2):
        assert len(set(res.destination_units[u].tolist())) == 1


def test_normalized_proposals_span_communication_and_compute():
    aff = np.zeros((2, 2, 2))
    aff[0, 0, 1] = aff[0, 1, 0] = 30
    stats = ProfileStatistics(demand=np.array([[10.0, 1.0], [0.0, 10.0]]), affinity=aff)
    layout, slot_rank = np.array([0, 0, 1]), np.array([0, 1, 1])
    m0 = initialize_mapping(stats.demand, layout, slot_rank, 2)
    comm_only, peak_c = optimize_mapping_normalized(stats.demand, stats.affinity, layout, slot_rank, m0,
                                                    ranks_per_node=1, assignment_weight=0.0)
    balanced, peak_b = optimize_mapping_normalized(stats.demand, stats.affinity, layout, slot_rank, m0,
                                                   ranks_per_node=1, assignment_weight=100.0)
    assert comm_only[0, 0] == 1 and peak_c == 21  # follow the co-selected expert to GPU 1
    assert balanced[0, 0] == 0 and peak_b == 11  # keep the load balanced


def test_mask_histogram_and_copy_set_communities():
    layout = np.array([0, 1, 2, 0])  # expert 0 on GPUs 0 and 1; 1 on GPU 0; 2 on GPU 1 (2 slots per GPU)
    slot_rank = np.array([0, 0, 1, 1])
    comm = copy_set_communities(layout, slot_rank, 3)
    assert comm.tolist() == [0, 1, 2]
    routes = [torch.tensor([[0, 1], [1, 2]]), torch.tensor([[2, 2], [0, 2]])]
    hist = community_mask_histogram(routes, comm, ranks_per_unit=1, num_communities=3)
    assert hist.shape == (2, 8)
    assert hist[0, 0b011] == 1 and hist[0, 0b110] == 1 and hist[1, 0b100] == 1 and hist[1, 0b101] == 1
    assert copy_set_communities(np.arange(40), np.arange(40) // 5, 40, max_communities=4) is None  # 8 sets
    # several steps in one call (sources_per_step each) equal the sum of the per-step histograms,
    # for int32 and int64 routes alike
    step2 = [torch.tensor([[1, 1], [0, 0]], dtype=torch.int32), torch.tensor([[1, 2]], dtype=torch.int32)]
    both = community_mask_histogram(routes + step2, comm, ranks_per_unit=1, num_communities=3, sources_per_step=2)
    assert np.array_equal(both, hist + community_mask_histogram(step2, comm, ranks_per_unit=1, num_communities=3))
    units = community_mask_histogram(routes + step2, comm, ranks_per_unit=2, num_communities=3, sources_per_step=2)
    assert units.shape == (1, 8) and np.array_equal(units[0], both.sum(0))


def test_proposals_join_the_alternation_and_never_lose():
    from placemoe_b200.placemoe.evaluator import RouteReplayEvaluator
    from placemoe_b200.placemoe.optimizer import OptimizerConfig, optimize_replica_allocation
    from placemoe_b200.placemoe.statistics import profile_route_statistics
    from placemoe_b200.placemoe.types import PlaceMoETopology

    g = torch.Generator().manual_seed(3)
    ep, e, k = 4, 16, 4
    w = torch.linspace(3.0, 0.2, e)
    steps = [[torch.multinomial(w.expand(256, e), k, generator=g) for _ in range(ep)] for _ in range(2)]
    topo = PlaceMoETopology(ep, ep, e, e // ep + 1)
    stats = profile_route_statistics(steps, num_experts=e)
    ev = RouteReplayEvaluator(steps, topo, hidden_size=1024, bytes_per_element=2)
    base = optimize_replica_allocation(stats, topo, ev, OptimizerConfig(normalized_weights=(), community_mapping=False))
    full = optimize_replica_allocation(stats, topo, ev, OptimizerConfig())
    labels = [c.label for c in full.candidates]
    assert any("normalized" in x for x in labels)
    assert full.best.cost.total_ms <= base.best.cost.total_ms + 1e-9
    for c in full.candidates:
        c.plan.validate(topo)
