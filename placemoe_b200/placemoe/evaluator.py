"""Exact route-replay cost of a plan on one NVSwitch level.

Every profiled token route is replayed through a mapping M: destination GPUs
are the ranks of the chosen copies; each remote GPU receives the token's
hidden row once (per-destination deduplication) plus ``meta_bytes`` per
assignment.  The cost model (milliseconds):

    comm    = communication_multiplier * (intra_ms_per_byte * peak_bytes
                                          + route_ms_per_assignment * peak_assignments)
    compute = compute_multiplier * compute_ms_per_assignment * peak_assignments
    total   = comm + compute

where ``peak_bytes`` is the max over GPUs of max(send, recv) bytes and
``peak_assignments`` the max over GPUs of expert assignments.  The replay is
the C++ ``evaluate_routes`` core.

Reference parity: the hybrid evaluator of
scripts/profile/build_hiermoe_hierarchical_init_layout.py:515-647 and its
endpoint statistics in veomni/distributed/moe/hiermoe/greedy_planner.py:747-900,
with the inter-node stage removed (one level).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .._build import load_planner
from .runtime.config import PlaceMoECalibration
from .types import LayerPlan, PlaceMoETopology

META_BYTES_PER_ASSIGNMENT = 8  # (unique ordinal, local slot) int32 pair


@dataclass(frozen=True)
class PlanCost:
    total_ms: float
    comm_ms: float
    compute_ms: float
    peak_bytes: float
    peak_assignments: float
    remote_rows: float
    remote_assignments: float
    total_assignments: float

    @property
    def dedup_ratio(self) -> float:
        return self.remote_assignments / max(self.remote_rows, 1.0)


class RouteReplayEvaluator:
    def __init__(self, samples, topology: PlaceMoETopology, *, hidden_size: int, bytes_per_element: int,
                 calibration: PlaceMoECalibration | None = None):
        """samples: list of steps, each a list (per source rank) of [T, k] int routes."""
        self.samples = [[torch.as_tensor(r).to(torch.int32).contiguous() for r in step] for step in samples]
        self._flat = [r for step in self.samples for r in step]
        self.topology = topology
        self.row_bytes = float(hidden_size * bytes_per_element)
        self.cal = calibration or PlaceMoECalibration()
        self.slot_rank = torch.from_numpy(topology.slot_ranks())

    def replay(self, mapping: np.ndarray) -> PlanCost:
        core = load_planner()
        m = torch.from_numpy(np.array(mapping, dtype=np.int64, copy=True))
        acc = core.evaluate_routes_batch(self._flat, m, self.slot_rank, self.row_bytes,
                                         float(META_BYTES_PER_ASSIGNMENT)).numpy().sum(axis=0)
        n = len(self.samples)
        peak_bytes, peak_asg = acc[0] / n, acc[1] / n
        c = self.cal
        comm = c.communication_multiplier * (c.intra_ms_per_byte * peak_bytes + c.route_ms_per_assignment * peak_asg)
        compute = c.compute_multiplier * c.compute_ms_per_assignment * peak_asg
        return PlanCost(comm + compute, comm, compute, peak_bytes, peak_asg, acc[2] / n, acc[3] / n, acc[4] / n)

    def evaluate(self, plan: LayerPlan) -> PlanCost:
        return self.replay(plan.source_logical_to_physical)

    def coefficients(self) -> tuple[float, float, float]:
        """(omega, gamma, local_weight) of the surrogate objectives in the same ms units.

        omega: a saved remote row ~ row_bytes * intra_ms_per_byte * comm_mult;
        gamma: one assignment on the critical GPU; local_weight: an assignment kept on its source GPU
        also saves its row transfer (upper bound, counted once per assignment).
        """
        c = self.cal
        omega = c.communication_multiplier * c.intra_ms_per_byte * self.row_bytes
        gamma = c.compute_multiplier * c.compute_ms_per_assignment + c.communication_multiplier * c.route_ms_per_assignment
        return omega, gamma, omega
