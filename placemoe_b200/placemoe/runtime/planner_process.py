"""Planner subprocess specification for hot updates.

``build_planner_command`` produces the argv of the planner CLI (the flag set
of ``placemoe_b200.placemoe.plan_placemoe``, which keeps the reference
planner's flag names), prefixed by ``taskset -c <cpus>`` when planner CPUs are
reserved.  ``planner_environment`` pins the BLAS/OpenMP thread counts.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/runtime/planner_process.py:15-145.
"""

from __future__ import annotations

import os
import subprocess
import sys
from dataclasses import dataclass
from typing import Mapping, Sequence

from .config import PlaceMoECalibration, PlaceMoEPlannerResources
from .scheduler import UpdateKind


@dataclass(frozen=True)
class HotUpdateJob:
    kind: UpdateKind
    source_step: int
    placement_versions: tuple[int, ...]
    submitted_at: float
    snapshot_ms: float
    job_dir: str
    layout_path: str
    report_path: str
    planner_log_path: str
    process: subprocess.Popen | None = None

    @property
    def update_mode(self) -> str:
        return self.kind.value


@dataclass(frozen=True)
class PlannerCommandSpec:
    python: str
    planner_path: str
    route_root: str
    kind: UpdateKind
    layer_keys: Sequence[str]
    ep_size: int
    ranks_per_node: int
    num_experts: int
    slots_per_rank: int
    primary_slots_per_rank: int
    redundant_slots_per_rank: int
    hidden_size: int
    bytes_per_element: int
    output_layout: str
    output_report: str
    input_layout: str = ""


def default_planner_path() -> str:
    return os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "plan_placemoe.py")


def build_planner_command(spec: PlannerCommandSpec, calibration: PlaceMoECalibration,
                          resources: PlaceMoEPlannerResources) -> list[str]:
    c = calibration
    args = {
        "--route-root": spec.route_root,
        "--optimize-steps": "0",
        "--validation-steps": "0",
        "--update-mode": spec.kind.value,
        "--layers": str(len(spec.layer_keys)),
        "--layer-keys": ",".join(spec.layer_keys),
        "--expected-total-layers": str(len(spec.layer_keys)),
        "--workers": str(resources.workers),
        "--candidate-workers": str(resources.candidate_workers),
        "--worker-threads": str(resources.worker_threads),
        "--ep-size": str(spec.ep_size),
        "--ranks-per-node": str(spec.ranks_per_node),
        "--num-experts": str(spec.num_experts),
        "--slots-per-rank": str(spec.slots_per_rank),
        "--primary-slots-per-rank": str(spec.primary_slots_per_rank),
        "--redundant-slots-per-rank": str(spec.redundant_slots_per_rank),
        "--active-redundant-slots": str(spec.redundant_slots_per_rank * spec.ep_size),
        "--hidden-size": str(spec.hidden_size),
        "--bytes-per-element": str(spec.bytes_per_element),
        "--inter-ms-per-byte": str(c.inter_ms_per_byte),
        "--intra-ms-per-byte": str(c.intra_ms_per_byte),
        "--route-ms-per-assignment": str(c.route_ms_per_assignment),
        "--communication-phase-multiplier": str(c.communication_multiplier),
        "--compute-ms-per-assignment": str(c.compute_ms_per_assignment),
        "--compute-phase-multiplier": str(c.compute_multiplier),
        "--comparison-layout": "none",
        "--output-layout": spec.output_layout,
        "--output-report": spec.output_report,
    }
    cmd = [spec.python, spec.planner_path]
    for k, v in args.items():
        cmd += [k, v]
    if spec.kind is UpdateKind.MAPPING_ONLY:
        if not spec.input_layout:
            raise ValueError("mapping-only planning requires input_layout.")
        cmd += ["--input-layout", spec.input_layout]
    if resources.planner_cpu_ids:
        cmd = ["taskset", "-c", resources.planner_cpu_ids, *cmd]
    return cmd


def planner_environment(resources: PlaceMoEPlannerResources, base: Mapping[str, str] | None = None) -> dict:
    env = dict(os.environ if base is None else base)
    n = str(resources.worker_threads)
    env.update({"OMP_NUM_THREADS": n, "MKL_NUM_THREADS": n, "OPENBLAS_NUM_THREADS": n, "PYTHONUNBUFFERED": "1"})
    repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    env["PYTHONPATH"] = repo + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    return env


def python_executable() -> str:
    return sys.executable
