"""The planner subprocess of a hot update: its job record, command line and environment.

A hot update runs the planner CLI (``placemoe_b200.placemoe.plan_placemoe``)
as a separate process, so the CPU-heavy search overlaps training.  This
module turns a job description into that process's argv and environment:

* ``PlannerCommandSpec`` -- what to plan (topology, layers, route bundle,
  output paths, and for a mapping-only update the current layout);
* ``build_planner_command`` -- the argv: the interpreter, the planner script,
  then one ``--flag value`` pair per entry of ``_FLAG_TABLE``, the
  calibration coefficients, and ``--input-layout`` for mapping-only updates;
  prefixed with ``taskset -c <cpus>`` when planner CPUs are reserved;
* ``planner_environment`` -- one BLAS/OpenMP thread per planner worker unless
  configured otherwise, the repository on ``PYTHONPATH``;
* ``HotUpdateJob`` -- the record of a submitted job (paths, the placement
  versions it was planned from, the process handle).

The flag names are the planner's command-line interface, which is the
reference's (veomni/distributed/moe/hiermoe/placemoe/runtime/planner_process.py:15-145),
so either runtime can launch either planner.
"""

from __future__ import annotations

import os
import subprocess
import sys
from dataclasses import dataclass
from typing import Callable, Mapping, Sequence

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


# flag -> value taken from (spec, resources); the order is the order on the command line
_FLAG_TABLE: list[tuple[str, Callable[[PlannerCommandSpec, PlaceMoEPlannerResources], object]]] = [
    ("--route-root", lambda s, r: s.route_root),
    ("--optimize-steps", lambda s, r: 0),
    ("--validation-steps", lambda s, r: 0),
    ("--update-mode", lambda s, r: s.kind.value),
    ("--layers", lambda s, r: len(s.layer_keys)),
    ("--layer-keys", lambda s, r: ",".join(s.layer_keys)),
    ("--expected-total-layers", lambda s, r: len(s.layer_keys)),
    ("--workers", lambda s, r: r.workers),
    ("--candidate-workers", lambda s, r: r.candidate_workers),
    ("--worker-threads", lambda s, r: r.worker_threads),
    ("--ep-size", lambda s, r: s.ep_size),
    ("--ranks-per-node", lambda s, r: s.ranks_per_node),
    ("--num-experts", lambda s, r: s.num_experts),
    ("--slots-per-rank", lambda s, r: s.slots_per_rank),
    ("--primary-slots-per-rank", lambda s, r: s.primary_slots_per_rank),
    ("--redundant-slots-per-rank", lambda s, r: s.redundant_slots_per_rank),
    ("--active-redundant-slots", lambda s, r: s.redundant_slots_per_rank * s.ep_size),
    ("--hidden-size", lambda s, r: s.hidden_size),
    ("--bytes-per-element", lambda s, r: s.bytes_per_element),
]

# calibration coefficient -> planner flag
_COEFF_FLAGS = {
    "inter_ms_per_byte": "--inter-ms-per-byte",
    "intra_ms_per_byte": "--intra-ms-per-byte",
    "route_ms_per_assignment": "--route-ms-per-assignment",
    "communication_multiplier": "--communication-phase-multiplier",
    "compute_ms_per_assignment": "--compute-ms-per-assignment",
    "compute_multiplier": "--compute-phase-multiplier",
}


def default_planner_path() -> str:
    return os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "plan_placemoe.py")


def build_planner_command(spec: PlannerCommandSpec, calibration: PlaceMoECalibration,
                          resources: PlaceMoEPlannerResources) -> list[str]:
    if spec.kind is UpdateKind.MAPPING_ONLY and not spec.input_layout:
        raise ValueError("a mapping-only update plans against the current layout: input_layout is required")
    pairs = [(flag, get(spec, resources)) for flag, get in _FLAG_TABLE]
    coeffs = calibration.coefficients()
    pairs += [(flag, coeffs[name]) for name, flag in _COEFF_FLAGS.items()]
    pairs += [("--comparison-layout", "none"), ("--output-layout", spec.output_layout),
              ("--output-report", spec.output_report)]
    if spec.kind is UpdateKind.MAPPING_ONLY:
        pairs.append(("--input-layout", spec.input_layout))
    argv = [spec.python, spec.planner_path] + [str(x) for pair in pairs for x in pair]
    return (["taskset", "-c", resources.planner_cpu_ids] if resources.planner_cpu_ids else []) + argv


def planner_environment(resources: PlaceMoEPlannerResources, base: Mapping[str, str] | None = None) -> dict:
    env = dict(os.environ if base is None else base)
    threads = str(resources.worker_threads)
    for var in ("OMP_NUM_THREADS", "MKL_NUM_THREADS", "OPENBLAS_NUM_THREADS"):
        env[var] = threads
    env["PYTHONUNBUFFERED"] = "1"
    repo = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..", ".."))
    env["PYTHONPATH"] = os.pathsep.join(p for p in (repo, env.get("PYTHONPATH", "")) if p)
    return env


def python_executable() -> str:
    return sys.executable
