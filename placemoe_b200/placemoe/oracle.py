"""Route oracle capture and idealised communication volumes.

``OracleCapture`` attaches a route recorder for a configured window of steps
(``PM_ORACLE_CAPTURE_DIR`` / ``PM_ORACLE_CAPTURE_STEPS``, e.g. ``"10-29"``) and
writes the planner's route bundles there, so planning inputs can be taken
from a normal training run without other changes.  ``dispatch_volumes``
gives, for captured routes and a placement, the rows a rank sends with and
without per-destination dedup and the per-rank received assignments -- the
quantities the planner optimises, for offline inspection.

Reference parity: veomni/distributed/moe/hiermoe/oracle.py:38 (snapshot
writer, environment knobs), :240-349 (idealised volume heuristics).
"""

from __future__ import annotations

import os

import numpy as np

ENV_DIR = "PM_ORACLE_CAPTURE_DIR"
ENV_STEPS = "PM_ORACLE_CAPTURE_STEPS"


def parse_steps(text: str) -> set[int]:
    out: set[int] = set()
    for part in (text or "").split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            out.update(range(int(a), int(b) + 1))
        else:
            out.add(int(part))
    return out


class OracleCapture:
    """Captures routes on the configured steps (no-op when the environment does not ask for it)."""

    def __init__(self, model, environ=None):
        env = os.environ if environ is None else environ
        self.root = env.get(ENV_DIR, "")
        self.steps = parse_steps(env.get(ENV_STEPS, ""))
        self.recorder = None
        if self.root and self.steps:
            from ..parallel.route_capture import RouteRecorder

            self.recorder = RouteRecorder(model, self.root)

    @property
    def active(self) -> bool:
        return self.recorder is not None

    def before_step(self, step: int) -> None:
        if self.recorder is not None:
            self.recorder.enabled = step in self.steps

    def after_step(self, step: int) -> list[str]:
        if self.recorder is not None and step in self.steps:
            return self.recorder.record_step(step)
        return []


def dispatch_volumes(routes_by_rank, mapping: np.ndarray, slot_rank: np.ndarray) -> dict[str, np.ndarray]:
    """routes_by_rank[s]: [T_s, k] logical experts; mapping [S, E] -> slot; slot_rank [slots] -> rank."""
    world = mapping.shape[0]
    dedup = np.zeros((world, world), dtype=np.int64)
    raw = np.zeros((world, world), dtype=np.int64)
    for s, r in enumerate(routes_by_rank):
        r = np.asarray(r, dtype=np.int64)
        if r.size == 0:
            continue
        dest = slot_rank[mapping[s][r]]  # [T, k]
        for d in range(world):
            hit = dest == d
            raw[s, d] += int(hit.sum())
            dedup[s, d] += int(hit.any(axis=1).sum())
    return {"rows_dedup": dedup, "rows_no_dedup": raw, "recv_assignments": raw.sum(axis=0),
            "dedup_ratio": np.divide(raw.sum(), max(dedup.sum(), 1))}
