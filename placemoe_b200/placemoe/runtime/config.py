"""Strict PlaceMoE runtime configuration (``VEOMNI_PLACEMOE_CONFIG``).

YAML or JSON, optionally nested under a top-level ``placemoe:`` key:

    initial_artifact: <schema-v2 artifact, loaded at startup>
    runtime_perf_model: <optional perf-model JSON>
    calibration: {artifact, require_scope, expected_scope,
                  inter_ms_per_byte, intra_ms_per_byte, route_ms_per_assignment,
                  communication_multiplier, compute_ms_per_assignment, compute_multiplier}
    hot_update: {enabled, layout_interval_steps, mapping_interval_steps,
                 last_update_step, work_root, planner_path, failure_policy}
    resources: {workers, candidate_workers, worker_threads, planner_cpu_ids, training_cpu_ids}

Relative paths resolve against the YAML's directory; unknown keys are
rejected; invalid values raise PlaceMoEConfigurationError before training.
The file interface (keys, defaults, validation rules) is kept identical to
veomni/distributed/moe/hiermoe/placemoe/runtime/config.py:18-345 so existing
configuration files work unchanged.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Mapping

import yaml

# Default cost coefficients (milliseconds), the reference's calibrated values.
DEFAULT_COEFFICIENTS = {
    "inter_ms_per_byte": 6.765449326279194e-08,
    "intra_ms_per_byte": 5.02482606728045e-09,
    "route_ms_per_assignment": 8.746548178958447e-05,
    "communication_multiplier": 3.1,
    "compute_ms_per_assignment": 2.82807e-05,
    "compute_multiplier": 4.19,
}
CONFIG_ENV = "VEOMNI_PLACEMOE_CONFIG"


class PlaceMoEConfigurationError(ValueError):
    """Invalid PlaceMoE configuration (raised before training starts)."""


def _as_mapping(v: Any, what: str) -> Mapping[str, Any]:
    if v is None:
        return {}
    if not isinstance(v, Mapping):
        raise PlaceMoEConfigurationError(f"{what} must be a mapping, got {type(v).__name__}.")
    return v


def _bool(v: Any, what: str) -> bool:
    if isinstance(v, bool):
        return v
    if isinstance(v, int) and v in (0, 1):
        return bool(v)
    if isinstance(v, str):
        s = v.strip().lower()
        if s in ("1", "true", "yes", "on", "y"):
            return True
        if s in ("0", "false", "no", "off", "n"):
            return False
    raise PlaceMoEConfigurationError(f"{what} must be a boolean, got {v!r}.")


def _int(v: Any, what: str, positive: bool = False) -> int:
    if isinstance(v, bool):
        raise PlaceMoEConfigurationError(f"{what} must be a non-negative integer, got {v!r}.")
    try:
        x = int(v)
    except (TypeError, ValueError) as err:
        raise PlaceMoEConfigurationError(f"{what} must be a non-negative integer, got {v!r}.") from err
    if x < 0:
        raise PlaceMoEConfigurationError(f"{what} must be non-negative, got {x}.")
    if positive and x == 0:
        raise PlaceMoEConfigurationError(f"{what} must be positive.")
    return x


def _pos_float(v: Any, what: str) -> float:
    if isinstance(v, bool):
        raise PlaceMoEConfigurationError(f"{what} must be positive, got {v!r}.")
    try:
        x = float(v)
    except (TypeError, ValueError) as err:
        raise PlaceMoEConfigurationError(f"{what} must be positive, got {v!r}.") from err
    if not x > 0:
        raise PlaceMoEConfigurationError(f"{what} must be positive, got {x}.")
    return x


def _path(v: Any, base: Path) -> str:
    if v is None:
        return ""
    s = os.path.expandvars(os.path.expanduser(str(v).strip()))
    if not s:
        return ""
    p = Path(s)
    return str((p if p.is_absolute() else base / p).resolve())


def _reject_unknown(d: Mapping[str, Any], allowed: set, what: str) -> None:
    extra = sorted(set(d) - allowed)
    if extra:
        raise PlaceMoEConfigurationError(f"unknown {what} fields: {', '.join(extra)}.")


@dataclass(frozen=True)
class PlaceMoECalibration:
    inter_ms_per_byte: float = DEFAULT_COEFFICIENTS["inter_ms_per_byte"]
    intra_ms_per_byte: float = DEFAULT_COEFFICIENTS["intra_ms_per_byte"]
    route_ms_per_assignment: float = DEFAULT_COEFFICIENTS["route_ms_per_assignment"]
    communication_multiplier: float = DEFAULT_COEFFICIENTS["communication_multiplier"]
    compute_ms_per_assignment: float = DEFAULT_COEFFICIENTS["compute_ms_per_assignment"]
    compute_multiplier: float = DEFAULT_COEFFICIENTS["compute_multiplier"]
    artifact: str = ""
    require_scope: bool = False
    expected_scope: Mapping[str, Any] = field(default_factory=dict)
    artifact_scope: Mapping[str, Any] = field(default_factory=dict)

    @classmethod
    def from_mapping(cls, payload: Mapping[str, Any], *, base_directory: Path) -> "PlaceMoECalibration":
        data = dict(payload)
        artifact = _path(data.pop("artifact", ""), base_directory)
        require = _bool(data.pop("require_scope", False), "calibration.require_scope")
        expected = dict(_as_mapping(data.pop("expected_scope", None), "calibration.expected_scope"))
        if require and not artifact:
            raise PlaceMoEConfigurationError("calibration.artifact is required when require_scope is true.")
        if require and not expected:
            raise PlaceMoEConfigurationError("calibration.expected_scope must not be empty when require_scope is true.")
        scope: Mapping[str, Any] = {}
        if artifact:
            blob = json.loads(Path(artifact).read_text(encoding="utf-8"))
            if not isinstance(blob, Mapping):
                raise PlaceMoEConfigurationError(f"calibration artifact {artifact} must contain a mapping.")
            status = blob.get("status", "accepted")
            if status != "accepted":
                raise PlaceMoEConfigurationError(
                    f"calibration artifact {artifact} has status {status!r}, expected 'accepted'.")
            raw_scope = blob.get("scope")
            if isinstance(raw_scope, Mapping):
                scope = dict(raw_scope)
            elif require:
                _as_mapping(raw_scope, "calibration artifact scope")
            if require:
                missing = sorted(set(expected) - set(scope))
                wrong = sorted(k for k, v in expected.items() if k in scope and scope[k] != v)
                if missing or wrong:
                    parts = []
                    if missing:
                        parts.append(f"missing keys {missing}")
                    if wrong:
                        parts.append("mismatched values " + str({k: {"expected": expected[k], "actual": scope[k]}
                                                                  for k in wrong}))
                    raise PlaceMoEConfigurationError(
                        f"calibration artifact {artifact} does not match expected scope: {'; '.join(parts)}.")
            coeffs = blob.get("coefficients", blob)
            if not isinstance(coeffs, Mapping):
                raise PlaceMoEConfigurationError(f"calibration artifact {artifact} has no coefficient mapping.")
            merged = dict(coeffs)
            merged.update(data)
            data = merged
        _reject_unknown(data, set(DEFAULT_COEFFICIENTS), "calibration")
        vals = {k: _pos_float(data.get(k, DEFAULT_COEFFICIENTS[k]), f"calibration.{k}") for k in DEFAULT_COEFFICIENTS}
        return cls(**vals, artifact=artifact, require_scope=require, expected_scope=expected, artifact_scope=scope)

    def coefficients(self) -> dict[str, float]:
        return {k: float(getattr(self, k)) for k in DEFAULT_COEFFICIENTS}


@dataclass(frozen=True)
class PlaceMoEPlannerResources:
    workers: int = 48
    candidate_workers: int = 4
    worker_threads: int = 1
    planner_cpu_ids: str = ""
    training_cpu_ids: str = ""

    @classmethod
    def from_mapping(cls, payload: Mapping[str, Any]) -> "PlaceMoEPlannerResources":
        _reject_unknown(payload, {"workers", "candidate_workers", "worker_threads", "planner_cpu_ids",
                                  "training_cpu_ids"}, "resource")
        d = cls()
        out = cls(
            workers=_int(payload.get("workers", d.workers), "resources.workers", positive=True),
            candidate_workers=_int(payload.get("candidate_workers", d.candidate_workers),
                                   "resources.candidate_workers", positive=True),
            worker_threads=_int(payload.get("worker_threads", d.worker_threads), "resources.worker_threads",
                                positive=True),
            planner_cpu_ids=str(payload.get("planner_cpu_ids", d.planner_cpu_ids)).strip(),
            training_cpu_ids=str(payload.get("training_cpu_ids", d.training_cpu_ids)).strip(),
        )
        if bool(out.planner_cpu_ids) != bool(out.training_cpu_ids):
            raise PlaceMoEConfigurationError(
                "resources.planner_cpu_ids and resources.training_cpu_ids must be configured together.")
        return out


@dataclass(frozen=True)
class HotUpdateConfig:
    enabled: bool = False
    layout_interval_steps: int | None = None
    mapping_interval_steps: int = 0
    last_update_step: int = 2**31 - 1
    work_root: str = "/tmp/veomni_placemoe_hot_update"
    planner_path: str = ""
    failure_policy: str = "continue"

    @classmethod
    def from_mapping(cls, payload: Mapping[str, Any], *, base_directory: Path) -> "HotUpdateConfig":
        _reject_unknown(payload, {"enabled", "layout_interval_steps", "mapping_interval_steps", "last_update_step",
                                  "work_root", "planner_path", "failure_policy"}, "hot_update")
        d = cls()
        raw_layout = payload.get("layout_interval_steps", d.layout_interval_steps)
        policy = str(payload.get("failure_policy", d.failure_policy)).strip().lower()
        if policy not in ("continue", "raise"):
            raise PlaceMoEConfigurationError("hot_update.failure_policy must be 'continue' or 'raise'.")
        return cls(
            enabled=_bool(payload.get("enabled", d.enabled), "hot_update.enabled"),
            layout_interval_steps=None if raw_layout is None else _int(raw_layout, "hot_update.layout_interval_steps"),
            mapping_interval_steps=_int(payload.get("mapping_interval_steps", d.mapping_interval_steps),
                                        "hot_update.mapping_interval_steps"),
            last_update_step=_int(payload.get("last_update_step", d.last_update_step), "hot_update.last_update_step"),
            work_root=_path(payload.get("work_root", d.work_root), base_directory),
            planner_path=_path(payload.get("planner_path", d.planner_path), base_directory),
            failure_policy=policy,
        )


@dataclass(frozen=True)
class PlaceMoERuntimeConfig:
    initial_artifact: str = ""
    runtime_perf_model: str = ""
    hot_update: HotUpdateConfig = field(default_factory=HotUpdateConfig)
    calibration: PlaceMoECalibration = field(default_factory=PlaceMoECalibration)
    resources: PlaceMoEPlannerResources = field(default_factory=PlaceMoEPlannerResources)
    source_path: str = ""

    @classmethod
    def from_file(cls, path) -> "PlaceMoERuntimeConfig":
        p = Path(path).expanduser().resolve()
        if not p.is_file():
            raise PlaceMoEConfigurationError(f"PlaceMoE config does not exist: {p}.")
        text = p.read_text(encoding="utf-8")
        payload = json.loads(text) if p.suffix.lower() == ".json" else yaml.safe_load(text)
        root = _as_mapping(payload, "PlaceMoE config")
        if "placemoe" in root:
            root = _as_mapping(root["placemoe"], "placemoe")
        _reject_unknown(root, {"initial_artifact", "runtime_perf_model", "hot_update", "calibration", "resources"},
                        "PlaceMoE")
        base = p.parent
        cfg = cls(
            initial_artifact=_path(root.get("initial_artifact", ""), base),
            runtime_perf_model=_path(root.get("runtime_perf_model", ""), base),
            hot_update=HotUpdateConfig.from_mapping(_as_mapping(root.get("hot_update"), "hot_update"),
                                                    base_directory=base),
            calibration=PlaceMoECalibration.from_mapping(_as_mapping(root.get("calibration"), "calibration"),
                                                         base_directory=base),
            resources=PlaceMoEPlannerResources.from_mapping(_as_mapping(root.get("resources"), "resources")),
            source_path=str(p),
        )
        cfg.validate()
        return cfg

    @classmethod
    def from_environment(cls, environment: Mapping[str, str] | None = None) -> "PlaceMoERuntimeConfig":
        env = os.environ if environment is None else environment
        path = env.get(CONFIG_ENV, "").strip()
        return cls.from_file(path) if path else cls()

    def validate(self) -> None:
        if self.hot_update.enabled:
            if not self.initial_artifact:
                raise PlaceMoEConfigurationError("initial_artifact is required when PlaceMoE hot updates are enabled.")
            if not self.hot_update.work_root:
                raise PlaceMoEConfigurationError("hot_update.work_root must not be empty.")


__all__ = ["CONFIG_ENV", "DEFAULT_COEFFICIENTS", "HotUpdateConfig", "PlaceMoECalibration",
           "PlaceMoEConfigurationError", "PlaceMoEPlannerResources", "PlaceMoERuntimeConfig"]
