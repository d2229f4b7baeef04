"""PlaceMoE runtime configuration (the file named by ``VEOMNI_PLACEMOE_CONFIG``).

YAML or JSON, optionally nested under a top-level ``placemoe:`` key::

    initial_artifact: <schema-v2 artifact, loaded at startup>
    runtime_perf_model: <optional perf-model JSON>
    calibration: {artifact, require_scope, expected_scope,
                  inter_ms_per_byte, intra_ms_per_byte, route_ms_per_assignment,
                  communication_multiplier, compute_ms_per_assignment, compute_multiplier}
    hot_update: {enabled, layout_interval_steps, mapping_interval_steps,
                 last_update_step, work_root, planner_path, failure_policy}
    resources: {workers, candidate_workers, worker_threads, planner_cpu_ids, training_cpu_ids}

Parsing is table-driven: every section is described by a list of ``_Field``
entries (key, value kind, default) and one generic reader converts, checks
and rejects unknown keys, so a bad file fails before training with a message
naming the offending key.  Paths are resolved against the file's directory.

The file format -- key names, defaults (including the six default cost
coefficients) and which values are accepted -- follows
veomni/distributed/moe/hiermoe/placemoe/runtime/config.py:18-345, so one
configuration file drives either implementation.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Mapping

import yaml

# Default cost coefficients (milliseconds): the values the reference ships as calibrated defaults.
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


# ------------------------------------------------------------------ value kinds
_TRUE = {"1", "true", "yes", "on", "y"}
_FALSE = {"0", "false", "no", "off", "n"}


def _kind_bool(value: Any, key: str, base: Path) -> bool:
    if isinstance(value, bool):
        return value
    if isinstance(value, int) and value in (0, 1):
        return bool(value)
    word = str(value).strip().lower() if isinstance(value, str) else None
    if word in _TRUE or word in _FALSE:
        return word in _TRUE
    raise PlaceMoEConfigurationError(f"{key}: expected true/false, found {value!r}")


def _whole(value: Any, key: str, *, minimum: int) -> int:
    ok = not isinstance(value, bool)
    try:
        number = int(value) if ok else 0
    except (TypeError, ValueError):
        ok = False
    if not ok or number < minimum:
        raise PlaceMoEConfigurationError(f"{key}: expected an integer >= {minimum}, found {value!r}")
    return number


def _kind_count(value: Any, key: str, base: Path) -> int:
    return _whole(value, key, minimum=0)


def _kind_positive_count(value: Any, key: str, base: Path) -> int:
    return _whole(value, key, minimum=1)


def _kind_optional_count(value: Any, key: str, base: Path) -> int | None:
    return None if value is None else _whole(value, key, minimum=0)


def _kind_positive_real(value: Any, key: str, base: Path) -> float:
    number = None
    if not isinstance(value, bool):
        try:
            number = float(value)
        except (TypeError, ValueError):
            number = None
    if number is None or not number > 0:
        raise PlaceMoEConfigurationError(f"{key}: expected a number > 0, found {value!r}")
    return number


def _kind_path(value: Any, key: str, base: Path) -> str:
    text = "" if value is None else os.path.expandvars(os.path.expanduser(str(value).strip()))
    if not text:
        return ""
    path = Path(text)
    return str((path if path.is_absolute() else base / path).resolve())


def _kind_text(value: Any, key: str, base: Path) -> str:
    return str(value).strip()


def _kind_policy(value: Any, key: str, base: Path) -> str:
    word = str(value).strip().lower()
    if word not in ("continue", "raise"):
        raise PlaceMoEConfigurationError(f"{key}: expected 'continue' or 'raise', found {value!r}")
    return word


def _kind_mapping(value: Any, key: str, base: Path) -> dict:
    if value is None:
        return {}
    if not isinstance(value, Mapping):
        raise PlaceMoEConfigurationError(f"{key}: expected a mapping, found {type(value).__name__}")
    return dict(value)


@dataclass(frozen=True)
class _Field:
    key: str
    kind: Callable[[Any, str, Path], Any]
    default: Any


def _read_section(payload: Any, fields: list[_Field], section: str, base: Path) -> dict[str, Any]:
    """Convert one section: every known key through its kind (default when absent); unknown keys fail."""
    data = _kind_mapping(payload, section, base)
    unknown = sorted(set(data) - {f.key for f in fields})
    if unknown:
        raise PlaceMoEConfigurationError(f"{section}: unknown keys {', '.join(unknown)}")
    return {f.key: f.kind(data.get(f.key, f.default), f"{section}.{f.key}", base) for f in fields}


# ------------------------------------------------------------------ sections
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

    _COEFFS = [_Field(k, _kind_positive_real, v) for k, v in DEFAULT_COEFFICIENTS.items()]
    _META = [_Field("artifact", _kind_path, ""), _Field("require_scope", _kind_bool, False),
             _Field("expected_scope", _kind_mapping, None)]

    @classmethod
    def from_mapping(cls, payload: Mapping[str, Any], *, base_directory: Path) -> "PlaceMoECalibration":
        data = _kind_mapping(payload, "calibration", base_directory)
        meta_keys = {f.key for f in cls._META}
        meta = _read_section({k: v for k, v in data.items() if k in meta_keys}, cls._META, "calibration",
                             base_directory)
        inline = {k: v for k, v in data.items() if k not in meta_keys}
        if meta["require_scope"] and not (meta["artifact"] and meta["expected_scope"]):
            raise PlaceMoEConfigurationError(
                "calibration.require_scope needs both calibration.artifact and a non-empty calibration.expected_scope")
        scope: dict = {}
        if meta["artifact"]:
            from_file, scope = _calibration_file(meta["artifact"], meta["expected_scope"] if meta["require_scope"]
                                                 else None)
            inline = {**from_file, **inline}  # inline values override the file
        coeffs = _read_section(inline, cls._COEFFS, "calibration", base_directory)
        return cls(**coeffs, artifact=meta["artifact"], require_scope=meta["require_scope"],
                   expected_scope=meta["expected_scope"], artifact_scope=scope)

    def coefficients(self) -> dict[str, float]:
        return {k: float(getattr(self, k)) for k in DEFAULT_COEFFICIENTS}


def _calibration_file(path: str, expected: Mapping[str, Any] | None) -> tuple[dict, dict]:
    """(coefficients, scope) of an accepted calibration artifact; ``expected`` scope keys must match."""
    blob = json.loads(Path(path).read_text(encoding="utf-8"))
    if not isinstance(blob, Mapping):
        raise PlaceMoEConfigurationError(f"calibration artifact {path}: top level is not a mapping")
    if blob.get("status", "accepted") != "accepted":
        raise PlaceMoEConfigurationError(f"calibration artifact {path}: status {blob.get('status')!r} is not "
                                         "'accepted'")
    raw_scope = blob.get("scope")
    if expected is not None and not isinstance(raw_scope, Mapping):
        raise PlaceMoEConfigurationError(f"calibration artifact {path}: no scope mapping to check")
    scope = dict(raw_scope) if isinstance(raw_scope, Mapping) else {}
    if expected is not None:
        diffs = [f"{k}: expected {v!r}, artifact has {scope.get(k, '<missing>')!r}"
                 for k, v in sorted(expected.items()) if k not in scope or scope[k] != v]
        if diffs:
            raise PlaceMoEConfigurationError(f"calibration artifact {path} is for another scope ({'; '.join(diffs)})")
    coeffs = blob.get("coefficients", blob)
    if not isinstance(coeffs, Mapping):
        raise PlaceMoEConfigurationError(f"calibration artifact {path}: coefficients are not a mapping")
    known = set(DEFAULT_COEFFICIENTS)
    # an artifact without a "coefficients" block carries them at top level, next to status/scope
    picked = {k: v for k, v in coeffs.items() if k in known or coeffs is not blob}
    return picked, scope


@dataclass(frozen=True)
class PlaceMoEPlannerResources:
    workers: int = 48
    candidate_workers: int = 4
    worker_threads: int = 1
    planner_cpu_ids: str = ""
    training_cpu_ids: str = ""

    _FIELDS = [_Field("workers", _kind_positive_count, 48), _Field("candidate_workers", _kind_positive_count, 4),
               _Field("worker_threads", _kind_positive_count, 1), _Field("planner_cpu_ids", _kind_text, ""),
               _Field("training_cpu_ids", _kind_text, "")]

    @classmethod
    def from_mapping(cls, payload: Mapping[str, Any]) -> "PlaceMoEPlannerResources":
        out = cls(**_read_section(payload, cls._FIELDS, "resources", Path(".")))
        if bool(out.planner_cpu_ids) != bool(out.training_cpu_ids):
            raise PlaceMoEConfigurationError("resources: planner_cpu_ids and training_cpu_ids go together "
                                             "(set both or neither)")
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

    _FIELDS = [_Field("enabled", _kind_bool, False), _Field("layout_interval_steps", _kind_optional_count, None),
               _Field("mapping_interval_steps", _kind_count, 0), _Field("last_update_step", _kind_count, 2**31 - 1),
               _Field("work_root", _kind_path, "/tmp/veomni_placemoe_hot_update"),
               _Field("planner_path", _kind_path, ""), _Field("failure_policy", _kind_policy, "continue")]

    @classmethod
    def from_mapping(cls, payload: Mapping[str, Any], *, base_directory: Path) -> "HotUpdateConfig":
        return cls(**_read_section(payload, cls._FIELDS, "hot_update", base_directory))


@dataclass(frozen=True)
class PlaceMoERuntimeConfig:
    initial_artifact: str = ""
    runtime_perf_model: str = ""
    hot_update: HotUpdateConfig = field(default_factory=HotUpdateConfig)
    calibration: PlaceMoECalibration = field(default_factory=PlaceMoECalibration)
    resources: PlaceMoEPlannerResources = field(default_factory=PlaceMoEPlannerResources)
    source_path: str = ""

    _TOP = [_Field("initial_artifact", _kind_path, ""), _Field("runtime_perf_model", _kind_path, ""),
            _Field("hot_update", _kind_mapping, None), _Field("calibration", _kind_mapping, None),
            _Field("resources", _kind_mapping, None)]

    @classmethod
    def from_file(cls, path) -> "PlaceMoERuntimeConfig":
        src = Path(path).expanduser().resolve()
        if not src.is_file():
            raise PlaceMoEConfigurationError(f"PlaceMoE configuration file not found: {src}")
        text = src.read_text(encoding="utf-8")
        payload = json.loads(text) if src.suffix.lower() == ".json" else yaml.safe_load(text)
        payload = _kind_mapping(payload, "PlaceMoE configuration", src.parent)
        if "placemoe" in payload:
            payload = _kind_mapping(payload["placemoe"], "placemoe", src.parent)
        top = _read_section(payload, cls._TOP, "placemoe", src.parent)
        cfg = cls(initial_artifact=top["initial_artifact"], runtime_perf_model=top["runtime_perf_model"],
                  hot_update=HotUpdateConfig.from_mapping(top["hot_update"], base_directory=src.parent),
                  calibration=PlaceMoECalibration.from_mapping(top["calibration"], base_directory=src.parent),
                  resources=PlaceMoEPlannerResources.from_mapping(top["resources"]), source_path=str(src))
        cfg.validate()
        return cfg

    @classmethod
    def from_environment(cls, environment: Mapping[str, str] | None = None) -> "PlaceMoERuntimeConfig":
        env = os.environ if environment is None else environment
        path = env.get(CONFIG_ENV, "").strip()
        return cls.from_file(path) if path else cls()

    def validate(self) -> None:
        """Cross-section rules: hot updates start from an installed artifact and need a work directory."""
        if not self.hot_update.enabled:
            return
        if not self.initial_artifact:
            raise PlaceMoEConfigurationError("hot_update.enabled needs initial_artifact (the layout to start from)")
        if not self.hot_update.work_root:
            raise PlaceMoEConfigurationError("hot_update.work_root is empty")


__all__ = ["CONFIG_ENV", "DEFAULT_COEFFICIENTS", "HotUpdateConfig", "PlaceMoECalibration",
           "PlaceMoEConfigurationError", "PlaceMoEPlannerResources", "PlaceMoERuntimeConfig"]
