"""Schema-v2 PlaceMoE artifact: build and validate.

The JSON layout is a fixed interchange format (identical keys and semantics to
veomni/distributed/moe/hiermoe/placemoe/artifacts.py:25-95, so artifacts written
by either implementation load in the other):

    {"schema_version": 2,
     "source": {..., "algorithm": "placemoe-v1", "initial_layout": "preloaded",
                "requires_static_preload": true},
     "topology": {"ep_size", "ranks_per_node", "num_experts",
                  "num_physical_slots", "slots_per_rank"},
     "replay": {"actions_by_step": {"1": []}},
     "layers": {name: {"slot_to_logical", "owner_slots", "source_logical_to_physical"}}}
"""

from __future__ import annotations

import json
import os
from collections.abc import Mapping
from typing import Any

from .types import LayerPlan, PlaceMoETopology

PLACEMOE_ARTIFACT_SCHEMA_VERSION = 2
ALGORITHM = "placemoe-v1"


class ArtifactError(ValueError):
    """A schema-v2 artifact that cannot be installed."""


def _require(ok: bool, problem: str) -> None:
    if not ok:
        raise ArtifactError(f"PlaceMoE artifact rejected: {problem}")


def _topology_row(topology: PlaceMoETopology) -> dict[str, int]:
    return {"ep_size": topology.ep_size, "ranks_per_node": topology.ranks_per_node,
            "num_experts": topology.num_experts, "num_physical_slots": topology.total_slots,
            "slots_per_rank": topology.slots_per_rank}


def build_placemoe_artifact(plans: Mapping[str, LayerPlan], topology: PlaceMoETopology, *,
                            source: Mapping[str, Any] | None = None) -> dict[str, Any]:
    """The artifact for ``plans`` (every plan checked against ``topology``) -- validated before it is returned."""
    _require(bool(plans), "no layer plans")
    _require(all(isinstance(k, str) and k for k in plans), "every layer needs a non-empty name")
    for plan in plans.values():
        plan.validate(topology)
    provenance = {**dict(source or {}), "algorithm": ALGORITHM, "initial_layout": "preloaded",
                  "requires_static_preload": True}
    payload = {
        "schema_version": PLACEMOE_ARTIFACT_SCHEMA_VERSION,
        "source": provenance,
        "topology": _topology_row(topology),
        "replay": {"actions_by_step": {"1": []}},
        "layers": {name: plan.to_runtime_payload() for name, plan in plans.items()},
    }
    validate_placemoe_artifact(payload)
    return payload


def artifact_topology(payload: Mapping[str, Any]) -> PlaceMoETopology:
    row = payload.get("topology")
    _require(isinstance(row, Mapping), "no topology object")
    try:
        topo = PlaceMoETopology(ep_size=int(row["ep_size"]),
                                ranks_per_node=int(row.get("ranks_per_node", row["ep_size"])),
                                num_experts=int(row["num_experts"]), slots_per_rank=int(row["slots_per_rank"]))
    except KeyError as missing:
        raise ArtifactError(f"PlaceMoE artifact rejected: topology lacks {missing}") from None
    declared = int(row.get("num_physical_slots", -1))
    _require(declared == topo.total_slots,
             f"topology declares {declared} physical slots, its sizes give {topo.total_slots}")
    return topo


def validate_placemoe_artifact(payload: Mapping[str, Any]) -> dict[str, LayerPlan]:
    """Every layer plan of a schema-v2 artifact, each checked against the artifact's topology."""
    version = payload.get("schema_version")
    _require(version == PLACEMOE_ARTIFACT_SCHEMA_VERSION,
             f"schema_version {version!r}, this reader understands {PLACEMOE_ARTIFACT_SCHEMA_VERSION}")
    provenance = payload.get("source")
    _require(isinstance(provenance, Mapping) and provenance.get("algorithm") == ALGORITHM,
             f"source.algorithm must be {ALGORITHM!r}")
    topo = artifact_topology(payload)
    layers = payload.get("layers")
    _require(isinstance(layers, Mapping) and len(layers) > 0, "empty or missing layer table")
    plans = {}
    for name, row in layers.items():
        _require(isinstance(name, str) and isinstance(row, Mapping), f"layer entry {name!r} is not a plan object")
        plans[name] = LayerPlan.from_runtime_payload(dict(row))
        plans[name].validate(topo)
    return plans


def write_artifact(payload: Mapping[str, Any], path: str) -> None:
    """Atomic write (temp file + rename) so a concurrent reader never sees a partial artifact."""
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    tmp = f"{path}.tmp.{os.getpid()}"
    with open(tmp, "w") as f:
        json.dump(payload, f)
    os.replace(tmp, path)


def load_artifact(path: str) -> tuple[dict[str, Any], PlaceMoETopology, dict[str, LayerPlan]]:
    with open(path) as f:
        payload = json.load(f)
    plans = validate_placemoe_artifact(payload)
    return payload, artifact_topology(payload), plans
