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


def build_placemoe_artifact(plans: Mapping[str, LayerPlan], topology: PlaceMoETopology, *,
                            source: Mapping[str, Any] | None = None) -> dict[str, Any]:
    if not plans:
        raise ValueError("A PlaceMoE artifact must contain at least one layer plan.")
    layers = {}
    for name, plan in plans.items():
        if not name:
            raise ValueError("Layer names must be non-empty.")
        plan.validate(topology)
        layers[name] = plan.to_runtime_payload()
    src = dict(source or {})
    src.update({"algorithm": ALGORITHM, "initial_layout": "preloaded", "requires_static_preload": True})
    payload = {
        "schema_version": PLACEMOE_ARTIFACT_SCHEMA_VERSION,
        "source": src,
        "topology": {
            "ep_size": topology.ep_size,
            "ranks_per_node": topology.ranks_per_node,
            "num_experts": topology.num_experts,
            "num_physical_slots": topology.total_slots,
            "slots_per_rank": topology.slots_per_rank,
        },
        "replay": {"actions_by_step": {"1": []}},
        "layers": layers,
    }
    validate_placemoe_artifact(payload)
    return payload


def artifact_topology(payload: Mapping[str, Any]) -> PlaceMoETopology:
    row = payload.get("topology")
    if not isinstance(row, Mapping):
        raise ValueError("PlaceMoE artifact is missing its topology.")
    topo = PlaceMoETopology(
        ep_size=int(row["ep_size"]),
        ranks_per_node=int(row.get("ranks_per_node", row["ep_size"])),
        num_experts=int(row["num_experts"]),
        slots_per_rank=int(row["slots_per_rank"]),
    )
    if int(row.get("num_physical_slots", -1)) != topo.total_slots:
        raise ValueError("Artifact physical-slot count does not match its topology.")
    return topo


def validate_placemoe_artifact(payload: Mapping[str, Any]) -> dict[str, LayerPlan]:
    if int(payload.get("schema_version", -1)) != PLACEMOE_ARTIFACT_SCHEMA_VERSION:
        raise ValueError("Unsupported PlaceMoE artifact schema version.")
    src = payload.get("source")
    if not isinstance(src, Mapping) or src.get("algorithm") != ALGORITHM:
        raise ValueError("Artifact was not produced by the PlaceMoE optimizer.")
    topo = artifact_topology(payload)
    rows = payload.get("layers")
    if not isinstance(rows, Mapping) or not rows:
        raise ValueError("PlaceMoE artifact must contain a non-empty layer table.")
    plans = {}
    for name, row in rows.items():
        if not isinstance(name, str) or not isinstance(row, Mapping):
            raise ValueError("PlaceMoE layer entries must map names to plan objects.")
        plan = LayerPlan.from_runtime_payload(dict(row))
        plan.validate(topo)
        plans[name] = plan
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
