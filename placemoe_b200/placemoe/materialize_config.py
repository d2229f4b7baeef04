"""Write a ready-to-run PlaceMoE runtime configuration for a machine and model.

    python -m placemoe_b200.placemoe.materialize_config --out run/placemoe.yaml \
        --ep-size 8 --num-experts 64 --redundant-slots-per-rank 1 --layers 16 \
        [--seed fixed-ep|mirrored-r2|eplb] [--demand demand.npy] [--calibration cal.json] \
        [--hot-update --layout-interval 100 --mapping-interval 20]

Produces: an initial schema-v2 artifact from the chosen seed layout (fixed
EP, mirrored two-copy replication, or EPLB-style replication on a demand
estimate), the calibration reference, planner resources from the CPU
affinity split (planner cores on the NUMA-balanced reserve, the rest for
training), and the hot-update block.  Paths in the YAML are relative to it.

Reference parity: scripts/placemoe/materialize_config.py.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import yaml


def materialize(out: str, ep_size: int, num_experts: int, layers: int, redundant: int = 0, seed: str = "fixed-ep",
                demand: str = "", calibration: str = "", hot_update: bool = False, layout_interval: int = 100,
                mapping_interval: int = 20, layer_key_template: str = "model.layers.{layer}.mlp.experts") -> dict:
    from .artifacts import build_placemoe_artifact, write_artifact
    from .runtime.cpu_affinity import parse_cpu_list, resolve_cpu_affinity
    from .seeds import eplb_plan, fixed_ep_plan, mirrored_r2_plan
    from .types import PlaceMoETopology

    primary = -(-num_experts // ep_size)
    topo = PlaceMoETopology(ep_size, ep_size, num_experts, primary + redundant)
    if seed == "fixed-ep":
        plan = fixed_ep_plan(topo)
    elif seed == "mirrored-r2":
        plan = mirrored_r2_plan(topo)
    elif seed == "eplb":
        d = np.load(demand) if demand else np.ones(num_experts)
        plan = eplb_plan(topo, d)
    else:
        raise ValueError(f"unknown seed {seed!r}")
    base = os.path.dirname(os.path.abspath(out))
    os.makedirs(base, exist_ok=True)
    plans = {layer_key_template.format(layer=i): plan for i in range(layers)}
    art = os.path.join(base, "initial_layout.json")
    write_artifact(build_placemoe_artifact(plans, topo, source={"planner": "materialize_config", "seed": seed}), art)
    aff = resolve_cpu_affinity()
    cfg = {
        "initial_artifact": os.path.relpath(art, base),
        "calibration": {"artifact": os.path.relpath(os.path.abspath(calibration), base)} if calibration else {},
        "hot_update": {"enabled": bool(hot_update), "layout_interval_steps": layout_interval if hot_update else 0,
                       "mapping_interval_steps": mapping_interval if hot_update else 0,
                       "work_root": "placemoe_work", "failure_policy": "continue"},
        "resources": {"workers": max(1, len(parse_cpu_list(aff.planner_cpu_ids))),
                      "planner_cpu_ids": aff.planner_cpu_ids, "training_cpu_ids": aff.training_cpu_ids},
    }
    with open(out, "w") as f:
        yaml.safe_dump({"placemoe": cfg}, f, sort_keys=False)
    return {"config": os.path.abspath(out), "artifact": art, "topology": {
        "ep_size": ep_size, "num_experts": num_experts, "slots_per_rank": topo.slots_per_rank}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", required=True)
    ap.add_argument("--ep-size", type=int, required=True)
    ap.add_argument("--num-experts", type=int, required=True)
    ap.add_argument("--layers", type=int, required=True)
    ap.add_argument("--redundant-slots-per-rank", type=int, default=0)
    ap.add_argument("--seed", default="fixed-ep", choices=("fixed-ep", "mirrored-r2", "eplb"))
    ap.add_argument("--demand", default="")
    ap.add_argument("--calibration", default="")
    ap.add_argument("--hot-update", action="store_true")
    ap.add_argument("--layout-interval", type=int, default=100)
    ap.add_argument("--mapping-interval", type=int, default=20)
    a = ap.parse_args(argv)
    print(json.dumps(materialize(a.out, a.ep_size, a.num_experts, a.layers, a.redundant_slots_per_rank, a.seed,
                                 a.demand, a.calibration, a.hot_update, a.layout_interval, a.mapping_interval)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
