"""Preflight check of a PlaceMoE runtime configuration before a training job.

    python -m placemoe_b200.placemoe.validate_config path/to/placemoe.yaml \
        [--ep-size 8] [--num-experts 64] [--slots-per-rank 9] [--layers 16]

Checks, in order: the YAML/JSON schema (unknown keys and bad values are
errors), the initial artifact (schema v2, every layer valid, topology equal
to the requested one), the calibration artifact (status accepted, scope),
the planner resources (CPU ids exist, planner and training sets disjoint) and
the work root (writable).  Prints one JSON report; exit code 1 on any error.

Reference parity: scripts/placemoe/validate_config.py.
"""

from __future__ import annotations

import argparse
import json
import os
import sys


def validate(path: str, ep_size: int = 0, num_experts: int = 0, slots_per_rank: int = 0, layers: int = 0) -> dict:
    from .artifacts import load_artifact
    from .runtime.config import PlaceMoEConfigurationError, PlaceMoERuntimeConfig

    report: dict = {"config": os.path.abspath(path), "errors": [], "warnings": []}
    try:
        cfg = PlaceMoERuntimeConfig.from_file(path)
        cfg.validate()
    except (PlaceMoEConfigurationError, OSError, ValueError) as e:
        report["errors"].append(f"config: {e}")
        return report
    report["hot_update"] = {"enabled": cfg.hot_update.enabled,
                            "layout_interval_steps": cfg.hot_update.layout_interval_steps,
                            "mapping_interval_steps": cfg.hot_update.mapping_interval_steps}
    if cfg.initial_artifact:
        try:
            _, topo, plans = load_artifact(cfg.initial_artifact)
            report["artifact"] = {"path": cfg.initial_artifact, "layers": len(plans), "ep_size": topo.ep_size,
                                  "num_experts": topo.num_experts, "slots_per_rank": topo.slots_per_rank}
            want = {"ep_size": ep_size, "num_experts": num_experts, "slots_per_rank": slots_per_rank}
            for k, v in want.items():
                if v and getattr(topo, k) != v:
                    report["errors"].append(f"artifact {k} = {getattr(topo, k)}, requested {v}")
            if layers and len(plans) != layers:
                report["errors"].append(f"artifact has {len(plans)} layers, requested {layers}")
        except (OSError, ValueError) as e:
            report["errors"].append(f"initial_artifact: {e}")
    else:
        report["warnings"].append("no initial_artifact: training starts from the identity placement")
    try:
        report["calibration"] = cfg.calibration.coefficients()
    except (PlaceMoEConfigurationError, ValueError) as e:
        report["errors"].append(f"calibration: {e}")
    from .runtime.cpu_affinity import parse_cpu_list

    res = cfg.resources
    ncpu = os.cpu_count() or 1
    sets = {}
    for name in ("planner_cpu_ids", "training_cpu_ids"):
        ids = parse_cpu_list(getattr(res, name, "") or "")
        sets[name] = set(ids)
        bad = [c for c in ids if c < 0 or c >= ncpu]
        if bad:
            report["errors"].append(f"resources.{name}: CPU ids {bad} do not exist (machine has {ncpu})")
    overlap = sets["planner_cpu_ids"] & sets["training_cpu_ids"]
    if overlap:
        report["errors"].append(f"resources: planner and training CPU sets overlap on {sorted(overlap)}")
    if cfg.hot_update.enabled:
        root = cfg.hot_update.work_root or os.path.join(os.path.dirname(os.path.abspath(path)), "placemoe_work")
        try:
            os.makedirs(root, exist_ok=True)
            probe = os.path.join(root, ".write_probe")
            with open(probe, "w") as f:
                f.write("ok")
            os.unlink(probe)
        except OSError as e:
            report["errors"].append(f"hot_update.work_root not writable: {e}")
    return report


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config")
    ap.add_argument("--ep-size", type=int, default=0)
    ap.add_argument("--num-experts", type=int, default=0)
    ap.add_argument("--slots-per-rank", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0)
    a = ap.parse_args(argv)
    rep = validate(a.config, a.ep_size, a.num_experts, a.slots_per_rank, a.layers)
    print(json.dumps(rep, indent=2))
    return 1 if rep["errors"] else 0


if __name__ == "__main__":
    sys.exit(main())
