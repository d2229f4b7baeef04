"""PlaceMoE planner CLI.

    python -m placemoe_b200.placemoe.plan_placemoe --route-root R --optimize-steps 0,1,2 \
        --validation-steps 3 --ep-size 8 --ranks-per-node 8 --num-experts 128 \
        --redundant-slots-per-rank 4 --hidden-size 2048 --output-layout L.json

Per layer (a process pool of ``--workers``): load the captured routes of the
optimisation steps -> statistics -> full (L, M) optimisation, or mapping-only
optimisation of ``--input-layout`` with ``--update-mode mapping`` -> select the
candidate with the lowest route-replay cost on the validation steps ->
schema-v2 artifact.  The report holds per-layer costs, the planner wall time
(``aggregate.planner_wall_ms``), the predicted speed-up over the comparison
layout (``validation_speedup``) and ``e2e_eligible`` (every layer at least as
good as the comparison).

Flag names follow the reference planner (scripts/profile/placemoe_planner.py:112-306)
so that the hot-update command line of either implementation drives either planner.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from concurrent.futures import ProcessPoolExecutor

import numpy as np


def _ints(text: str) -> tuple[int, ...]:
    text = (text or "").strip()
    return tuple(int(x) for x in text.split(",") if x.strip()) if text else ()


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--route-root", required=True)
    p.add_argument("--optimize-steps", default="0")
    p.add_argument("--validation-steps", default="")
    p.add_argument("--update-mode", choices=("full", "mapping"), default="full")
    p.add_argument("--input-layout", default="")
    p.add_argument("--layers", type=int, default=0, help="number of layers (0 = infer from --layer-keys)")
    p.add_argument("--layer-keys", default="", help="comma-separated artifact layer names")
    p.add_argument("--layer-key-template", default="model.layers.{layer}.mlp.experts")
    p.add_argument("--expected-total-layers", type=int, default=0)
    p.add_argument("--workers", type=int, default=1)
    p.add_argument("--candidate-workers", type=int, default=1)
    p.add_argument("--worker-threads", type=int, default=1)
    p.add_argument("--ep-size", type=int, required=True)
    p.add_argument("--ranks-per-node", type=int, default=0)
    p.add_argument("--num-experts", type=int, required=True)
    p.add_argument("--slots-per-rank", type=int, default=0)
    p.add_argument("--primary-slots-per-rank", type=int, default=0)
    p.add_argument("--redundant-slots-per-rank", type=int, default=0)
    p.add_argument("--active-redundant-slots", type=int, default=-1)
    p.add_argument("--hidden-size", type=int, required=True)
    p.add_argument("--bytes-per-element", type=int, default=2)
    p.add_argument("--inter-ms-per-byte", type=float, default=None)
    p.add_argument("--intra-ms-per-byte", type=float, default=None)
    p.add_argument("--route-ms-per-assignment", type=float, default=None)
    p.add_argument("--communication-phase-multiplier", type=float, default=None)
    p.add_argument("--compute-ms-per-assignment", type=float, default=None)
    p.add_argument("--compute-phase-multiplier", type=float, default=None)
    p.add_argument("--comparison-layout", default="fixed-ep", help="'none', 'fixed-ep', 'eplb' or an artifact path")
    p.add_argument("--emit", choices=("placemoe", "eplb"), default="placemoe",
                   help="'eplb': write the EPLB-style replication seed instead of the optimised plan "
                        "(comparison runs)")
    p.add_argument("--rounds", type=int, default=2)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--output-layout", required=True)
    p.add_argument("--output-report", default="")
    return p


def _calibration(args):
    from .runtime.config import PlaceMoECalibration

    d = PlaceMoECalibration()
    pick = lambda v, dv: dv if v is None else v  # noqa: E731
    return PlaceMoECalibration(
        inter_ms_per_byte=pick(args.inter_ms_per_byte, d.inter_ms_per_byte),
        intra_ms_per_byte=pick(args.intra_ms_per_byte, d.intra_ms_per_byte),
        route_ms_per_assignment=pick(args.route_ms_per_assignment, d.route_ms_per_assignment),
        communication_multiplier=pick(args.communication_phase_multiplier, d.communication_multiplier),
        compute_ms_per_assignment=pick(args.compute_ms_per_assignment, d.compute_ms_per_assignment),
        compute_multiplier=pick(args.compute_phase_multiplier, d.compute_multiplier),
    )


def _topology(args):
    from .types import PlaceMoETopology

    spr = args.slots_per_rank
    if not spr:
        primary = args.primary_slots_per_rank or -(-args.num_experts // args.ep_size)
        spr = primary + args.redundant_slots_per_rank
    return PlaceMoETopology(args.ep_size, args.ranks_per_node or args.ep_size, args.num_experts, spr)


def plan_layer(job: dict) -> dict:
    """Plan one layer (runs in a worker process)."""
    os.environ.setdefault("OMP_NUM_THREADS", str(job["threads"]))
    import torch

    if job.get("pooled"):  # a worker process: the route replay runs on --worker-threads threads
        torch.set_num_threads(max(1, int(job["threads"])))
    from .evaluator import RouteReplayEvaluator
    from .optimizer import OptimizerConfig, optimize_fixed_layout_mapping, optimize_replica_allocation
    from .routes import load_routes
    from .seeds import eplb_plan, fixed_ep_plan
    from .statistics import profile_route_statistics
    from .types import LayerPlan

    t0 = time.perf_counter()
    topo, cal = job["topology"], job["calibration"]
    opt = load_routes(job["route_root"], steps=job["optimize_steps"], layer=job["layer"], ep_size=topo.ep_size)
    val = (load_routes(job["route_root"], steps=job["validation_steps"], layer=job["layer"], ep_size=topo.ep_size)
           if job["validation_steps"] else opt)
    stats = profile_route_statistics(opt, num_experts=topo.num_experts)
    ev_opt = RouteReplayEvaluator(opt, topo, hidden_size=job["hidden"], bytes_per_element=job["bpe"], calibration=cal)
    ev_val = RouteReplayEvaluator(val, topo, hidden_size=job["hidden"], bytes_per_element=job["bpe"], calibration=cal)
    cfg = OptimizerConfig(rounds=job["rounds"], seed=job["seed"])
    if job.get("emit") == "eplb":
        from .optimizer import OptimizerCandidate as Candidate

        plan = eplb_plan(topo, stats.demand)
        best = Candidate(plan, ev_opt.evaluate(plan), "eplb")
        vcost, n_cand = ev_val.evaluate(plan), 1
    else:
        if job["mode"] == "mapping":
            current = LayerPlan.from_runtime_payload(job["input_plan"])
            res = optimize_fixed_layout_mapping(stats, topo, current, ev_opt, cfg)
        else:
            res = optimize_replica_allocation(stats, topo, ev_opt, cfg)
        # held-out selection among the candidates (best few by optimisation cost)
        ranked = sorted(res.candidates, key=lambda c: c.cost.total_ms)[:8]
        scored = [(ev_val.evaluate(c.plan), c) for c in ranked]
        vcost, best = min(scored, key=lambda r: (r[0].total_ms, r[1].label))
        n_cand = len(res.candidates)
    comparison = None
    if job["comparison"] == "fixed-ep":
        try:
            comparison = ev_val.evaluate(fixed_ep_plan(topo)).total_ms
        except ValueError:
            comparison = None
    elif job["comparison"] == "eplb":
        comparison = ev_val.evaluate(eplb_plan(topo, stats.demand)).total_ms
    elif job["comparison_plan"] is not None:
        comparison = ev_val.evaluate(LayerPlan.from_runtime_payload(job["comparison_plan"])).total_ms
    return {
        "layer": job["layer"], "key": job["key"], "plan": best.plan.to_runtime_payload(), "label": best.label,
        "optimize_cost_ms": best.cost.total_ms, "validation_cost_ms": vcost.total_ms,
        "validation_comm_ms": vcost.comm_ms, "validation_compute_ms": vcost.compute_ms,
        "dedup_ratio": vcost.dedup_ratio, "comparison_cost_ms": comparison,
        "candidates": n_cand, "wall_ms": (time.perf_counter() - t0) * 1e3,
    }


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    from .artifacts import build_placemoe_artifact, load_artifact, write_artifact
    from .types import LayerPlan

    t0 = time.perf_counter()
    topo = _topology(args)
    cal = _calibration(args)
    keys = [k for k in args.layer_keys.split(",") if k] if args.layer_keys else []
    nlayers = args.layers or len(keys)
    if not nlayers:
        raise SystemExit("--layers or --layer-keys is required")
    if not keys:
        keys = [args.layer_key_template.format(layer=i) for i in range(nlayers)]
    if len(keys) != nlayers:
        raise SystemExit("--layer-keys does not match --layers")
    if args.expected_total_layers and args.expected_total_layers != nlayers:
        raise SystemExit("--expected-total-layers does not match the planned layer count")
    input_plans = {}
    if args.update_mode == "mapping":
        if not args.input_layout:
            raise SystemExit("--update-mode mapping requires --input-layout")
        _, in_topo, input_plans = load_artifact(args.input_layout)
        if in_topo != topo:
            raise SystemExit("--input-layout topology differs from the requested topology")
    comparison_plans = {}
    if args.comparison_layout not in ("none", "fixed-ep", "eplb"):
        _, _, comparison_plans = load_artifact(args.comparison_layout)
    jobs = []
    for i, key in enumerate(keys):
        jobs.append({
            "layer": i, "key": key, "topology": topo, "calibration": cal, "route_root": args.route_root,
            "optimize_steps": _ints(args.optimize_steps), "validation_steps": _ints(args.validation_steps),
            "hidden": args.hidden_size, "bpe": args.bytes_per_element, "rounds": args.rounds, "seed": args.seed,
            "mode": args.update_mode, "threads": args.worker_threads,
            "pooled": args.workers > 1 and nlayers > 1,
            "input_plan": input_plans[key].to_runtime_payload() if key in input_plans else None,
            "comparison": args.comparison_layout, "emit": args.emit,
            "comparison_plan": comparison_plans[key].to_runtime_payload() if key in comparison_plans else None,
        })
        if args.update_mode == "mapping" and key not in input_plans:
            raise SystemExit(f"--input-layout has no layer {key}")
    if args.workers > 1 and len(jobs) > 1:
        import multiprocessing as mp

        with ProcessPoolExecutor(max_workers=min(args.workers, len(jobs)), mp_context=mp.get_context("spawn")) as ex:
            rows = list(ex.map(plan_layer, jobs))
    else:
        rows = [plan_layer(j) for j in jobs]
    plans = {r["key"]: LayerPlan.from_runtime_payload(r["plan"]) for r in rows}
    payload = build_placemoe_artifact(plans, topo, source={
        "planner": "placemoe_b200", "update_mode": args.update_mode,
        "optimize_steps": list(_ints(args.optimize_steps)), "validation_steps": list(_ints(args.validation_steps)),
    })
    write_artifact(payload, args.output_layout)
    wall = (time.perf_counter() - t0) * 1e3
    val = sum(r["validation_cost_ms"] for r in rows)
    comp = [r["comparison_cost_ms"] for r in rows]
    have_comp = all(c is not None for c in comp)
    report = {
        "layers": [{k: v for k, v in r.items() if k != "plan"} for r in rows],
        "aggregate": {
            "planner_wall_ms": wall,
            "validation_cost_ms": val,
            "comparison_cost_ms": sum(comp) if have_comp else None,
            "validation_speedup": (sum(comp) / val) if have_comp and val > 0 else None,
            "e2e_eligible": bool(have_comp and all(r["validation_cost_ms"] <= r["comparison_cost_ms"] + 1e-9
                                                   for r in rows)),
            "mean_dedup_ratio": float(np.mean([r["dedup_ratio"] for r in rows])),
        },
        "topology": {"ep_size": topo.ep_size, "ranks_per_node": topo.ranks_per_node,
                     "num_experts": topo.num_experts, "slots_per_rank": topo.slots_per_rank},
    }
    if args.output_report:
        os.makedirs(os.path.dirname(os.path.abspath(args.output_report)), exist_ok=True)
        with open(args.output_report, "w") as f:
            json.dump(report, f, indent=2)
    print(json.dumps(report["aggregate"]))
    return 0


if __name__ == "__main__":
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(os.path.dirname(here))
    if root not in sys.path:
        sys.path.insert(0, root)
    from placemoe_b200.placemoe.plan_placemoe import main as _main

    sys.exit(_main())
