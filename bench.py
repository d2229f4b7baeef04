"""Headline benchmark: MoE training tokens/s (OLMoE-1B-7B shape, FSDP-style DP + EP = world size).

    python bench.py [--gpus N --steps K --warmup W] [--impl native|reference] [--model olmoe_1b_7b]

For N > 1 launch with torchrun (one rank per GPU, NCCL).  Per rank: a batch of
``--batch-per-gpu`` sequences x ``--seq`` tokens of uniform random ids
(synthetic, seeded), random-init weights of the named architecture, router
bias 0.5 * log Zipf(s=1.0) redrawn per layer.  A step = forward + backward of
every micro-batch + replica/DP gradient reduction + grad clipping + AdamW.

Timing: W untimed warm-up steps; then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the
launching stream; the max over ranks is reported.  The working set of a step
(weights, optimizer state, activations: tens of GB) is far larger than the
126 MB L2, so no separate L2 flush is done.  ``e2e`` repeats the
measurement through the public Trainer.train_step API with the input copied
host->device from pinned memory and the loss read back every step.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

BASELINE_METRIC = "MoE train tokens/s (Qwen3-30B-A3B EP8; OLMoE at 1/2/4/8 GPU); exposed a2a ms/step"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--model", default="olmoe_1b_7b")
    p.add_argument("--seq", type=int, default=4096)
    p.add_argument("--batch-per-gpu", type=int, default=8)
    p.add_argument("--micro-batch", type=int, default=0,
                   help="sequences per micro-batch (default 4; 1 for qwen3_30b_a3b, whose 48 layers of saved "
                        "activations and receive slabs would not fit 180 GB at 2)")
    p.add_argument("--redundant-slots", type=int, default=-1,
                   help="extra expert slots per GPU for replicas (default when N > 1: 4 for qwen3_30b_a3b, "
                        "else 1; 0 on one GPU)")
    p.add_argument("--placement", default="placemoe", choices=("placemoe", "fixed_ep", "eplb"),
                   help="N > 1: PlaceMoE L,M planned from captured routes, plain EP, or EPLB-style replication "
                        "from the captured demand")
    p.add_argument("--plan-steps", type=int, default=-1,
                   help="steps of captured routes the PlaceMoE planner uses before timing (default: 20 when N > 1)")
    p.add_argument("--capture-seq", type=int, default=-1,
                   help="sequence length of the route-capture steps before planning (default: the full --seq; "
                        "1024 for qwen3_30b_a3b, whose unplanned skewed layout would otherwise size the receive "
                        "slabs for ~4x the balanced load)")
    p.add_argument("--artifact", default="")
    p.add_argument("--layers", type=int, default=0, help="override layer count (diagnostics only)")
    p.add_argument("--ep-transport", default="auto", choices=("auto", "p2p", "nccl"))
    p.add_argument("--dense-sharding", default="auto", choices=["auto", "on", "off"],
                   help="shard dense masters/moments/gradients over the ranks (peer-memory RS/AG); auto = N > 1")
    p.add_argument("--adaptive", type=int, default=0,
                   help="N > 1: after the timed run, N steps with PlaceMoE hot updates while the router bias "
                        "rotates, then N steps on the static placement for comparison")
    p.add_argument("--rotate-every", type=int, default=50, help="adaptive run: rotate the bias every R steps")
    p.add_argument("--rotate-by", type=int, default=16, help="adaptive run: experts per rotation")
    p.add_argument("--mapping-every", type=int, default=20, help="adaptive run: mapping-only update interval")
    p.add_argument("--layout-every", type=int, default=100, help="adaptive run: full (layout) update interval")
    p.add_argument("--ref-no-recompute", action="store_true",
                   help="reference arm: gradient checkpointing off (its trainer default is on)")
    p.add_argument("--ref-hiermoe", default="off", choices=("off", "dedup"),
                   help="reference arm, N > 1: 'dedup' enables its HierMoE token-deduplicated dispatch/combine "
                        "(direct all-to-all, no expert swap); its trainer default is off")
    p.add_argument("--ulysses", type=int, default=1,
                   help="Ulysses sequence-parallel group size (consecutive ranks share a batch; attention runs "
                        "on whole sequences over head groups)")
    p.add_argument("--recompute-expert-rows", action="store_true",
                   help="re-gather dispatched expert inputs in the backward instead of keeping them (memory)")
    args = p.parse_args()
    if args.micro_batch <= 0:
        args.micro_batch = 1 if args.model == "qwen3_30b_a3b" else 4
    return args


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = f"/tmp/pm_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = sorted(v for v in (num(r[1]) for r in rows) if v is not None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": num(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max((num(r[3]) or 0) for r in rows)}


def plan_placement(trainer, pool, args, rank, world):
    """PlaceMoE static placement for the timed run: capture routes for ``plan_steps``
    training steps, plan L,M on rank 0 (CPU planner), install on every rank with
    parameter + optimizer-state migration.  Returns a summary for the JSON line."""
    import tempfile

    import torch

    import torch.distributed as dist

    from placemoe_b200.parallel.migration import migrate_layer
    from placemoe_b200.parallel.route_capture import RouteRecorder
    from placemoe_b200.placemoe import plan_placemoe
    from placemoe_b200.placemoe.artifacts import validate_placemoe_artifact

    root = tempfile.mkdtemp(prefix="pm_routes_") if rank == 0 else ""
    holder = [root]
    dist.broadcast_object_list(holder, src=0)
    root = holder[0]
    rec = RouteRecorder(trainer.model, root)
    rec.enabled = True
    cap_seq = args.capture_seq if args.capture_seq > 0 else args.seq
    for s in range(args.plan_steps):
        trainer.train_step(next(pool)[:, :cap_seq])
        rec.record_step(s)
    rec.enabled = False
    for blk in trainer.model.moe_blocks():
        blk.route_sink = None
    cfg = trainer.model_cfg
    t0 = time.perf_counter()
    payload = [None]
    report = [None]
    if rank == 0:
        out = os.path.join(root, "layout.json")
        ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
        workers = min(8, ncpu)
        plan_placemoe.main([
            "--route-root", root, "--optimize-steps", ",".join(str(i) for i in range(args.plan_steps)),
            "--ep-size", str(world), "--num-experts", str(cfg.num_experts),
            "--redundant-slots-per-rank", str(args.redundant_slots), "--hidden-size", str(cfg.hidden_size),
            "--layers", str(cfg.num_hidden_layers), "--workers", str(workers),
            "--worker-threads", str(max(1, ncpu // workers)),
            "--output-layout", out, "--output-report", os.path.join(root, "report.json"),
            "--emit", "eplb" if args.placement == "eplb" else "placemoe",
        ])
        with open(os.path.join(root, "report.json")) as f:
            report[0] = json.load(f)["aggregate"]
        with open(out) as f:
            payload[0] = json.load(f)
    dist.broadcast_object_list(payload, src=0)
    planner_ms = (time.perf_counter() - t0) * 1e3
    plans = validate_placemoe_artifact(payload[0])
    t1 = time.perf_counter()
    moved = 0
    for blk in trainer.model.moe_blocks():
        moved += migrate_layer(trainer, blk, plans[blk.layer_key])
    trainer._norm_table = None
    trainer.optimizer.reset_tables()
    # the capture steps ran on the unplanned layout; the planned one is balanced, so the receive slabs go
    # back to the default capacity (a new arena is allocated at the next step, collectively)
    ep = trainer.pstate.ep
    if hasattr(ep, "arena"):
        ep.arena = None
        ep.capacity_factor = 2.0
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    dist.barrier()
    agg = report[0] or {}
    return {"plan_steps": args.plan_steps, "planner_ms": round(planner_ms, 1),
            "install_ms": round((time.perf_counter() - t1) * 1e3, 1), "moved_slots": moved,
            "emitted": args.placement,
            "modelled_speedup_vs_fixed_ep": (round(agg["validation_speedup"], 3)
                                             if agg.get("validation_speedup") else None),
            "mean_dedup_ratio": round(agg.get("mean_dedup_ratio", 0.0), 3)}


def adaptive_run(trainer, pool, args, rank, world):
    """Hot-update run: ``args.adaptive`` steps with mapping-only updates every ``mapping_every`` steps and
    full layout updates (expert weights + AdamW moments migrated peer to peer) every ``layout_every``
    steps, planned asynchronously on rank 0's CPU from captured routes, while the router bias
    permutation rotates by ``rotate_by`` experts every ``rotate_every`` steps.  Then the same number of
    steps, same rotation, on the static placement (run first, before any update).  Device time is measured
    with CUDA events around every step (max over ranks)."""
    import tempfile

    import torch
    import torch.distributed as dist

    from placemoe_b200.parallel.hot_update import HotUpdateManager
    from placemoe_b200.placemoe.runtime.config import HotUpdateConfig, PlaceMoEPlannerResources, PlaceMoERuntimeConfig

    root = tempfile.mkdtemp(prefix="pm_hot_") if rank == 0 else ""
    holder = [root]
    dist.broadcast_object_list(holder, src=0)
    cfg = PlaceMoERuntimeConfig(
        hot_update=HotUpdateConfig(enabled=True, layout_interval_steps=args.layout_every,
                                   mapping_interval_steps=args.mapping_every, work_root=holder[0]),
        resources=PlaceMoEPlannerResources(workers=min(8, os.cpu_count() or 1), candidate_workers=1))
    blocks = trainer.model.moe_blocks()
    base = [blk.router_bias.clone() for blk in blocks]

    def run(n, manager):
        trainer.hot_update = manager
        for blk, b in zip(blocks, base):
            blk.router_bias.copy_(b)
        times = []
        for i in range(n):
            if i and i % args.rotate_every == 0:
                for blk in blocks:
                    blk.router_bias.copy_(torch.roll(blk.router_bias, args.rotate_by))
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            trainer.train_step(next(pool), read_loss=False)
            e.record()
            times.append((s, e))
        torch.cuda.synchronize()
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in times)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        trainer.hot_update = None
        return float(t.item())

    t_static = run(args.adaptive, None)  # first: the static artifact as installed
    mgr = HotUpdateManager(trainer, cfg)
    t_adapt = run(args.adaptive, mgr)
    tokens = args.batch_per_gpu * args.seq * world * args.adaptive
    ev = mgr.events
    applied = [e for e in ev if e["event"] == "applied"]
    full = [e for e in applied if e["kind"] == "full"]
    return {
        "steps": args.adaptive, "rotate_every": args.rotate_every, "rotate_by": args.rotate_by,
        "mapping_every": args.mapping_every, "layout_every": args.layout_every,
        "tokens_per_s_adaptive": round(tokens / (t_adapt / 1e3), 1),
        "tokens_per_s_static": round(tokens / (t_static / 1e3), 1),
        "mapping_updates": sum(1 for e in applied if e["kind"] == "mapping"),
        "layout_updates": len(full),
        "migration_ms_per_layout_update": round(sum(e["migration_ms"] for e in full) / max(1, len(full)), 1),
        "moved_slots_per_layout_update": round(sum(e["moved_slots"] for e in full) / max(1, len(full)), 1),
        "planner_ms_mean": round(sum(e["planner_ms"] for e in applied) / max(1, len(applied)), 1),
        "staleness_steps_mean": round(sum(e["staleness_steps"] for e in applied) / max(1, len(applied)), 2),
        "failed_or_stale": sum(1 for e in ev if e["event"] in ("failed", "rejected_stale")),
    }


def run_reference(args):
    from baseline_reference import run as ref_run  # noqa: E402  (baseline/ helper)

    return ref_run(args)


def main():
    args = parse()
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        try:
            import baseline_reference
        except Exception as e:  # pragma: no cover
            print(json.dumps({"impl": "reference", "unavailable": f"reference harness failed to import: {e}"}))
            return 0
        return baseline_reference.main(args)

    import torch
    import torch.distributed as dist

    from placemoe_b200.data import PinnedBatchPool
    from placemoe_b200.models.config import get_preset
    from placemoe_b200.ops import kernels
    from placemoe_b200.trainer.base import TrainConfig, Trainer, init_distributed

    rank, world = init_distributed()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    big = args.model == "qwen3_30b_a3b"
    if args.placement == "fixed_ep":
        args.redundant_slots = 0
    if args.redundant_slots < 0:
        args.redundant_slots = (4 if big else 1) if world > 1 else 0
    if args.capture_seq < 0:
        args.capture_seq = 1024 if big else 0
    if args.plan_steps < 0:
        args.plan_steps = 20 if world > 1 and not args.artifact and args.placement != "fixed_ep" else 0
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    overrides = {"num_hidden_layers": args.layers} if args.layers else {}
    mcfg = get_preset(args.model, **overrides)
    cfg = TrainConfig(model=args.model, seq_len=args.seq, batch_per_rank=args.batch_per_gpu,
                      micro_batch_size=args.micro_batch, redundant_slots_per_rank=args.redundant_slots,
                      placemoe_artifact=args.artifact, total_steps=args.warmup + 2 * args.steps + 1,
                      ep_transport=args.ep_transport, recompute_expert_rows=args.recompute_expert_rows,
                      dense_sharding=args.dense_sharding, ulysses_size=args.ulysses)
    trainer = Trainer(cfg, mcfg)
    # ranks of one sequence-parallel group read the same sequences (each keeps its chunk of them)
    pool = PinnedBatchPool(mcfg.vocab_size, args.batch_per_gpu, args.seq, n=2, seed=0, rank=rank // args.ulysses)
    dev_batches = [b.to("cuda") for b in pool.batches]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    plan_info = plan_placement(trainer, pool, args, rank, world) if args.plan_steps > 0 else None

    for i in range(args.warmup):
        trainer.train_step(next(pool))
    barrier()

    # ---- device-timed region: inputs already resident, no host reads
    kn = kernels()
    kn.reset()
    kn.counting = True
    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select exactly the timed steps
    start.record()
    for i in range(args.steps):
        trainer.train_step(dev_batches[i % len(dev_batches)], read_loss=False)
    end.record()
    torch.cuda.nvtx.range_pop()
    barrier()
    clocks = sampler.stop()
    kn.counting = False
    launches = kn.launches()
    ms = start.elapsed_time(end) / args.steps

    # ---- end-to-end through the public API: pinned H2D input + loss D2H every step
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    last = None
    for i in range(args.steps):
        last = trainer.train_step(next(pool), read_loss=True)
    e2.record()
    barrier()
    ms_e2e = s2.elapsed_time(e2) / args.steps

    # ---- exposed all-to-all: one more step with CUDA events around every EP communication kernel.
    # Those kernels run on the compute stream, so their summed time is the exposed a2a time per step.
    a2a = {}
    from placemoe_b200.parallel import p2p_ep

    if world > 1 and isinstance(trainer.pstate.ep, p2p_ep.P2PExpertParallel):
        barrier()
        p2p_ep.TIMER = p2p_ep.PhaseTimer()
        trainer.train_step(dev_batches[0], read_loss=False)
        barrier()
        a2a = p2p_ep.TIMER.phases()
        p2p_ep.TIMER = None
    adaptive = adaptive_run(trainer, pool, args, rank, world) if args.adaptive > 0 and world > 1 else None
    names = ["dispatch", "combine", "scatter", "combine_bwd"]
    t = torch.tensor([ms, ms_e2e, sum(a2a.values())] + [a2a.get(n, 0.0) for n in names], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    vals = t.tolist()
    ms, ms_e2e, a2a_ms = vals[:3]
    a2a_phases = dict(zip(names, (round(v, 3) for v in vals[3:])))
    tokens = args.batch_per_gpu * args.seq * world // args.ulysses  # an SP group shares its sequences
    value = tokens / (ms / 1e3)
    e2e = tokens / (ms_e2e / 1e3)
    if rank == 0:
        flops = mcfg.flops_per_token(args.seq) * tokens
        line = {
            "metric": "MoE train tokens/s",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic uniform token ids (seeded), random-init weights",
            "config": {
                "model": f"{args.model} ({mcfg.num_hidden_layers}L, H{mcfg.hidden_size}, {mcfg.num_experts}E "
                         f"top{mcfg.num_experts_per_tok}, I{mcfg.moe_intermediate_size}, V{mcfg.vocab_size})",
                "global_batch": args.batch_per_gpu * world // args.ulysses,
                "seq_len": args.seq,
                "micro_batch": args.micro_batch,
                "parallelism": f"dp{world // args.ulysses}+ep{world}" +
                               (f"+sp{args.ulysses}" if args.ulysses > 1 else "") +
                               ("+dense-shard" if trainer.dense_shards is not None else ""),
                "ep_transport": args.ep_transport if world > 1 else "none",
                "placement": ((f"PlaceMoE static L,M planned from {args.plan_steps} captured steps, "
                               if args.placement == "placemoe" else
                               f"EPLB-style replication from {args.plan_steps} captured steps, ")
                              + f"{args.redundant_slots} replica slot(s)/GPU" if plan_info else
                              ("artifact " + args.artifact if args.artifact else
                               ("fixed EP" if world > 1 else "single GPU"))),
                "router_bias": f"{mcfg.router_bias_scale} * log Zipf(s={mcfg.router_bias_zipf_s})",
                "l2": "working set >> 126 MB L2 (no explicit flush)",
                "baseline_metric": BASELINE_METRIC,
            },
            "clocks": clocks,
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": pool.bytes_per_batch,
                    "d2h_bytes_per_step": 4, "ms_per_step": round(ms_e2e, 3), "last_loss": last},
            "exposed_a2a_ms_per_step": round(a2a_ms, 3) if world > 1 and a2a else None,
            "a2a_phases_ms_per_step": a2a_phases if world > 1 and a2a else None,
            "gpu_launches": launches,
            "peak_mem_gb": round(torch.cuda.max_memory_allocated() / 2**30, 1),
            "planner": plan_info,
            "adaptive": adaptive,
            "model_tflops_per_gpu": round(flops / (ms / 1e3) / world / 1e12, 1),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
