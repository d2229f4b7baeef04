"""The CPU/gloo plumbing run of the benchmark plan: EP=2 with a planned PlaceMoE artifact.

Tiny Qwen3-MoE (4 layers, hidden 256, 8q/2kv x 32, 16 experts top-4, I 128,
vocab 1024), fp32, batch 2 x 256 uniform ids (seed 0), router bias
0.5 * log Zipf(1.1).  Routes of 4 steps are captured, the planner builds an
artifact with one extra replica slot per rank, and a run that loads it at
startup must reproduce the losses of the run without placement (1e-5).
"""

import json
import os

import torch

from dist_utils import run_distributed

STEPS = 10  # the 10-step plumbing run of the benchmark plan


def _trainer(artifact="", capture=False, redundant=0):
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=256, batch_per_rank=2, micro_batch_size=2, lr=1e-3,
                      device="cpu", placemoe_artifact=artifact, capture_routes=capture,
                      redundant_slots_per_rank=redundant, max_grad_norm=1.0, total_steps=STEPS, seed=0)
    return Trainer(cfg)


def _batches(rank):
    from placemoe_b200.data import SyntheticTokens

    data = SyntheticTokens(1024, 2, 256, seed=0, rank=rank)
    return [next(data) for _ in range(STEPS)]


def _worker(rank, world, workdir):
    import torch.distributed as dist

    from placemoe_b200.parallel.route_capture import RouteRecorder
    from placemoe_b200.placemoe.plan_placemoe import main as plan_main

    torch.manual_seed(0)
    batches = _batches(rank)
    # run A: fixed EP, capture routes of the first 4 steps
    tr = _trainer(capture=True)
    rec = RouteRecorder(tr.model, os.path.join(workdir, "routes"))
    base = []
    for s, b in enumerate(batches):
        rec.enabled = s < 4
        base.append(tr.train_step(b))
        if s < 4:
            rec.record_step(s)
    # planner on rank 0 (one extra replica slot per rank)
    art = os.path.join(workdir, "layout.json")
    if rank == 0:
        rc = plan_main(["--route-root", os.path.join(workdir, "routes"), "--optimize-steps", "0,1,2",
                        "--validation-steps", "3", "--layers", "4", "--ep-size", "2", "--num-experts", "16",
                        "--redundant-slots-per-rank", "1", "--hidden-size", "256", "--bytes-per-element", "4",
                        "--output-layout", art, "--output-report", os.path.join(workdir, "report.json")])
        assert rc == 0
    dist.barrier()
    payload = json.load(open(art))
    assert payload["schema_version"] == 2 and payload["topology"]["slots_per_rank"] == 9
    # run B: load the artifact at startup
    tr2 = _trainer(artifact=art)
    assert tr2.model.layers[0].mlp.num_local_slots == 9
    placed = [tr2.train_step(b) for b in batches]
    for a, b in zip(base, placed):
        assert abs(a - b) <= 1e-5 * max(1.0, abs(a)), (base, placed)
    # copies of every replicated expert stay identical after optimizer steps
    for blk in tr2.model.moe_blocks():
        pl = blk.placement
        for group in pl.replica_groups():
            owner = group[0]
            for p in (blk.gate_up_proj, blk.down_proj):
                full = [None] * world
                mine = {int(s): p[int(s) % 9].detach() for s in group if int(s) // 9 == rank}
                dist.all_gather_object(full, mine)
                merged = {k: v for d in full for k, v in d.items()}
                for s in group:
                    assert torch.equal(merged[int(s)], merged[int(owner)])
    if rank == 0:
        with open(os.path.join(workdir, "losses.json"), "w") as f:
            json.dump({"base": base, "placed": placed}, f)


def test_ep2_placemoe_artifact_preserves_loss(tmp_path):
    run_distributed(_worker, 2, str(tmp_path))
    res = json.load(open(tmp_path / "losses.json"))
    assert len(res["placed"]) == STEPS
