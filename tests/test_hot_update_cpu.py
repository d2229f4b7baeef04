"""Hot updates on CPU/gloo ranks: migration atomicity, mapping-only install, planner failure policy, staleness."""

import os

import numpy as np
import pytest
import torch

from dist_utils import run_distributed


def _trainer(redundant=1):
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=2, micro_batch_size=2, lr=1e-3,
                      device="cpu", redundant_slots_per_rank=redundant, seed=0, max_grad_norm=0.0)
    return Trainer(cfg)


def _new_payload(tr, seed):
    from placemoe_b200.placemoe import build_placemoe_artifact, eplb_plan

    rng = np.random.default_rng(seed)
    plans = {blk.layer_key: eplb_plan(tr.topology, rng.random((tr.topology.ep_size, tr.topology.num_experts)) * 10)
             for blk in tr.model.moe_blocks()}
    return build_placemoe_artifact(plans, tr.topology)


@torch.no_grad()
def _eval_loss(tr, b):
    loss, _ = tr.model(b, labels=b)
    import torch.distributed as dist

    t = loss.detach().clone()
    dist.all_reduce(t)
    return float(t)


def _worker_migrate(rank, world, workdir):
    import torch.distributed as dist

    from placemoe_b200.parallel.hot_update import HotUpdateManager
    from placemoe_b200.placemoe.runtime.config import PlaceMoERuntimeConfig

    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(rank))
    ref = _trainer()
    tr = _trainer()
    for _ in range(2):
        ref.train_step(b)
        tr.train_step(b)
    mgr = HotUpdateManager(tr, PlaceMoERuntimeConfig())
    before = _eval_loss(tr, b)
    payload = _new_payload(tr, seed=3)
    assert mgr.apply_artifact(payload, None, step=2)
    ev = mgr.events[-1]
    assert ev["event"] == "applied" and ev["moved_slots"] >= 0
    after = _eval_loss(tr, b)
    assert abs(before - after) < 1e-5, (before, after)
    # replicas equal their owner copies, including optimizer moments
    for blk in tr.model.moe_blocks():
        for group in blk.placement.replica_groups():
            for p in (blk.gate_up_proj, blk.down_proj):
                st = tr.optimizer.state[p]
                mine = {int(s): (p[int(s) % 9].clone(), st["exp_avg"][int(s) % 9].clone())
                        for s in group if int(s) // 9 == rank}
                full = [None] * world
                dist.all_gather_object(full, mine)
                merged = {k: v for d in full for k, v in d.items()}
                owner = merged[int(group[0])]
                for s in group:
                    assert torch.equal(merged[int(s)][0], owner[0]) and torch.equal(merged[int(s)][1], owner[1])
    # training continues exactly like the run that never migrated
    for _ in range(2):
        a, c = ref.train_step(b), tr.train_step(b)
        assert abs(a - c) < 1e-5, (a, c)

    # failure injection: rank 1 cannot stage its copies -> every rank keeps the old placement
    from placemoe_b200.parallel import migration

    old = [blk.placement.slot_to_logical.copy() for blk in tr.model.moe_blocks()]
    real = migration.allocate_staging

    def broken(like):
        if rank == 1:
            raise MemoryError("injected staging failure")
        return real(like)

    migration.allocate_staging = broken
    try:
        from placemoe_b200.placemoe import validate_placemoe_artifact

        plans = validate_placemoe_artifact(_new_payload(tr, seed=9))
        blk = tr.model.moe_blocks()[0]
        moved = migration.migrate_layer(tr, blk, plans[blk.layer_key])
        assert moved == 0
    finally:
        migration.allocate_staging = real
    assert np.array_equal(tr.model.moe_blocks()[0].placement.slot_to_logical, old[0])

    # consensus: rank 1 is handed a different plan -> every rank raises, nothing changes
    plans_a = validate_placemoe_artifact(_new_payload(tr, seed=11))
    plans_b = validate_placemoe_artifact(_new_payload(tr, seed=12 if rank == 1 else 11))
    with pytest.raises(migration.MigrationConsensusError, match="disagree"):
        migration.migrate_layer(tr, blk, plans_b[blk.layer_key])
    assert np.array_equal(blk.placement.slot_to_logical, old[0])
    # consensus: rank 0's optimizer holds an extra state tensor per slot -> asymmetric payload everywhere
    real_state = migration._slot_state

    def extra(b, o, j):
        ts = real_state(b, o, j)
        return ts + [ts[0]] if rank == 0 else ts

    migration._slot_state = extra
    try:
        with pytest.raises(migration.MigrationConsensusError, match="asymmetric"):
            migration.migrate_layer(tr, blk, plans_a[blk.layer_key])
    finally:
        migration._slot_state = real_state
    assert np.array_equal(blk.placement.slot_to_logical, old[0])
    # and the same plan still installs afterwards
    migration.migrate_layer(tr, blk, plans_a[blk.layer_key])
    assert np.array_equal(blk.placement.slot_to_logical, np.asarray(plans_a[blk.layer_key].slot_to_logical))


def test_full_install_migrates_state_atomically(tmp_path):
    run_distributed(_worker_migrate, 2, str(tmp_path))


def _worker_policy(rank, world, workdir):
    from placemoe_b200.parallel.hot_update import HotUpdateManager
    from placemoe_b200.placemoe.runtime.config import HotUpdateConfig, PlaceMoERuntimeConfig
    from placemoe_b200.placemoe.runtime.planner_process import HotUpdateJob
    from placemoe_b200.placemoe.runtime.scheduler import UpdateKind

    tr = _trainer()
    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(rank))
    bad = os.path.join(workdir, "missing_planner.py")
    cfg = PlaceMoERuntimeConfig(initial_artifact="x", hot_update=HotUpdateConfig(
        enabled=True, mapping_interval_steps=1, layout_interval_steps=0, work_root=os.path.join(workdir, "hu"),
        planner_path=bad, failure_policy="continue"))
    mgr = HotUpdateManager(tr, cfg, capture_steps=1)
    tr.hot_update = mgr
    before = [blk.placement.slot_to_logical.copy() for blk in tr.model.moe_blocks()]
    for _ in range(8):
        tr.train_step(b)
        if any(e["event"] == "failed" for e in mgr.events):
            break
    assert any(e["event"] == "failed" for e in mgr.events), mgr.events
    for blk, old in zip(tr.model.moe_blocks(), before):
        assert np.array_equal(blk.placement.slot_to_logical, old)
    # stale plan: versions moved since submission -> rejected
    job = HotUpdateJob(UpdateKind.MAPPING_ONLY, 0, tuple(v + 1 for v in mgr._versions()), 0.0, 0.0, "", "", "", "")
    assert not mgr.apply_artifact(mgr.current_artifact(), job, step=9)
    assert mgr.events[-1]["event"] == "rejected_stale"
    # mapping-only install of the current layout with a changed mapping
    payload = mgr.current_artifact()
    job = HotUpdateJob(UpdateKind.MAPPING_ONLY, 0, mgr._versions(), 0.0, 0.0, "", "", "", "")
    assert mgr.apply_artifact(payload, job, step=10)
    assert all(blk.placement.version >= 1 for blk in tr.model.moe_blocks())


def test_planner_failure_keeps_placement_and_stale_plans_are_rejected(tmp_path):
    run_distributed(_worker_policy, 2, str(tmp_path))


def test_failure_policy_raise_single_process(tmp_path):
    from placemoe_b200.parallel.hot_update import HotUpdateManager
    from placemoe_b200.placemoe.runtime.config import HotUpdateConfig, PlaceMoERuntimeConfig

    tr = _trainer(redundant=0)
    cfg = PlaceMoERuntimeConfig(initial_artifact="x", hot_update=HotUpdateConfig(
        enabled=True, mapping_interval_steps=1, work_root=str(tmp_path / "hu"),
        planner_path=str(tmp_path / "nope.py"), failure_policy="raise"))
    tr.hot_update = HotUpdateManager(tr, cfg, capture_steps=1)
    b = torch.randint(0, 1024, (2, 64))
    with pytest.raises(RuntimeError):
        for _ in range(10):
            tr.train_step(b)
