"""Checkpoint / resume on CPU: DCP round trip with logical experts, placement restore, HF export."""

import json
import os

import numpy as np
import torch

from dist_utils import run_distributed


def _trainer(artifact="", redundant=0):
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=2, micro_batch_size=2, lr=1e-3,
                      device="cpu", placemoe_artifact=artifact, redundant_slots_per_rank=redundant, seed=0)
    return Trainer(cfg)


def _artifact(path, ep=2, e=16, spr=9, seed=0):
    """A valid random plan with one replica slot per rank."""
    from placemoe_b200.placemoe import PlaceMoETopology, build_placemoe_artifact, eplb_plan, write_artifact

    topo = PlaceMoETopology(ep, ep, e, spr)
    rng = np.random.default_rng(seed)
    plans = {f"model.layers.{i}.mlp.experts": eplb_plan(topo, rng.random((ep, e)) * 10) for i in range(4)}
    write_artifact(build_placemoe_artifact(plans, topo), path)


def _worker(rank, world, workdir):
    from placemoe_b200.checkpoint import export_hf, load_checkpoint, save_checkpoint

    torch.manual_seed(0)
    art = os.path.join(workdir, "a.json")
    if rank == 0:
        _artifact(art)
    import torch.distributed as dist

    dist.barrier()
    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(rank))
    tr = _trainer(artifact=art)
    for _ in range(2):
        tr.train_step(b)
    path = save_checkpoint(tr, os.path.join(workdir, "ckpt"))
    ref_next = tr.train_step(b)  # loss of the step after the checkpoint
    # resume into a run WITHOUT placement (identity layout, 8 slots/rank): logical experts must carry over
    tr2 = _trainer()
    load_checkpoint(tr2, path)
    assert tr2.global_step == 2
    got_next = tr2.train_step(b)
    assert abs(got_next - ref_next) < 1e-4, (got_next, ref_next)
    # resume into the same placement restores it exactly
    tr3 = _trainer(artifact=art)
    extra = load_checkpoint(tr3, path)
    assert "placemoe" in extra
    for blk, blk3 in zip(tr.model.moe_blocks(), tr3.model.moe_blocks()):
        assert np.array_equal(blk.placement.slot_to_logical, blk3.placement.slot_to_logical)
    assert abs(tr3.train_step(b) - ref_next) < 1e-4
    out = export_hf(tr2, os.path.join(workdir, "hf"))
    if rank == 0:
        cfg = json.load(open(os.path.join(out, "config.json")))
        assert cfg["num_experts"] == 16
        from safetensors import safe_open

        with safe_open(os.path.join(out, "model.safetensors"), framework="pt") as f:
            keys = set(f.keys())
        assert "model.layers.3.mlp.experts.15.down_proj.weight" in keys
        assert "model.layers.0.self_attn.k_proj.weight" in keys


def test_checkpoint_roundtrip_across_placements(tmp_path):
    run_distributed(_worker, 2, str(tmp_path))


def test_hf_export_load_roundtrip_single_process(tmp_path):
    from placemoe_b200.checkpoint import export_hf, load_hf_weights

    tr = _trainer()
    out = export_hf(tr, str(tmp_path / "hf"))
    tr2 = _trainer()
    with torch.no_grad():
        for p in tr2.model.parameters():
            p.zero_()
    load_hf_weights(tr2, out)
    for (n, a), (_, b) in zip(tr.model.named_parameters(), tr2.model.named_parameters()):
        assert torch.allclose(a.bfloat16().float(), b, atol=0, rtol=0), n


def _digest_worker(rank, world, workdir):
    """Rank 1's placement digest is replaced by a fake that disagrees: every rank must refuse the load
    before any tensor is read, and the model must keep its pre-load values."""
    import pytest

    from placemoe_b200.checkpoint import checkpointer, load_checkpoint, save_checkpoint

    torch.manual_seed(0)
    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(rank))
    tr = _trainer()
    tr.train_step(b)
    path = save_checkpoint(tr, os.path.join(workdir, "ckpt"))
    tr2 = _trainer()
    before = {n: p.detach().clone() for n, p in tr2.model.named_parameters()}
    if rank == 1:
        real = checkpointer.placement_digest
        checkpointer.placement_digest = lambda trainer: real(trainer) + 1
    try:
        with pytest.raises(RuntimeError, match="differs across ranks"):
            load_checkpoint(tr2, path)
    finally:
        if rank == 1:
            checkpointer.placement_digest = real
    for n, p in tr2.model.named_parameters():
        assert torch.equal(p.detach(), before[n]), n
    assert tr2.global_step == 0


def test_checkpoint_digest_mismatch_refused_on_every_rank(tmp_path):
    run_distributed(_digest_worker, 2, str(tmp_path))
