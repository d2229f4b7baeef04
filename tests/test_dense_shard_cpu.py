"""Sharded dense parameters (ZeRO-2 style) on CPU / gloo: shard layout, equivalence with replicated
training, identical replicas, and checkpoint round trips between sharded and replicated runs."""

import os

import pytest
import torch

from dist_utils import run_distributed


def test_shard_layout_is_aligned_and_covers_everything():
    from placemoe_b200.parallel.dense_shard import SHARD_ALIGN, shard_layout, shardable

    offs, s, n_pad = shard_layout([10, 7, 300], 4)
    assert offs == [0, 10, 17] and s % SHARD_ALIGN == 0 and n_pad == 4 * s and n_pad >= 317
    assert shardable("layers.0.self_attn.qkv_proj", torch.zeros(4, 4))
    assert not shardable("layers.0.mlp.gate", torch.zeros(4, 4))
    assert not shardable("norm.weight", torch.zeros(4))


def _trainer(sharding):
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=2, micro_batch_size=1, lr=1e-3,
                      device="cpu", seed=0, dense_sharding=sharding, max_grad_norm=0.5)
    return Trainer(cfg)


def _worker(rank, world, workdir):
    import torch.distributed as dist

    from placemoe_b200.checkpoint import load_checkpoint, save_checkpoint

    g = torch.Generator().manual_seed(rank)
    batches = [torch.randint(0, 1024, (2, 64), generator=g) for _ in range(4)]
    ref = _trainer("off")
    sh = _trainer("on")
    assert sh.dense_shards is not None and ref.dense_shards is None
    for b in batches[:3]:
        lr_, ls = ref.train_step(b), sh.train_step(b)
        assert abs(lr_ - ls) < 1e-5, (lr_, ls)
    sh.optimizer.sync_params()
    for (n, a), (_, c) in zip(ref.model.named_parameters(), sh.model.named_parameters()):
        assert torch.allclose(a, c, atol=2e-6, rtol=1e-5), n
        if n.endswith(("gate_up_proj", "down_proj")):  # expert slots differ per rank by design
            continue
        ws = [torch.empty_like(c.data) for _ in range(world)]
        dist.all_gather(ws, c.data.contiguous())
        assert all(torch.equal(ws[0], w) for w in ws), n
    # checkpoint of the sharded run resumes both a sharded and a replicated run
    path = save_checkpoint(sh, os.path.join(workdir, "ckpt"))
    nxt = sh.train_step(batches[3])
    for mode in ("on", "off"):
        tr = _trainer(mode)
        load_checkpoint(tr, path)
        got = tr.train_step(batches[3])
        assert abs(got - nxt) < 1e-5, (mode, got, nxt)


def test_sharded_dense_matches_replicated_dp2(tmp_path):
    run_distributed(_worker, 2, str(tmp_path))


def test_sharding_rejects_muon():
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    with pytest.raises(ValueError):
        Trainer(TrainConfig(model="tiny_qwen3_moe", device="cpu", optimizer="muon", dense_sharding="on",
                            seq_len=64, batch_per_rank=2, micro_batch_size=1))
