"""Optimizers and learning-rate schedules on CPU: schedule shapes, Newton-Schulz orthogonality,
Muon descent, the Muon + AdamW split inside the trainer, and a checkpoint round trip of Muon state."""

import math

import pytest
import torch


def test_lr_schedules():
    from placemoe_b200.optim import build_lr_scheduler

    cos = build_lr_scheduler("cosine", 1.0, warmup_steps=10, total_steps=110, min_lr_ratio=0.1)
    assert cos(0) == pytest.approx(0.1) and cos(9) == pytest.approx(1.0)
    assert cos(10) == pytest.approx(1.0)
    assert cos(60) == pytest.approx(0.1 + 0.9 * 0.5)
    assert cos(110) == pytest.approx(0.1) and cos(500) == pytest.approx(0.1)
    lin = build_lr_scheduler("linear", 2.0, warmup_ratio=0.0, total_steps=100, min_lr_ratio=0.0)
    assert lin(50) == pytest.approx(1.0) and lin(100) == pytest.approx(0.0)
    const = build_lr_scheduler("constant", 0.5, warmup_steps=4, total_steps=10)
    assert const(1) == pytest.approx(0.25) and const(7) == pytest.approx(0.5)
    with pytest.raises(ValueError):
        build_lr_scheduler("step", 1.0)


@pytest.mark.parametrize("shape", [(64, 32), (32, 96), (3, 48, 16)])
def test_newton_schulz_is_nearly_orthogonal(shape):
    from placemoe_b200.optim import zeropower_newton_schulz

    torch.manual_seed(0)
    g = torch.randn(*shape)
    o = zeropower_newton_schulz(g)
    sv = torch.linalg.svdvals(o.double())
    # the quintic iteration maps every singular value into roughly [0.7, 1.2]
    assert sv.min() > 0.55 and sv.max() < 1.25
    # batched input = per-matrix results
    if g.dim() == 3:
        for i in range(g.shape[0]):
            assert torch.allclose(o[i], zeropower_newton_schulz(g[i]), atol=1e-5)


def test_muon_descends_on_a_matrix_objective():
    from placemoe_b200.optim import Muon

    torch.manual_seed(1)
    target = torch.randn(32, 16)
    w = torch.nn.Parameter(torch.zeros(32, 16))
    opt = Muon([w], lr=0.05, momentum=0.9)
    first = None
    for _ in range(60):
        loss = (w - target).pow(2).sum()
        first = first if first is not None else loss.item()
        w.grad = None
        loss.backward()
        opt.step()
    assert (w - target).pow(2).sum().item() < 0.2 * first
    with pytest.raises(ValueError):
        Muon([torch.nn.Parameter(torch.zeros(4))])


def _trainer(optimizer="muon", **kw):
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=2, micro_batch_size=1, lr=1e-3,
                      device="cpu", optimizer=optimizer, lr_scheduler="linear", warmup_steps=1, total_steps=4,
                      seed=0, **kw)
    return Trainer(cfg)


def test_trainer_muon_split_and_schedule():
    from placemoe_b200.optim import MultiOptimizer, state_tensors

    tr = _trainer()
    opt = tr.optimizer
    assert isinstance(opt, MultiOptimizer) and set(opt.optimizers) == {"muon", "adamw"}
    muon_ids = {id(p) for g in opt.optimizers["muon"].param_groups for p in g["params"]}
    blk = tr.model.moe_blocks()[0]
    assert id(blk.gate_up_proj) in muon_ids and id(tr.model.embed_tokens) not in muon_ids
    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(0))
    losses = [tr.train_step(b) for _ in range(3)]
    assert all(math.isfinite(x) for x in losses)
    names = [n for n, _ in state_tensors(opt, blk.gate_up_proj)]
    assert names == ["momentum_buffer"]
    assert [n for n, _ in state_tensors(opt, tr.model.embed_tokens)] == ["exp_avg", "exp_avg_sq"]
    # warmup of 1 step then linear decay; each optimizer keeps its own base rate
    lrs = {name: o.param_groups[0]["lr"] for name, o in opt.optimizers.items()}
    assert lrs["muon"] == pytest.approx(tr.cfg.muon_lr * tr.lr_schedule.multiplier(2))
    assert lrs["adamw"] == pytest.approx(tr.cfg.lr * tr.lr_schedule.multiplier(2))


def _muon_ckpt_worker(rank, world, workdir):
    from placemoe_b200.checkpoint import load_checkpoint, save_checkpoint

    torch.manual_seed(0)
    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(rank))
    tr = _trainer()
    for _ in range(2):
        tr.train_step(b)
    path = save_checkpoint(tr, workdir + "/ckpt")
    ref = tr.train_step(b)
    tr2 = _trainer()
    load_checkpoint(tr2, path)
    got = tr2.train_step(b)
    assert abs(got - ref) < 1e-4, (got, ref)


def test_muon_checkpoint_roundtrip(tmp_path):
    from dist_utils import run_distributed

    run_distributed(_muon_ckpt_worker, 2, str(tmp_path))
