"""Ulysses sequence parallelism on CPU (gloo, 2 ranks): the exchanges against an explicit gather, and
training with the sequence split over 2 ranks against training on whole sequences."""

import torch

from dist_utils import run_distributed


def _exchange_worker(rank, world):
    from placemoe_b200.parallel.ulysses import UlyssesGroup, heads_to_seq, seq_to_heads

    grp = UlyssesGroup(None, "cpu", 0)
    b, s, h, d = 2, 8, 4, 3
    chunk = s // world
    full = torch.arange(b * s * h * d, dtype=torch.float32).view(b, s, h, d)  # same on every rank
    local = full[:, rank * chunk:(rank + 1) * chunk].reshape(b * chunk, h, d).requires_grad_()
    heads = seq_to_heads(local, grp, b, chunk)  # [b*s, h/P, d]
    hp = h // world
    expect = full[:, :, rank * hp:(rank + 1) * hp].reshape(b * s, hp, d)
    assert torch.equal(heads, expect)
    back = heads_to_seq(heads, grp, b, chunk)
    assert torch.equal(back.view(b * chunk, h, d), local.detach())
    # gradients flow back through both exchanges unchanged
    (back * 2.0).sum().backward()
    assert torch.equal(local.grad, torch.full_like(local, 2.0))


def test_ulysses_exchanges_match_gather():
    run_distributed(_exchange_worker, 2)


def _train_worker(rank, world):
    import torch.distributed as dist

    from placemoe_b200.trainer.base import TrainConfig, Trainer

    g = torch.Generator().manual_seed(5)
    batches = [torch.randint(0, 1024, (2, 64), generator=g) for _ in range(3)]  # same on both ranks
    losses = {}
    for sp in (1, 2):
        cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=2, micro_batch_size=2, lr=1e-3,
                          device="cpu", seed=0, ulysses_size=sp, max_grad_norm=0.0)
        tr = Trainer(cfg)
        out = []
        for ids in batches:
            loss = torch.tensor(tr.train_step(ids))
            if sp > 1:  # every rank holds a chunk loss; the batch loss is their mean
                dist.all_reduce(loss)
                loss = loss / sp
            out.append(float(loss))
        losses[sp] = out
    for a, b in zip(losses[1], losses[2]):
        assert abs(a - b) < 1e-4 * max(1.0, abs(a)), (losses[1], losses[2])


def test_ulysses_training_matches_whole_sequences():
    run_distributed(_train_worker, 2)


def _train_packed_worker(rank, world):
    import torch.distributed as dist

    from placemoe_b200.trainer.base import TrainConfig, Trainer

    g = torch.Generator().manual_seed(6)
    batches = [torch.randint(0, 1024, (2, 64), generator=g) for _ in range(3)]  # same on both ranks
    # documents cross the chunk boundary (token 32 of each row), one is a single token
    cu = torch.tensor([0, 10, 40, 41, 64, 64 + 30, 64 + 33, 128], dtype=torch.int32)
    losses = {}
    for sp in (1, 2):
        cfg = TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=2, micro_batch_size=2, lr=1e-3,
                          device="cpu", seed=0, ulysses_size=sp, max_grad_norm=0.0)
        tr = Trainer(cfg)
        out = []
        for ids in batches:
            loss = torch.tensor(tr.train_step(ids, cu_seqlens=cu))
            if sp > 1:
                dist.all_reduce(loss)
                loss = loss / sp
            out.append(float(loss))
        losses[sp] = out
    for a, b in zip(losses[1], losses[2]):
        assert abs(a - b) < 1e-4 * max(1.0, abs(a)), (losses[1], losses[2])


def test_ulysses_training_with_packed_documents_matches_whole_sequences():
    run_distributed(_train_packed_worker, 2)
