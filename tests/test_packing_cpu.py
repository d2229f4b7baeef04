"""Packed sequences on CPU: the collator, document bounds, and the model on a packed row equal to the
model on each document alone (positions restart, attention and loss stay inside documents)."""

import pytest
import torch


def test_pack_documents_and_bounds():
    from placemoe_b200.data import PackedSyntheticTokens, pack_documents
    from placemoe_b200.ops.attention import doc_bounds

    docs = [torch.arange(5), torch.arange(100, 112), torch.arange(200, 203)]
    ids, cu = pack_documents(docs, rows=2, seq_len=8)
    # doc 1 is split at the row boundary; the last document is truncated
    assert cu.tolist() == [0, 5, 8, 16]
    assert ids[1].tolist() == list(range(103, 111))
    lo, hi = doc_bounds(cu, 16, 8)
    assert lo.tolist() == [0] * 5 + [5] * 3 + [0] * 8 and hi.tolist() == [5] * 5 + [8] * 3 + [8] * 8
    with pytest.raises(ValueError):
        doc_bounds(torch.tensor([0, 10, 16]), 16, 8)  # crosses a row
    with pytest.raises(ValueError):
        pack_documents([torch.arange(3)], rows=1, seq_len=8)  # too few tokens
    it = PackedSyntheticTokens(1024, rows=3, seq_len=256, min_len=16, max_len=300, seed=1)
    ids, cu = next(it)
    assert ids.shape == (3, 256) and cu[0] == 0 and cu[-1] == 768 and (cu.diff() > 0).all()


def test_packed_model_equals_separate_documents():
    from placemoe_b200.models.config import get_preset
    from placemoe_b200.models.moe_decoder import build_model

    torch.manual_seed(0)
    cfg = get_preset("tiny_qwen3_moe", router_aux_loss_coef=0.0)
    model = build_model(cfg, device="cpu", seed=3).eval()
    lens = [7, 20, 5]
    docs = [torch.randint(0, cfg.vocab_size, (n,)) for n in lens]
    ids = torch.cat(docs)[None]
    cu = torch.tensor([0, 7, 27, 32], dtype=torch.int32)
    with torch.no_grad():
        packed = model(ids, cu_seqlens=cu)[0]
        off = 0
        for d in docs:
            alone = model(d[None])[0]
            assert torch.allclose(packed[off: off + d.numel()], alone, atol=1e-4), off
            off += d.numel()
        # the loss ignores the transitions between documents
        loss_packed, _ = model(ids, labels=ids, cu_seqlens=cu)
        tot, cnt = 0.0, 0
        for d in docs:
            l, _ = model(d[None], labels=d[None])
            tot += l.item() * (d.numel() - 1)
            cnt += d.numel() - 1
    assert abs(loss_packed.item() - tot / cnt) < 1e-4


def test_trainer_steps_on_packed_rows():
    from placemoe_b200.data import PackedSyntheticTokens
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    tr = Trainer(TrainConfig(model="tiny_qwen3_moe", seq_len=64, batch_per_rank=4, micro_batch_size=2, lr=1e-3,
                             device="cpu", seed=0))
    data = PackedSyntheticTokens(1024, rows=4, seq_len=64, min_len=8, max_len=40, seed=0)
    ids, cu = next(data)
    losses = [tr.train_step(ids, cu_seqlens=cu) for _ in range(3)]
    assert losses[-1] < losses[0]
