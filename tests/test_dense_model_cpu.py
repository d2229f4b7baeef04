"""Dense decoder families (Qwen3 dense / Llama): presets, HF config mapping, training on CPU with
data parallelism (gloo), and the HF export / load round trip."""

import math
import os

import torch

from dist_utils import run_distributed


def test_dense_presets_and_hf_config():
    from placemoe_b200.models.config import from_hf_config, get_preset

    q = get_preset("qwen3_8b")
    assert q.is_dense and q.qk_norm == "per_head" and q.intermediate_size == 12288
    # 8.2B parameters (untied embeddings)
    assert abs(q.num_params() / 1e9 - 8.19) < 0.05
    ll = get_preset("llama3_8b")
    assert ll.qk_norm == "none" and abs(ll.num_params() / 1e9 - 8.03) < 0.05
    cfg = from_hf_config({"model_type": "llama", "vocab_size": 1000, "hidden_size": 64, "num_hidden_layers": 2,
                          "num_attention_heads": 4, "num_key_value_heads": 2, "intermediate_size": 128,
                          "rope_theta": 500000.0})
    assert cfg.is_dense and cfg.head_dim == 16 and cfg.qk_norm == "none"


def test_dense_mlp_reference_matches_formula():
    from placemoe_b200.models.config import get_preset
    from placemoe_b200.models.moe_decoder import DenseMLP

    torch.manual_seed(0)
    m = DenseMLP(get_preset("tiny_qwen3_dense"))
    with torch.no_grad():
        m.w_gate_up.normal_(0, 0.05)
        m.w_down.normal_(0, 0.05)
    x = torch.randn(10, 256)
    i = m.w_gate_up.shape[1] // 2
    g, u = x @ m.w_gate_up[0, :i].t(), x @ m.w_gate_up[0, i:].t()
    ref = (torch.nn.functional.silu(g) * u) @ m.w_down[0].t()
    assert torch.allclose(m(x), ref, atol=1e-5)


def _worker(rank, world, workdir):
    from placemoe_b200.checkpoint import export_hf, load_hf_weights
    from placemoe_b200.trainer.base import TrainConfig, Trainer

    cfg = TrainConfig(model="tiny_qwen3_dense", seq_len=64, batch_per_rank=2, micro_batch_size=1, lr=1e-3,
                      device="cpu", seed=0)
    tr = Trainer(cfg)
    assert tr.model.moe_blocks() == [] and tr.pstate.ep is None
    b = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(rank))
    losses = [tr.train_step(b) for _ in range(3)]
    assert all(math.isfinite(x) for x in losses) and losses[-1] < losses[0]
    # replicas stay identical under data parallelism
    w = tr.model.layers[0].mlp.w_down.detach().clone()
    ws = [torch.empty_like(w) for _ in range(world)]
    torch.distributed.all_gather(ws, w)
    assert all(torch.equal(ws[0], x) for x in ws)
    out = export_hf(tr, os.path.join(workdir, "hf"))
    torch.distributed.barrier()
    tr2 = Trainer(cfg)
    load_hf_weights(tr2, os.path.join(workdir, "hf"))
    for (n, a), (_, c) in zip(tr.model.named_parameters(), tr2.model.named_parameters()):
        assert torch.equal(a.bfloat16().float(), c), n
    if rank == 0:
        import json

        hf = json.load(open(os.path.join(out, "config.json")))
        assert hf["architectures"] == ["Qwen3ForCausalLM"] and hf["intermediate_size"] == 512


def test_dense_training_dp2_and_hf_roundtrip(tmp_path):
    run_distributed(_worker, 2, str(tmp_path))


def test_gradient_checkpointing_matches_plain_backward():
    """Recomputing every decoder layer in the backward (the layers carry the residual and the pending
    branch output between them) gives the loss and gradients of the plain backward."""
    from placemoe_b200.models.config import get_preset
    from placemoe_b200.models.moe_decoder import build_model

    cfg = get_preset("small_qwen3_moe")
    ids = torch.randint(0, cfg.vocab_size, (2, 64), generator=torch.Generator().manual_seed(0))
    out = []
    for ckpt in (False, True):
        m = build_model(cfg, device="cpu", seed=5)
        m.train()
        m.gradient_checkpointing = ckpt
        loss, aux = m(ids, labels=ids)
        (loss + aux).backward()
        out.append((loss.item(), {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}))
    (l0, g0), (l1, g1) = out
    assert abs(l0 - l1) < 1e-6 and g0.keys() == g1.keys() and len(g0) > 0
    for n in g0:
        assert torch.allclose(g0[n], g1[n], rtol=1e-5, atol=1e-6), n
