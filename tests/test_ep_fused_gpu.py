"""Fused peer-memory dispatch / combine kernels on one GPU (a one-rank EP group) vs the local MoE path.

With one rank every assignment of a token lands on the same GPU, so the
kernels' dedup (one stored row per token, local copies for its other
assignments), position lists, padding rows and pre-reduced combine are all
exercised; the multi-rank offsets are covered by the 2- and 4-GPU tests.
Checked: outputs, input gradients, router gradients and expert weight
gradients against the single-GPU kernels path (same math, different
summation order), over two iterations in a row.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _block(cfg, slots, plan, topo):
    from placemoe_b200.models.moe_decoder import MoEBlock
    from placemoe_b200.parallel.data_parallel import expert_init_from_full
    from placemoe_b200.parallel.placement import build_placements

    with torch.device("cuda"):
        blk = MoEBlock(cfg, 0, slots)
    plans = {blk.layer_key: plan} if plan is not None else None
    init = expert_init_from_full(cfg, topo, plans, 0, seed=5)
    torch.manual_seed(1)
    with torch.no_grad():
        blk.gate.normal_(0, 0.02)
        init(0, "gate_up_proj", blk.gate_up_proj)
        init(0, "down_proj", blk.down_proj)
    blk.placement = build_placements(plans, topo, 0, [blk.layer_key])[blk.layer_key]
    blk.train()
    return blk


@pytest.mark.parametrize("tokens,replica", [(1024, False), (3001, True), (64, False)])
def test_fused_ep_one_rank_matches_local_path(tokens, replica):
    from placemoe_b200.models.config import get_preset
    from placemoe_b200.ops import check_device_error
    from placemoe_b200.parallel.data_parallel import expert_topology
    from placemoe_b200.parallel.p2p_ep import P2PExpertParallel
    from placemoe_b200.placemoe.types import LayerPlan, identity_plan

    cfg = get_preset("small_qwen3_moe")
    e = cfg.num_experts
    topo = expert_topology(e, 1, 1 if replica else 0)
    plan = None
    if replica:  # expert 3 also in the extra slot, and the source uses that copy
        base = identity_plan(topo)
        layout = np.array(base.slot_to_logical)
        layout[e] = 3
        mapping = np.array(base.source_logical_to_physical)
        mapping[0, 3] = e
        plan = LayerPlan(layout, mapping, np.array(base.owner_slots))
    res = {}
    for name in ("local", "fused"):
        blk = _block(cfg, topo.slots_per_rank, plan, topo)
        if name == "fused":
            blk.ep = P2PExpertParallel()
            blk.ep_slab = 0
        g = torch.Generator(device="cuda").manual_seed(7)
        outs = []
        for it in range(2):
            x = torch.randn(tokens, cfg.hidden_size, device="cuda", generator=g).bfloat16().requires_grad_()
            dy = torch.randn(tokens, cfg.hidden_size, device="cuda", generator=g).bfloat16()
            for p in (blk.gate, blk.gate_up_proj, blk.down_proj):
                if getattr(p, "main_grad", None) is not None:
                    p.main_grad.zero_()
            y = blk(x)
            y.float().mul(dy.float()).sum().backward()
            torch.cuda.synchronize()
            check_device_error()
            outs.append([y.detach().float(), x.grad.float(), blk.gate.main_grad.clone(),
                         blk.gate_up_proj.main_grad.clone(), blk.down_proj.main_grad.clone()])
        res[name] = outs
        if name == "fused":
            blk.ep.check_capacity()
    for it in range(2):
        for i, (a, b) in enumerate(zip(res["local"][it], res["fused"][it])):
            err = ((a - b).abs().max() / (a.abs().max() + 1e-6)).item()
            assert err < 2e-2, (it, i, err)
