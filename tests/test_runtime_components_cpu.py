"""Router replay, MoE state validation, online mapping correction, oracle volumes, dispatch checks,
EP plan and op table (CPU)."""

import numpy as np
import pytest
import torch


def _tiny_model():
    from placemoe_b200.models.config import get_preset
    from placemoe_b200.models.moe_decoder import build_model

    return build_model(get_preset("tiny_qwen3_moe"), None, "cpu", 0, None)


def test_router_replay_reuses_routes_and_keeps_router_gradients():
    from placemoe_b200.ops.router_replay import RouterReplay

    torch.manual_seed(0)
    model = _tiny_model()
    rr = RouterReplay()
    for blk in model.moe_blocks():
        blk.router_replay = rr
    ids = torch.randint(0, model.config.vocab_size, (1, 64))
    rr.start_record()
    model(ids, labels=ids)
    routes = {blk.layer_idx: blk.last_route.clone() for blk in model.moe_blocks()}
    assert len(rr) == len(routes)
    with torch.no_grad():  # perturb the router: fresh routing would change
        for blk in model.moe_blocks():
            blk.gate.add_(torch.randn_like(blk.gate))
    rr.start_replay()
    loss, _ = model(ids, labels=ids)
    loss.backward()
    for blk in model.moe_blocks():
        assert torch.equal(blk.last_route.long(), routes[blk.layer_idx].long())
        assert blk.gate.grad is not None and blk.gate.grad.abs().sum() > 0
    rr.stop()


def test_configure_hiermoe_validation():
    from placemoe_b200.arguments.parser import HierMoEConfig
    from placemoe_b200.parallel.hiermoe_state import (HierMoEConfigurationError, checkpoint_state,
                                                      configure_hiermoe, get_hiermoe_state)

    st = configure_hiermoe(HierMoEConfig(communication_mode="hierarchical", redundant_slot_increment_per_device=1),
                           ep_size=8, ranks_per_node=8)
    assert st.mode == "direct" and get_hiermoe_state() is st
    with pytest.raises(HierMoEConfigurationError):
        configure_hiermoe(HierMoEConfig(redundant_slot_increment_per_device=1), ep_size=8, ep_fsdp_size=2)
    with pytest.raises(HierMoEConfigurationError):
        configure_hiermoe(HierMoEConfig(redundant_slot_increment_per_device=1), ep_size=8, fsdp_offload_enabled=True)
    with pytest.raises(HierMoEConfigurationError):
        configure_hiermoe(HierMoEConfig(communication_mode="hierarchical"), ep_size=16, ranks_per_node=8)
    with pytest.raises(HierMoEConfigurationError):
        configure_hiermoe(HierMoEConfig(communication_mode="bogus"), ep_size=8)
    model = _tiny_model()
    assert checkpoint_state(model)["version"] == 3


def test_online_lut_update_lowers_imbalance():
    from placemoe_b200.placemoe.online_lut import _objective, online_lut_update
    from placemoe_b200.placemoe.seeds import mirrored_r2_plan
    from placemoe_b200.placemoe.types import PlaceMoETopology

    topo = PlaceMoETopology(2, 2, 4, 4)
    plan = mirrored_r2_plan(topo)
    demand = np.array([[40.0, 1, 1, 1], [40.0, 1, 1, 1]])  # expert 0 is hot for both sources
    slot_rank = np.arange(8) // 4
    before = _objective(np.asarray(plan.source_logical_to_physical), demand, slot_rank, 2, 0.1)
    new, changes = online_lut_update(plan, topo, demand, max_changes=2)
    after = _objective(np.asarray(new.source_logical_to_physical), demand, slot_rank, 2, 0.1)
    assert after <= before
    assert np.array_equal(new.slot_to_logical, plan.slot_to_logical)


def test_oracle_steps_and_volumes():
    from placemoe_b200.placemoe.oracle import OracleCapture, dispatch_volumes, parse_steps

    assert parse_steps("1-3,7") == {1, 2, 3, 7}
    assert not OracleCapture(_tiny_model(), environ={}).active
    mapping = np.array([[0, 1, 2, 3], [0, 1, 2, 3]])
    slot_rank = np.array([0, 0, 1, 1])
    routes = [np.array([[0, 2], [1, 3]]), np.array([[2, 3]])]
    v = dispatch_volumes(routes, mapping, slot_rank)
    assert v["rows_no_dedup"][1, 1] == 2 and v["rows_dedup"][1, 1] == 1
    assert v["recv_assignments"].sum() == 6


def test_dispatch_check_and_plan():
    from placemoe_b200.models.parallel_plan import check_plan, sharding_of
    from placemoe_b200.ops.registry import table
    from placemoe_b200.parallel.data_parallel import expert_topology
    from placemoe_b200.parallel.placement import build_placements
    from placemoe_b200.parallel.validation import check_dispatch

    model = _tiny_model()
    assert sharding_of("layers.0.mlp.gate_up_proj") == "Shard(0)"
    assert sharding_of("model.layers.3.mlp.down_proj") == "Shard(0)"
    assert sharding_of("layers.0.self_attn.qkv_proj") == "Replicate()"
    assert check_plan(model, model.config.num_experts) == []
    assert check_plan(model, 3)
    topo = expert_topology(model.config.num_experts, 1)
    pl = build_placements(None, topo, 0, ["x"])["x"]
    idx = torch.randint(0, model.config.num_experts, (10, 4))
    assert check_dispatch(idx, pl, torch.tensor([40])) == []
    assert check_dispatch(idx, pl, torch.tensor([39]))
    assert {s.op for s in table()} >= {"linear", "attention", "replica_grad_reduce", "state_migration"}
