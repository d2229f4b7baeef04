"""Fused peer-memory EP kernels vs the NCCL all-to-all EP path on 2 and 4 GPUs (same routing, same weights).

Runs as child processes, one per GPU, with NVLS disabled; each case is
skipped when the machine has fewer GPUs.  The placement has one extra slot per
GPU holding EPLB-style replicas of the hottest experts (router bias skewed),
so sources use different copies of one expert.
"""

import os

import numpy as np
import pytest
import torch

from dist_utils import free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, port, out_q):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from placemoe_b200.models.config import get_preset
        from placemoe_b200.models.moe_decoder import MoEBlock
        from placemoe_b200.ops import check_device_error
        from placemoe_b200.parallel.data_parallel import expert_init_from_full, expert_topology
        from placemoe_b200.parallel.ep import ExpertParallel
        from placemoe_b200.parallel.p2p_ep import P2PExpertParallel
        from placemoe_b200.parallel.placement import build_placements
        from placemoe_b200.placemoe.seeds import eplb_plan

        cfg = get_preset("small_qwen3_moe", router_bias_zipf_s=1.0, router_bias_scale=1.0)
        topo = expert_topology(cfg.num_experts, world, 1)
        demand = np.exp(MoEBlock(cfg, 0, topo.slots_per_rank).router_bias.numpy())
        plan = eplb_plan(topo, demand)
        plans = {"model.layers.0.mlp.experts": plan}
        init = expert_init_from_full(cfg, topo, plans, rank, seed=5)
        results = {}
        for name, ep_cls in (("nccl", ExpertParallel), ("p2p", P2PExpertParallel)):
            with torch.device("cuda"):
                blk = MoEBlock(cfg, 0, topo.slots_per_rank)
            torch.manual_seed(1)
            with torch.no_grad():
                blk.gate.normal_(0, 0.02)
                init(0, "gate_up_proj", blk.gate_up_proj)
                init(0, "down_proj", blk.down_proj)
            blk.placement = build_placements(plans, topo, rank, [blk.layer_key])[blk.layer_key]
            blk.ep = ep_cls()
            g = torch.Generator(device="cuda").manual_seed(100 + rank)
            x = torch.randn(512, cfg.hidden_size, device="cuda", generator=g).bfloat16().requires_grad_()
            dy = torch.randn(512, cfg.hidden_size, device="cuda", generator=g).bfloat16()
            outs = []
            for it in range(2):  # two iterations: the arena, epochs and parity are reused
                x.grad = None
                for p in (blk.gate, blk.gate_up_proj, blk.down_proj):
                    if getattr(p, "main_grad", None) is not None:
                        p.main_grad.zero_()
                y = blk(x)
                y.float().mul(dy.float()).sum().backward()
                torch.cuda.synchronize()
                check_device_error()
                outs.append((y.detach().float(), x.grad.float(), blk.gate.main_grad.clone(),
                             blk.gate_up_proj.main_grad.clone(), blk.down_proj.main_grad.clone()))
            if name == "p2p":
                blk.ep.check_capacity()
            results[name] = outs[0] + outs[1]
        errs = []
        for a, b in zip(results["nccl"], results["p2p"]):
            errs.append(((a - b).abs().max() / (a.abs().max() + 1e-6)).item())
        out_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_p2p_transport_matches_nccl_transport(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = {}
    while not q.empty():
        r, errs = q.get()
        res[r] = errs
    assert len(res) == world
    for r, errs in res.items():
        # y, dx, d(gate), d(gate_up), d(down) of two iterations: same math, different summation order
        assert all(e < 2e-2 for e in errs), (r, errs)
