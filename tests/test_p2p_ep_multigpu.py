"""Peer-memory EP transport vs the NCCL all-to-all EP path on 2 GPUs (same routing, same weights).

Runs as 2 child processes, one per GPU, with NVLS disabled; skipped on fewer
than 2 GPUs.
"""

import os

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

        cfg = get_preset("small_qwen3_moe")
        topo = expert_topology(cfg.num_experts, world, 1)
        init = expert_init_from_full(cfg, topo, None, rank, seed=5)
        results = {}
        for name, ep_cls in (("nccl", ExpertParallel), ("p2p", P2PExpertParallel)):
            with torch.device("cuda"):
                blk = MoEBlock(cfg, 0, topo.slots_per_rank)
            torch.manual_seed(1)
            with torch.no_grad():
                blk.gate.normal_(0, 0.02)
                init(0, "gate_up_proj", blk.gate_up_proj)
                init(0, "down_proj", blk.down_proj)
            blk.placement = build_placements(None, topo, rank, [blk.layer_key])[blk.layer_key]
            blk.ep = ep_cls()
            g = torch.Generator(device="cuda").manual_seed(100 + rank)
            x = torch.randn(512, cfg.hidden_size, device="cuda", generator=g).bfloat16().requires_grad_()
            dy = torch.randn(512, cfg.hidden_size, device="cuda", generator=g).bfloat16()
            y = blk(x)
            y.float().mul(dy.float()).sum().backward()
            torch.cuda.synchronize()
            check_device_error()
            results[name] = (y.detach().float(), x.grad.float(), blk.gate.main_grad.clone(),
                             blk.gate_up_proj.main_grad.clone(), blk.down_proj.main_grad.clone())
        errs = []
        for a, b in zip(results["nccl"], results["p2p"]):
            errs.append(((a - b).abs().max() / (a.abs().max() + 1e-6)).item())
        out_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_p2p_transport_matches_nccl_transport():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
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
    assert len(res) == 2
    for r, errs in res.items():
        # y, dx, d(gate), d(gate_up), d(down): same math, different summation order
        assert all(e < 2e-2 for e in errs), (r, errs)
