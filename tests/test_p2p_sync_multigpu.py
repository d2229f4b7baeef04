"""Peer-memory replica-gradient reduction and migration transfers vs their NCCL counterparts (2 and 4 GPUs).

Runs as child processes, one per GPU, with NVLS disabled; each case is skipped when the
machine has fewer GPUs than it needs.  The 4-rank trainer case uses a placement in which
only ranks 0 and 1 hold replicated experts: ranks 2 and 3 still take part in every
replica-gradient barrier.
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
        import numpy as np

        from placemoe_b200.models.config import get_preset
        from placemoe_b200.models.moe_decoder import MoEBlock
        from placemoe_b200.ops import check_device_error
        from placemoe_b200.parallel.data_parallel import expert_topology, sync_replica_gradients
        from placemoe_b200.parallel.p2p_sync import PeerExchange, ReplicaGradSync, p2p_transfer, sync_layer
        from placemoe_b200.parallel.placement import build_placements
        from placemoe_b200.placemoe.seeds import mirrored_r2_plan

        cfg = get_preset("small_qwen3_moe")
        topo = expert_topology(cfg.num_experts, world, cfg.num_experts // world)  # two copies of every expert
        plan = mirrored_r2_plan(topo)
        with torch.device("cuda"):
            blk = MoEBlock(cfg, 0, topo.slots_per_rank)
        blk.placement = build_placements({blk.layer_key: plan}, topo, rank, [blk.layer_key])[blk.layer_key]
        g = torch.Generator(device="cuda").manual_seed(10 + rank)
        grads = {}
        for p in (blk.gate_up_proj, blk.down_proj):
            p.main_grad = torch.randn(p.shape, device="cuda", generator=g)
            grads[p] = p.main_grad.clone()

        class _M:
            def moe_blocks(self):
                return [blk]

        sync_replica_gradients(_M(), {blk.layer_key: blk.placement})
        ref = {p: p.main_grad.clone() for p in grads}
        for p in grads:
            p.main_grad.copy_(grads[p])
        x = PeerExchange(None, "cuda", max(p.numel() * 4 for p in grads))
        rs = ReplicaGradSync(x)
        sync_layer(blk, rs._plan(blk), x)
        torch.cuda.synchronize()
        check_device_error()
        err_sync = max((p.main_grad - ref[p]).abs().max().item() for p in grads)

        # migration transfers: every slot state moves to the other rank's slot of the same index
        spr = topo.slots_per_rank
        transfers = [(s, (s + spr) % (2 * spr)) for s in range(2 * spr)]
        n = 4096
        outgoing, staging, expect = {}, {}, {}
        for i, (s, d) in enumerate(transfers):
            payload = torch.full((n,), float(s * 1000 + 7), device="cuda")
            if s // spr == rank:
                outgoing[i] = payload
            if d // spr == rank:
                staging[d] = torch.zeros(n, device="cuda")
                expect[d] = payload
        p2p_transfer(x, transfers, spr, rank, outgoing, staging)
        torch.cuda.synchronize()
        check_device_error()
        err_mig = max((staging[d] - expect[d]).abs().max().item() for d in staging)
        out_q.put((rank, err_sync, err_mig, int(np.asarray(plan.slot_to_logical).size)))
    finally:
        dist.destroy_process_group()


def test_p2p_replica_sync_and_migration_match_nccl():
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
        r, e1, e2, _ = q.get()
        res[r] = (e1, e2)
    assert len(res) == 2
    for r, (e1, e2) in res.items():
        assert e1 < 1e-5, (r, e1)
        assert e2 == 0.0, (r, e2)


def partial_replica_artifact(path, cfg, world):
    """Artifact for every layer: fixed EP plus one replica on rank 1 (of rank 0's first expert) and one on
    rank 0 (of rank 1's first expert); the extra slots of the other ranks stay empty."""
    import numpy as np

    from placemoe_b200.parallel.data_parallel import expert_topology
    from placemoe_b200.placemoe.artifacts import build_placemoe_artifact, write_artifact
    from placemoe_b200.placemoe.types import LayerPlan, identity_plan

    topo = expert_topology(cfg.num_experts, world, 1)
    base = identity_plan(topo)
    spr = topo.slots_per_rank
    per = -(-cfg.num_experts // world)
    layout = np.array(base.slot_to_logical)
    mapping = np.array(base.source_logical_to_physical)
    layout[2 * spr - 1] = 0  # rank 1's extra slot: expert 0 (owned by rank 0)
    layout[spr - 1] = per  # rank 0's extra slot: expert `per` (owned by rank 1)
    mapping[1, 0] = 2 * spr - 1
    mapping[0, per] = spr - 1
    plan = LayerPlan(layout, mapping, np.array(base.owner_slots))
    plans = {f"model.layers.{i}.mlp.experts": plan for i in range(cfg.num_hidden_layers)}
    write_artifact(build_placemoe_artifact(plans, topo), path)


def _trainer_worker(rank, world, port, out_q, artifact=""):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from placemoe_b200.trainer.base import TrainConfig, Trainer

        losses, diffs = {}, []
        for mode in ("off", "auto"):  # replicated dense AdamW, then sharded dense (peer-memory RS / AG)
            cfg = TrainConfig(model="small_qwen3_moe", seq_len=256, batch_per_rank=2, micro_batch_size=1, lr=1e-3,
                              redundant_slots_per_rank=1, ep_transport="p2p", seed=0, dense_sharding=mode,
                              placemoe_artifact=artifact)
            tr = Trainer(cfg)
            if artifact:  # replicas on ranks 0 and 1 only: every rank still runs the layer's sync
                assert tr.replica_sync is not None
            assert (tr.dense_shards is not None) == (mode == "auto")
            g = torch.Generator().manual_seed(100 + rank)  # different data per rank
            losses[mode] = [tr.train_step(torch.randint(0, tr.model_cfg.vocab_size, (2, 256), generator=g))
                            for _ in range(3)]
            if artifact:  # copies of one expert on ranks 0 and 1 must have stayed identical
                w = tr.model.moe_blocks()[0].gate_up_proj.data.contiguous()
                ws = [torch.empty_like(w) for _ in range(world)]
                dist.all_gather(ws, w)
                spr = w.shape[0]
                diffs.append((ws[0][spr - 1] - ws[1][0]).abs().max().item())
                diffs.append((ws[1][spr - 1] - ws[0][0]).abs().max().item())
            sync = getattr(tr.optimizer, "sync_params", None)
            if sync is not None:
                sync()
            torch.cuda.synchronize()
            # dense parameters must stay identical replicas across ranks
            for name, p in tr.model.named_parameters():
                if name.endswith(("gate_up_proj", "down_proj")):
                    continue
                ps = [torch.empty_like(p.data) for _ in range(world)]
                dist.all_gather(ps, p.data.contiguous())
                diffs.append(max((ps[0] - q).abs().max().item() for q in ps[1:]))
            del tr
        loss_gap = max(abs(a - b) / abs(a) for a, b in zip(losses["off"], losses["auto"]))
        out_q.put((rank, max(diffs), loss_gap))
    finally:
        dist.destroy_process_group()


def _run_trainer_case(world, artifact=""):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_trainer_worker, args=(r, world, port, q, artifact)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = {}
    while not q.empty():
        r, d, gap = q.get()
        res[r] = (d, gap)
    assert len(res) == world, res
    for d, gap in res.values():
        assert d == 0.0 and gap < 1e-3, res


def test_dense_replicas_stay_identical_with_peer_memory_ep():
    """Different data per rank, peer-memory EP, replicated and sharded dense optimizer: dense weights must be
    the same on every rank after steps, and both modes must train alike."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run_trainer_case(2)


def test_four_ranks_uneven_replica_membership(tmp_path):
    """4 ranks, replicas held by ranks 0 and 1 only, dense sharding on and off: training completes (no
    barrier waits out), dense replicas stay identical and both dense modes agree."""
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    from placemoe_b200.models.config import get_preset

    path = str(tmp_path / "partial_replicas.json")
    partial_replica_artifact(path, get_preset("small_qwen3_moe"), 4)
    _run_trainer_case(4, path)
