"""Ulysses sequence parallelism on 2 GPUs: the peer-memory exchange kernels against the gather they
implement, and a training step with the sequence split over the 2 GPUs against whole sequences.

Child processes, one per GPU, NVLS off; skipped with fewer than 2 GPUs.
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
        from placemoe_b200.ops import check_device_error
        from placemoe_b200.parallel.ulysses import UlyssesGroup, heads_to_seq, seq_to_heads
        from placemoe_b200.trainer.base import TrainConfig, Trainer

        grp = UlyssesGroup(None, "cuda", 1 << 20)
        b, s, h, d = 2, 512, 8, 128
        chunk = s // world
        g = torch.Generator(device="cuda").manual_seed(3)
        full = torch.randn(b, s, h, d, device="cuda", generator=g).bfloat16()
        ok = []
        for _ in range(2):  # two exchanges each way: both buffer regions are used
            local = full[:, rank * chunk:(rank + 1) * chunk].reshape(b * chunk, h, d).contiguous()
            heads = seq_to_heads(local, grp, b, chunk)
            hp = h // world
            ok.append(torch.equal(heads, full[:, :, rank * hp:(rank + 1) * hp].reshape(b * s, hp, d)))
            back = heads_to_seq(heads, grp, b, chunk)
            ok.append(torch.equal(back.view(b * chunk, h, d), local))
        torch.cuda.synchronize()
        check_device_error()
        gb = torch.Generator().manual_seed(9)
        batches = [torch.randint(0, 4096, (2, 512), generator=gb) for _ in range(2)]
        losses = {}
        for sp in (1, 2):
            cfg = TrainConfig(model="small_qwen3_moe", seq_len=512, batch_per_rank=2, micro_batch_size=2,
                              lr=1e-3, seed=0, ulysses_size=sp, ep_transport="p2p")
            tr = Trainer(cfg)
            out = []
            for ids in batches:
                loss = torch.tensor([tr.train_step(ids)], device="cuda")
                if sp > 1:
                    dist.all_reduce(loss)
                    loss /= sp
                out.append(float(loss))
            losses[sp] = out
            del tr
        torch.cuda.synchronize()
        check_device_error()
        out_q.put((rank, all(ok), losses[1], losses[2]))
    finally:
        dist.destroy_process_group()


def test_ulysses_exchange_and_training_on_two_gpus():
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
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = []
    while not q.empty():
        res.append(q.get())
    assert len(res) == 2
    for rank, ok, l1, l2 in res:
        assert ok, rank
        for a, b in zip(l1, l2):  # bf16 compute, different summation order
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), (rank, l1, l2)
