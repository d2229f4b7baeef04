"""Spawn helper for multi-rank CPU tests (gloo, 127.0.0.1 rendezvous)."""

import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, errq):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import torch

    # ranks share the machine's cores: no oversubscription
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))
    try:
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        fn(rank, world, *args)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def run_distributed(fn, world: int, *args):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    import time

    deadline = time.monotonic() + 900
    for p in procs:
        p.join(max(1.0, deadline - time.monotonic()))
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errors.append((-1, "worker timed out"))
    if errors or any(p.exitcode != 0 for p in procs):
        raise AssertionError("distributed worker failed:\n" + "\n".join(f"rank {r}: {e}" for r, e in errors))
