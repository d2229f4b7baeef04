"""NVLink / NCCL calibration probe: fits the planner's cost model on this machine.

    torchrun --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 -m placemoe_b200.bench.link_probe \
        --out calibration.json

Probes, every rank at once (median over repeats of the max over ranks, CUDA
events on the launching stream):
  * peer copy: each rank pulls ``n`` bytes from the next rank's symmetric buffer
    with the ``p2p_pull`` kernel (the transport of dispatch / combine / migration);
  * NCCL ``all_to_all_single`` of ``n`` bytes per rank (the baseline transport);
  * expert compute: the grouped SwiGLU fc1 + fc2 forward at two token counts
    (ms per routed assignment).
Writes the reference's calibration JSON (``status: accepted`` + coefficients)
plus the raw fits; pass it as ``calibration.artifact`` in the PlaceMoE config.

Reference parity: startup perf-model fitting of
veomni/distributed/moe/hiermoe/perf_model.py:91-229.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist


def _timed(fn, repeats: int) -> list[float]:
    out = []
    for _ in range(repeats):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return out


def _gather(samples: list[float]) -> list[list[float]]:
    t = torch.tensor(samples, device="cuda", dtype=torch.float64)
    allt = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(allt, t)
    return [x.tolist() for x in allt]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="1,4,16,64,256")
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--out", default="")
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=1024)
    ap.add_argument("--experts", type=int, default=8)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from ..ops import check_device_error, kernels
    from ..parallel.p2p_sync import FLAGS_BYTES, PeerExchange
    from ..placemoe.perf_model import LinkFit, PerfModel, fit_linear, robust_time

    sizes = [int(float(x) * (1 << 20)) for x in args.sizes_mb.split(",")]
    x = PeerExchange(None, "cuda", max(sizes))
    kn = kernels()
    peer_t, nccl_t = [], []
    for n in sizes:
        dst = torch.empty(n, dtype=torch.uint8, device="cuda")
        src_rank = (rank + 1) % world
        peer_t.append(robust_time(_gather(_timed(lambda: kn.p2p_pull(dst, x.peers, src_rank, FLAGS_BYTES),
                                                 args.repeats))))
        a = torch.empty(n, dtype=torch.uint8, device="cuda")
        b = torch.empty_like(a)
        nccl_t.append(robust_time(_gather(_timed(lambda: dist.all_to_all_single(b, a), args.repeats))))
    links = {"nvlink": fit_linear(sizes, peer_t), "nccl_a2a": fit_linear(sizes, nccl_t)}
    # expert compute: grouped fc1 (SwiGLU) + fc2 forward at two sizes -> ms per assignment
    from ..ops.moe import ALIGN

    comp_sizes, comp_t = [], []
    E, H, I = args.experts, args.hidden, args.inter
    w1 = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).bfloat16()
    w2 = (torch.randn(E, H, I, device="cuda") * 0.02).bfloat16()
    for rows_per_expert in (512, 2048):
        rows = rows_per_expert * E
        offs = torch.arange(0, rows + 1, rows_per_expert, device="cuda", dtype=torch.int32)
        xd = torch.randn(rows, H, device="cuda").bfloat16()
        sc = torch.ones(rows, device="cuda")
        h = torch.empty(rows, I, device="cuda", dtype=torch.bfloat16)
        gu = torch.empty(rows, 2 * I, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)

        def ffn():
            kn.moe_fc1_swiglu(xd, w1, offs, sc, h, gu, ALIGN, None)
            kn.moe_grouped_gemm(h, w2, offs, y, False, ALIGN)

        comp_sizes.append(rows)
        comp_t.append(robust_time(_gather(_timed(ffn, args.repeats))))
    model = PerfModel(links=links, compute=fit_linear(comp_sizes, comp_t), ranks_per_node=world, ep_size=world)
    torch.cuda.synchronize()
    check_device_error()
    if rank == 0:
        payload = model.calibration_payload(scope={"ep_size": world, "device": torch.cuda.get_device_name(),
                                                   "hidden": H, "inter": I})
        payload["probe"] = {"sizes_bytes": sizes, "peer_copy_ms": peer_t, "nccl_a2a_ms": nccl_t,
                            "compute_rows": comp_sizes, "compute_ms": comp_t,
                            "peer_copy_gbs": links["nvlink"].bandwidth_gbs,
                            "nccl_a2a_gbs": links["nccl_a2a"].bandwidth_gbs}
        print(json.dumps(payload["probe"] | {"coefficients": payload["coefficients"]}), flush=True)
        if args.out:
            with open(args.out, "w") as f:
                json.dump(payload, f, indent=2)
    dist.barrier()
    dist.destroy_process_group()
    return LinkFit


if __name__ == "__main__":
    main()
