"""Standalone MoE layer fwd+bwd microbenchmark under expert parallelism (EP = world size).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m placemoe_b200.bench.moe_layer \
        --tokens 16384 --hidden 4096 --experts 64 --topk 8 --inter 1536 --extra-slots 1 --skew 1.0 \
        --transport p2p

Per rank: ``--tokens`` hidden states N(0,1); router weights N(0, 1/H) so the
logits are ~N(0,1); a per-expert bias of ``log Zipf(s)`` weights over a seeded
expert permutation; expert weights N(0, 0.02).  With ``--extra-slots`` each GPU
holds replica slots placed by the EPLB-style seed on the expected demand.

Transports:
  p2p      peer-memory dedup dispatch / pre-reduced combine (the product path);
  nccl     the same dedup algorithm over NCCL all-to-all with host-exchanged splits;
  baseline one row per assignment over NCCL all-to-all + ``torch._grouped_mm``
           (cuBLAS) expert GEMMs, the comparison point.

Timing: ``--warmup`` iterations, then ``--iters`` iterations each bracketed by
CUDA events on the launching stream (forward and backward separately), a
barrier + synchronize around the timed block, max over ranks.  Inputs and
weights exceed the 126 MB L2 (16384 x 4096 bf16 = 128 MiB of hidden states per
rank plus 1.2 GB of expert weights), so no explicit flush is done.

Roofline per rank (reported as the max over ranks):
  compute  = 18 * A_r * H * I flops (fc1 2I-wide + fc2; fwd, dgrad, wgrad) over the
             measured bf16 GEMM peak;
  NVLink   = bytes leaving this GPU (dispatch + combine rows, both passes) over the
             link bandwidth measured at start-up: a peer pull of 256 MiB from the next
             rank (``p2p_pull``, CUDA events, best of 5, min over ranks); 770 GB/s per
             direction when the probe is skipped;
  target   = max(compute, NVLink); frac = target / measured.
Per fused communication kernel (peer-memory transport) the bench also reports its
time (max over ranks), the NVLink bytes it moves and the achieved GB/s against the
measured link: dispatch moves the deduplicated rows out, combine the pre-reduced
partials back, scatter the output gradients out, combine_bwd the data gradients back.
"""

from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

LINK_GBS = 770.0  # per direction, the pool's measured peer copy; used when the probe is skipped


def measure_link_gbs(world: int, rank: int, nbytes: int = 256 << 20) -> float:
    """Peer pull bandwidth from rank+1 into this GPU (GB/s, best of 5; min over ranks)."""
    from ..ops import kernels
    from ..parallel.p2p_sync import FLAGS_BYTES, PeerExchange

    x = PeerExchange(None, "cuda", nbytes)
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    src = (rank + 1) % world
    best = float("inf")
    for i in range(6):
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        kernels().p2p_pull(dst, x.peers, src, FLAGS_BYTES)
        e.record()
        torch.cuda.synchronize()
        if i:
            best = min(best, s.elapsed_time(e))
    gbs = torch.tensor([nbytes / (best * 1e-3) / 1e9], device="cuda")
    dist.all_reduce(gbs, op=dist.ReduceOp.MIN)
    del x
    return float(gbs.item())


def _peaks():
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    p = os.path.join(root, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def _expected_demand(bias: np.ndarray, k: int, n: int = 200000, seed: int = 0) -> np.ndarray:
    """Monte-Carlo expected top-k counts per expert for N(0,1) logits + bias."""
    g = np.random.default_rng(seed)
    z = g.standard_normal((n, bias.shape[0])) + bias[None, :]
    top = np.argpartition(-z, k - 1, axis=1)[:, :k]
    return np.bincount(top.reshape(-1), minlength=bias.shape[0]).astype(np.float64) / n


class _BaselineMoE:
    """NCCL all-to-all (no dedup) + torch grouped GEMM experts."""

    def __init__(self, group, world, rank):
        self.group, self.world, self.rank = group, world, rank
        self.w1 = self.w2 = None

    def moe_forward(self, blk, x, bias, aux_coef):
        from ..parallel.ep import ExpertParallel, all_to_all

        t, h = x.shape
        k = blk.cfg.num_experts_per_tok
        w, idx, aux = ExpertParallel._route(self, blk, x, bias, aux_coef)
        dest_tab, slot_tab = blk.placement.route_tables(x.device)
        dest = dest_tab.long()[idx].reshape(-1)
        slot = slot_tab.long()[idx].reshape(-1)
        spr = blk.num_local_slots
        order = torch.argsort(dest * spr + slot, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world)
        meta = torch.stack([slot[order], torch.zeros_like(order)], 1)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        tok = torch.arange(t, device=x.device).repeat_interleave(k)[order]
        xs = x.index_select(0, tok)
        rx = all_to_all(xs, sc, rc, self.group)
        rslot = all_to_all(meta, sc, rc, self.group)[:, 0]
        o2 = torch.argsort(rslot, stable=True)
        per = torch.bincount(rslot, minlength=spr)
        offs = torch.cumsum(per, 0).to(torch.int32)
        if self.w1 is None:  # bf16 leaf weights (the baseline keeps no fp32 masters)
            self.w1 = blk.gate_up_proj.detach().to(torch.bfloat16).requires_grad_()
            self.w2 = blk.down_proj.detach().to(torch.bfloat16).requires_grad_()
        xin = rx[o2]
        gu = torch._grouped_mm(xin, self.w1.transpose(1, 2), offs=offs)
        inter = gu.shape[1] // 2
        hmid = F.silu(gu[:, :inter]) * gu[:, inter:]
        yo = torch._grouped_mm(hmid, self.w2.transpose(1, 2), offs=offs)
        y_recv = torch.empty_like(yo).index_copy(0, o2, yo)
        back = all_to_all(y_recv, rc, sc, self.group)
        ws = w.reshape(-1)[order].to(back.dtype)
        y = torch.zeros(t, h, device=x.device, dtype=torch.float32).index_add(0, tok, (back * ws[:, None]).float())
        return y.to(x.dtype), aux, idx


def run(args):
    from ..models.config import get_preset
    from ..models.moe_decoder import MoEBlock
    from ..ops import check_device_error
    from ..parallel import p2p_ep
    from ..parallel.data_parallel import expert_init_from_full, expert_topology
    from ..parallel.ep import ExpertParallel
    from ..parallel.placement import build_placements
    from ..placemoe.seeds import eplb_plan, fixed_ep_plan

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    if world > 1 and not args.no_link_probe and not args.link_gbs:
        args.link_gbs = measure_link_gbs(world, rank)
    cfg = get_preset("olmoe_1b_7b", hidden_size=args.hidden, moe_intermediate_size=args.inter,
                     num_experts=args.experts, num_experts_per_tok=args.topk, router_bias_zipf_s=args.skew,
                     router_bias_scale=1.0, router_aux_loss_coef=0.0, norm_topk_prob=False)
    topo = expert_topology(cfg.num_experts, world, args.extra_slots if world > 1 else 0)
    with torch.device("cuda"):
        blk = MoEBlock(cfg, 0, topo.slots_per_rank)
    bias = blk.router_bias.cpu().numpy()
    if args.extra_slots and world > 1:
        plan = eplb_plan(topo, _expected_demand(bias, cfg.num_experts_per_tok))
    else:
        plan = fixed_ep_plan(topo) if world > 1 else None
    plans = {blk.layer_key: plan} if plan is not None else None
    blk.placement = build_placements(plans, topo, rank, [blk.layer_key])[blk.layer_key]
    init = expert_init_from_full(cfg, topo, plans, rank, seed=3)
    torch.manual_seed(11)
    with torch.no_grad():
        blk.gate.normal_(0, args.hidden ** -0.5)
        init(0, "gate_up_proj", blk.gate_up_proj)
        init(0, "down_proj", blk.down_proj)
    if world > 1:
        blk.ep = {"p2p": lambda: p2p_ep.P2PExpertParallel(),
                  "nccl": lambda: ExpertParallel(),
                  "baseline": lambda: _BaselineMoE(None, world, rank)}[args.transport]()
    elif args.transport == "baseline":
        blk.ep = _BaselineMoE(None, 1, 0)
    blk.train()
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    x = torch.randn(args.tokens, args.hidden, device="cuda", generator=g).bfloat16().requires_grad_()
    dy = torch.randn(args.tokens, args.hidden, device="cuda", generator=g).bfloat16()

    def it():
        x.grad = None
        y = blk(x)
        return y

    for _ in range(args.warmup):
        it().backward(dy)
    torch.cuda.synchronize()
    dist.barrier()
    use_timer = args.transport == "p2p" and world > 1
    fwd_ms, bwd_ms, phases = [], [], {}
    for _ in range(args.iters):
        if use_timer:
            p2p_ep.TIMER = p2p_ep.PhaseTimer()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        y = it()
        e1.record()
        y.backward(dy)
        e2.record()
        torch.cuda.synchronize()
        fwd_ms.append(e0.elapsed_time(e1))
        bwd_ms.append(e1.elapsed_time(e2))
        if use_timer:
            for kk, v in p2p_ep.TIMER.phases().items():
                phases[kk] = phases.get(kk, 0.0) + v / args.iters
            p2p_ep.TIMER = None
    dist.barrier()
    check_device_error()
    # per-rank routing volume of the last iteration (same routing every iteration)
    with torch.no_grad():
        idx = blk.last_route
        dest_tab, slot_tab = blk.placement.route_tables(x.device)
        dest = dest_tab.long()[idx]
        asg_to = torch.bincount(dest.reshape(-1), minlength=world)
        rows_to = F.one_hot(dest, world).amax(1).sum(0)
        stats = torch.stack([asg_to, rows_to]).to(torch.float64)  # [2, W] from this rank
        all_stats = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(all_stats, stats)
        S = torch.stack(all_stats)  # [src, 2, dst]
    A_recv = S[:, 0, :].sum(0)  # assignments received per rank
    remote_rows_out = torch.tensor([S[r, 1].sum() - S[r, 1, r] for r in range(world)])
    remote_rows_in = torch.tensor([S[:, 1, r].sum() - S[r, 1, r] for r in range(world)])
    remote_asg_out = torch.tensor([S[r, 0].sum() - S[r, 0, r] for r in range(world)])
    dedup = args.transport != "baseline"
    rows_out = remote_rows_out if dedup else remote_asg_out
    rows_in = remote_rows_in if dedup else torch.tensor([S[:, 0, r].sum() - S[r, 0, r] for r in range(world)])
    peak_tf, src = _peaks()
    h, i = args.hidden, args.inter
    gemm_ms = 18.0 * A_recv.max().item() * h * i / (peak_tf * 1e12) * 1e3
    # bytes leaving a GPU: dispatch rows out + combine partials back, in forward and backward
    link_bytes = 2 * (rows_out + rows_in).max().item() * h * 2
    link_gbs = args.link_gbs or LINK_GBS
    link_ms = link_bytes / (link_gbs * 1e9) * 1e3
    t = torch.tensor([float(np.median(fwd_ms)), float(np.median(bwd_ms))], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ph = torch.tensor([phases.get(kk, 0.0) for kk in sorted(phases)], device="cuda", dtype=torch.float64)
    if ph.numel():
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
    f, b = t.tolist()
    target = max(gemm_ms, link_ms)
    row = {"bench": "moe_layer", "transport": args.transport, "n_gpus": world, "tokens_per_rank": args.tokens,
           "hidden": h, "experts": args.experts, "topk": args.topk, "inter": i,
           "slots_per_rank": topo.slots_per_rank, "skew_s": args.skew, "fwd_ms": round(f, 3), "bwd_ms": round(b, 3),
           "total_ms": round(f + b, 3), "roofline": {"gemm_ms": round(gemm_ms, 3), "nvlink_ms": round(link_ms, 3),
                                                     "target_ms": round(target, 3),
                                                     "frac": round(target / (f + b), 3), "peak": src,
                                                     "link_bytes_per_rank_max": link_bytes},
           "assignments_recv_max": int(A_recv.max().item()), "assignments_recv_min": int(A_recv.min().item()),
           "remote_rows_out_max": int(rows_out.max().item()),
           "tflops_per_rank": round(18.0 * A_recv.max().item() * h * i / ((f + b) * 1e-3) / 1e12, 1)}
    if ph.numel():
        pm = dict(zip(sorted(phases), ph.tolist()))
        row["phases_ms_max_over_ranks"] = {kk: round(v, 3) for kk, v in pm.items()}
        # NVLink bytes per fused kernel (max over ranks): rows out for dispatch / scatter, rows back for
        # the combines (pre-reduced: one partial per (token, GPU) pair)
        moved = {"dispatch": rows_out.max().item() * h * 2, "scatter": rows_out.max().item() * h * 2,
                 "combine": rows_in.max().item() * h * 2, "combine_bwd": rows_in.max().item() * h * 2}
        row["fused_kernels"] = {
            kk: {"ms": round(pm[kk], 3), "nvlink_bytes": int(moved[kk]),
                 "achieved_gbs": round(moved[kk] / (pm[kk] * 1e-3) / 1e9, 1),
                 "frac_of_link": round(moved[kk] / (pm[kk] * 1e-3) / 1e9 / link_gbs, 3)}
            for kk in pm if kk in moved and pm[kk] > 0}
        row["link_gbs"] = round(link_gbs, 1)
        row["link_source"] = "measured peer pull" if args.link_gbs else "nominal pool figure"
    if rank == 0:
        print(json.dumps(row), flush=True)
    if isinstance(blk.ep, p2p_ep.P2PExpertParallel):
        blk.ep.arena = None
    return row


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--inter", type=int, default=1536)
    ap.add_argument("--extra-slots", type=int, default=1)
    ap.add_argument("--skew", type=float, default=1.0)
    ap.add_argument("--transport", default="p2p", choices=("p2p", "nccl", "baseline"))
    ap.add_argument("--sweep", action="store_true", help="tokens {2048,8192,16384} x skew {0,0.6,1.0,1.4}")
    ap.add_argument("--no-link-probe", action="store_true", help="use 770 GB/s instead of measuring the link")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args()
    args.link_gbs = 0.0
    if args.sweep:
        for tk in (2048, 8192, 16384):
            for s in (0.0, 0.6, 1.0, 1.4):
                args.tokens, args.skew = tk, s
                run(args)
    else:
        run(args)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
