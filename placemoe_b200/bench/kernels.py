"""Kernel microbenchmarks with CUDA-event timing and roofline fractions.

    python -m placemoe_b200.bench.kernels --op gemm --m 8192 --n 2048 --k 2048
    python -m placemoe_b200.bench.kernels --op moe_fc1 --tokens 16384 --experts 64 --hidden 2048 --inter 1024
    python -m placemoe_b200.bench.kernels --op attn --batch 2 --seq 4096 --heads 16 --kv-heads 16
    python -m placemoe_b200.bench.kernels --op all

Timing: warm-up launches, then ``--iters`` launches between two CUDA events
on the launching stream with a synchronize on both sides; inputs are larger
than the 126 MB L2 or an L2-flush write of 256 MB precedes every timed
launch (``--flush``).  Fractions are against ``MEASURED_PEAKS.json``
(bf16_tflops burst, hbm_gbs) when present, else 1.59 PFLOP/s and 6.65 TB/s.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


def time_fn(fn, iters=20, warmup=5, flush=True):
    buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda") if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        if buf is not None:
            buf.fill_(1.0)  # evict L2
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def report(name, ms, flops=0.0, nbytes=0.0):
    tf, gbs, src = peaks()
    row = {"op": name, "ms": round(ms, 4)}
    if flops:
        row["tflops"] = round(flops / ms / 1e9, 1)
        row[f"frac_of_{src}_bf16"] = round(flops / ms / 1e9 / tf, 3)
    if nbytes:
        row["gbs"] = round(nbytes / ms / 1e6, 1)
        row[f"frac_of_{src}_hbm"] = round(nbytes / ms / 1e6 / gbs, 3)
    print(json.dumps(row), flush=True)
    return row


def bench_gemm(m, n, k, iters):
    from placemoe_b200.ops.gemm import gemm_nn, gemm_nt, gemm_tn

    a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    f = 2.0 * m * n * k
    report(f"gemm_fwd[{m}x{n}x{k}]", time_fn(lambda: gemm_nt(a, b, out=out), iters), f)
    # the same product through cuBLAS (torch.matmul), for a same-box comparison
    bt = b.t()
    report(f"cublas_fwd[{m}x{n}x{k}]", time_fn(lambda: torch.matmul(a, bt, out=out), iters), f)
    w = torch.randn(k, n, device="cuda", dtype=torch.bfloat16)
    out2 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    report(f"gemm_dgrad[{m}x{n}x{k}]", time_fn(lambda: gemm_nn(a, w, out=out2), iters), f)
    dy = torch.randn(k, m, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(k, n, device="cuda", dtype=torch.bfloat16)
    acc = torch.zeros(m, n, device="cuda", dtype=torch.float32)
    report(f"gemm_wgrad_f32acc[{m}x{n}x{k}]", time_fn(lambda: gemm_tn(dy, x, out=acc, accumulate=True), iters), f)


def _moe_inputs(tokens, experts, k, hidden, inter, skew=1.0, align=128):
    from placemoe_b200.models.config import zipf_router_bias
    from placemoe_b200.ops import kernels
    from placemoe_b200.ops.moe import capacity_rows

    g = torch.Generator(device="cuda").manual_seed(0)
    logits = torch.randn(tokens, experts, device="cuda", generator=g) + torch.from_numpy(
        zipf_router_bias(experts, skew)).cuda()
    idx, w, _, _ = kernels().router_topk_fwd(logits.contiguous(), None, k, False)
    cap = capacity_rows(tokens, k, experts, align)
    offsets, counts, row_of, row_token, row_scale = kernels().moe_plan(idx, None, w, experts, cap, align)
    x = torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    xd = torch.empty(cap, hidden, device="cuda", dtype=torch.bfloat16)
    kernels().gather_rows(x, row_token, offsets[experts:], xd)
    w1 = (torch.randn(experts, 2 * inter, hidden, device="cuda") * 0.02).bfloat16()
    w2 = (torch.randn(experts, hidden, inter, device="cuda") * 0.02).bfloat16()
    return offsets, row_of, row_token, row_scale, xd, w1, w2, cap


def bench_moe(tokens, experts, k, hidden, inter, iters, skew, align=128):
    from placemoe_b200.ops import kernels

    kn = kernels()
    offsets, row_of, row_token, row_scale, xd, w1, w2, cap = _moe_inputs(tokens, experts, k, hidden, inter, skew,
                                                                         align)
    rows = tokens * k
    h = torch.empty(cap, inter, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(cap, 2 * inter, device="cuda", dtype=torch.bfloat16)
    f1 = 2.0 * rows * 2 * inter * hidden
    report(f"moe_fc1_swiglu[T{tokens} E{experts} k{k} H{hidden} I{inter} align{align}]",
           time_fn(lambda: kn.moe_fc1_swiglu(xd, w1, offsets, row_scale, h, gu, align, None), iters), f1)
    y = torch.empty(cap, hidden, device="cuda", dtype=torch.bfloat16)
    f2 = 2.0 * rows * inter * hidden
    report("moe_fc2", time_fn(lambda: kn.moe_grouped_gemm(h, w2, offsets, y, False, align), iters), f2)
    dgu = torch.empty_like(gu)
    dscale = torch.zeros(cap, device="cuda")
    report("moe_fc2_dgrad_dswiglu",
           time_fn(lambda: kn.moe_fc2_dgrad_dswiglu(y, w2, offsets, gu, row_scale, dgu, dscale, align), iters), f2)
    dx = torch.empty_like(xd)
    report("moe_fc1_dgrad", time_fn(lambda: kn.moe_grouped_gemm(dgu, w1, offsets, dx, True, align), iters), f1)
    dw1 = torch.zeros(experts, 2 * inter, hidden, device="cuda")
    report("moe_fc1_wgrad_f32acc", time_fn(lambda: kn.moe_wgrad(dgu, xd, offsets, dw1, True, None), iters), f1)
    dw2 = torch.zeros(experts, hidden, inter, device="cuda")
    report("moe_fc2_wgrad_f32acc", time_fn(lambda: kn.moe_wgrad(y, h, offsets, dw2, True, None), iters), f2)
    # the same fc1 GEMMs reading token rows through TMA row gathers (no dispatched copy)
    xt = torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    report("moe_fc1_swiglu_gathered",
           time_fn(lambda: kn.moe_fc1_swiglu(xt, w1, offsets, row_scale, h, gu, align, row_token), iters), f1)
    report("moe_fc1_wgrad_f32acc_gathered",
           time_fn(lambda: kn.moe_wgrad(dgu, xt, offsets, dw1, True, row_token), iters), f1)


def bench_attn(batch, seq, heads, kv_heads, dim, iters):
    from placemoe_b200.ops import kernels

    t = batch * seq
    q = torch.randn(t, heads, dim, device="cuda", dtype=torch.bfloat16)
    kk = torch.randn(t, kv_heads, dim, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(t, kv_heads, dim, device="cuda", dtype=torch.bfloat16)
    f = 4.0 * batch * seq * seq / 2 * heads * dim  # causal
    o, lse = kernels().attn_fwd(q, kk, v, seq)
    report(f"attn_fwd[B{batch} S{seq} H{heads}/{kv_heads} D{dim}]",
           time_fn(lambda: kernels().attn_fwd(q, kk, v, seq), iters), f)
    do = torch.randn_like(o)
    report("attn_bwd", time_fn(lambda: kernels().attn_bwd(q, kk, v, o, lse, do, seq), iters), 2.5 * f)


def bench_attn_compare(batch, seq, heads, kv_heads, dim, iters):
    """Same-box comparison of the tcgen05 attention kernels with PyTorch SDPA backends (causal).

    SDPA runs in its own [B, H, S, D] layout; its backward time is (forward + backward) - forward.
    FLOPs count the causal half: forward 4*B*S^2/2*H*D, backward 2.5x that.
    """
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from placemoe_b200.ops import kernels

    t = batch * seq
    f = 4.0 * batch * seq * seq / 2 * heads * dim
    tag = f"B{batch} S{seq} H{heads}/{kv_heads} D{dim}"
    q = torch.randn(t, heads, dim, device="cuda", dtype=torch.bfloat16)
    kk = torch.randn(t, kv_heads, dim, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(t, kv_heads, dim, device="cuda", dtype=torch.bfloat16)
    o, lse = kernels().attn_fwd(q, kk, v, seq)
    do = torch.randn_like(o)
    report(f"ours attn_fwd[{tag}]", time_fn(lambda: kernels().attn_fwd(q, kk, v, seq), iters), f)
    report(f"ours attn_bwd[{tag}]", time_fn(lambda: kernels().attn_bwd(q, kk, v, o, lse, do, seq), iters), 2.5 * f)
    qb = q.view(batch, seq, heads, dim).transpose(1, 2).contiguous().requires_grad_()
    kb = kk.view(batch, seq, kv_heads, dim).transpose(1, 2).contiguous().requires_grad_()
    vb = v.view(batch, seq, kv_heads, dim).transpose(1, 2).contiguous().requires_grad_()
    dob = do.view(batch, seq, heads, dim).transpose(1, 2).contiguous()
    gqa = heads != kv_heads
    for name, backend in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION),
                          ("efficient", SDPBackend.EFFICIENT_ATTENTION)):
        try:
            with sdpa_kernel(backend):
                def fwd():
                    with torch.no_grad():
                        return F.scaled_dot_product_attention(qb, kb, vb, is_causal=True, enable_gqa=gqa)

                def fwd_bwd():
                    out = F.scaled_dot_product_attention(qb, kb, vb, is_causal=True, enable_gqa=gqa)
                    out.backward(dob)
                    qb.grad = kb.grad = vb.grad = None

                tf = time_fn(fwd, iters)
                tfb = time_fn(fwd_bwd, iters)
            report(f"sdpa-{name} fwd[{tag}]", tf, f)
            report(f"sdpa-{name} bwd[{tag}]", max(tfb - tf, 1e-6), 2.5 * f)
        except RuntimeError as e:  # backend not available for this shape / GPU
            print(json.dumps({"op": f"sdpa-{name}[{tag}]", "unavailable": str(e).splitlines()[0][:200]}), flush=True)


def bench_ep_local(tokens, iters):
    """Fused EP kernels on a one-rank group (OLMoE expert shape): every assignment stays on this GPU, so
    this times the kernels' local work -- histograms, positions, row stores, padding, local copies, the
    fp32 pre-reduction and token sums -- without NVLink traffic.  Per-kernel CUDA-event times (mean)."""
    import torch.distributed as dist  # noqa: F401  (the one-rank arena needs no process group)

    from placemoe_b200.models.config import get_preset
    from placemoe_b200.models.moe_decoder import MoEBlock
    from placemoe_b200.parallel import p2p_ep
    from placemoe_b200.parallel.data_parallel import expert_topology
    from placemoe_b200.parallel.placement import build_placements

    cfg = get_preset("olmoe_1b_7b")
    topo = expert_topology(cfg.num_experts, 1, 0)
    with torch.device("cuda"):
        blk = MoEBlock(cfg, 0, topo.slots_per_rank)
    torch.manual_seed(0)
    with torch.no_grad():
        blk.gate.normal_(0, 0.02)
        blk.gate_up_proj.normal_(0, 0.02)
        blk.down_proj.normal_(0, 0.02)
    blk.placement = build_placements(None, topo, 0, [blk.layer_key])[blk.layer_key]
    blk.ep = p2p_ep.P2PExpertParallel()
    blk.ep_slab = 0
    blk.train()
    x = torch.randn(tokens, cfg.hidden_size, device="cuda").bfloat16().requires_grad_()
    dy = torch.randn(tokens, cfg.hidden_size, device="cuda").bfloat16()
    for _ in range(3):
        blk(x).backward(dy)
    torch.cuda.synchronize()
    acc: dict = {}
    for _ in range(iters):
        p2p_ep.TIMER = p2p_ep.PhaseTimer()
        blk(x).backward(dy)
        torch.cuda.synchronize()
        for k, v in p2p_ep.TIMER.phases().items():
            acc[k] = acc.get(k, 0.0) + v / iters
    p2p_ep.TIMER = None
    rows = tokens * cfg.num_experts_per_tok * cfg.hidden_size * 2  # bytes of the expert-side rows
    tok = tokens * cfg.hidden_size * 2
    # HBM bytes each kernel must move at one rank: dispatch reads x and writes every expert row (primary
    # stores + local copies read the primary); combine reads every expert row, writes and re-reads one
    # partial per token and writes y; scatter mirrors dispatch for dy; combine_bwd mirrors combine.
    need = {"dispatch": tok + 2 * rows, "scatter": tok + 2 * rows, "combine": rows + 3 * tok,
            "combine_bwd": rows + 3 * tok}
    for k in ("dispatch", "combine", "scatter", "combine_bwd"):
        if k in acc:
            report(f"ep_{k}[one rank, T{tokens} k{cfg.num_experts_per_tok} H{cfg.hidden_size}]", acc[k],
                   nbytes=need[k])
    # one more pass with CTA 0's phase timestamps (%globaltimer) to split each kernel's time
    from placemoe_b200.ops import kernels

    marks = torch.zeros(24, dtype=torch.int64, device="cuda")
    kernels().ep_phase_marks(marks)
    y = blk(x)
    torch.cuda.synchronize()
    fwd = marks.tolist()  # dispatch 0-7, combine (forward) 8-11
    y.backward(dy)
    torch.cuda.synchronize()
    bwd = marks.tolist()  # scatter 16-19, combine_bwd 8-11
    kernels().ep_phase_marks(None)

    def split(m, base, names):
        return {n: round((m[base + i + 1] - m[base + i]) / 1e3, 1) for i, n in enumerate(names)}

    print(json.dumps({"ep_phases_us": {
        "dispatch": split(fwd, 0, ["histogram", "count_exchange", "segments", "positions", "row_stores",
                                   "rows_barrier", "local_copies"]),
        "combine": split(fwd, 8, ["pre_reduce", "barrier", "token_sums"]),
        "scatter": split(bwd, 16, ["row_stores", "barrier", "local_copies"]),
        "combine_bwd": split(bwd, 8, ["pre_reduce", "barrier", "token_sums"])}}), flush=True)


def bench_memory(tokens, hidden, iters):
    from placemoe_b200.ops import kernels

    x = torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(hidden, device="cuda")
    report(f"rmsnorm_fwd[{tokens}x{hidden}]", time_fn(lambda: kernels().rmsnorm_fwd(x, w, 1e-6), iters),
           nbytes=2 * x.numel() * 2)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="all",
                    choices=("all", "gemm", "moe", "attn", "attn_compare", "memory", "ep_local"))
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=2048)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=1024)
    ap.add_argument("--skew", type=float, default=1.0)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=16)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--align", type=int, default=0, help="MoE segment alignment (0: both 128 and 256)")
    a = ap.parse_args()
    if a.op in ("all", "gemm"):
        bench_gemm(a.m, a.n, a.k, a.iters)
        if a.op == "all":
            bench_gemm(16384, 4096, 4096, a.iters)
            bench_gemm(8192, 8192, 8192, a.iters)
    if a.op in ("all", "moe"):
        for al in (128, 256) if a.align == 0 else (a.align,):
            bench_moe(a.tokens, a.experts, a.topk, a.hidden, a.inter, a.iters, a.skew, al)
    if a.op in ("all", "attn"):
        bench_attn(a.batch, a.seq, a.heads, a.kv_heads, a.dim, a.iters)
    if a.op == "ep_local":
        bench_ep_local(a.tokens, a.iters)
    if a.op == "attn_compare":
        bench_attn_compare(a.batch, a.seq, a.heads, a.kv_heads, a.dim, a.iters)
    if a.op in ("all", "memory"):
        bench_memory(a.tokens, a.hidden, a.iters)
    from placemoe_b200.ops import check_device_error

    torch.cuda.synchronize()
    check_device_error()


if __name__ == "__main__":
    main()


