"""Numerics of the memory-bound and attention kernels against fp32 PyTorch references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).abs().max() / (b.abs().max() + 1e-6)).item()


# rows > 148 SMs x 8 warps x 4 stages exercise the reuse of every ring stage
@pytest.mark.parametrize("rows,hidden,wdtype", [(1000, 2048, torch.float32), (20011, 2048, torch.float32),
                                                (9000, 4096, torch.bfloat16), (5, 256, torch.float32),
                                                (12000, 512, torch.float32)])
def test_rmsnorm_fwd_bwd(rows, hidden, wdtype):
    from placemoe_b200.ops.norm import rmsnorm, rmsnorm_reference

    torch.manual_seed(0)
    x = torch.randn(rows, hidden, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda")).to(wdtype).requires_grad_()
    y = rmsnorm(x, w, 1e-6)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().clone().requires_grad_()
    yr = rmsnorm_reference(xr, wr, 1e-6)
    yr.backward(g.float())
    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 2e-2
    assert rel(w.grad, wr.grad) < 1e-2


@pytest.mark.parametrize("rows,hidden,wdtype", [(20011, 2048, torch.float32), (9000, 4096, torch.float32),
                                                (5, 256, torch.bfloat16), (3000, 1024, torch.float32)])
def test_add_rmsnorm_fwd_bwd(rows, hidden, wdtype):
    """Residual add fused into the RMSNorm (forward) and the residual-path gradient fused into its
    backward, against the fp32 reference of h = x + res, y = rmsnorm(h) with h also used downstream."""
    from placemoe_b200.ops import check_device_error
    from placemoe_b200.ops.mp import add_rmsnorm
    from placemoe_b200.ops.norm import rmsnorm_reference

    torch.manual_seed(1)
    x = torch.randn(rows, hidden, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    res = torch.randn(rows, hidden, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda")).to(wdtype).requires_grad_()
    h, y = add_rmsnorm(x, res, w, 1e-6)
    assert torch.equal(h, x.detach() + res.detach())  # the same bf16 rounding as a tensor add
    gh, gy = torch.randn_like(h), torch.randn_like(y)
    torch.autograd.backward([h, y], [gh, gy])
    xr, rr = x.detach().float().requires_grad_(), res.detach().float().requires_grad_()
    wr = w.detach().float().clone().requires_grad_()
    hr = xr + rr
    yr = rmsnorm_reference(hr, wr, 1e-6)
    torch.autograd.backward([hr, yr], [gh.float(), gy.float()])
    torch.cuda.synchronize()
    check_device_error()
    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 2e-2 and rel(res.grad, rr.grad) < 2e-2
    wg = w.main_grad if getattr(w, "main_grad", None) is not None else w.grad
    assert rel(wg, wr.grad) < 1e-2


# t = 5000 gives every CTA of the persistent grid several tokens, so every ring stage is reused
@pytest.mark.parametrize("hq,hkv,d,mode,t", [(16, 16, 128, "full", 512), (32, 4, 128, "per_head", 512),
                                           (8, 2, 64, "per_head", 512), (64, 32, 128, "per_head", 512),
                                           (24, 8, 64, "full", 512), (16, 16, 128, "full", 5000),
                                           (32, 4, 128, "per_head", 5000)])
def test_qkv_norm_rope(hq, hkv, d, mode, t):
    from placemoe_b200.ops.norm import qkv_norm_rope, rope_inv_freq

    torch.manual_seed(1)
    width = (hq + 2 * hkv) * d
    qkv = torch.randn(t, width, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    qg, kg = (d, d) if mode == "per_head" else (hq * d, hkv * d)
    qw = (1 + 0.1 * torch.randn(qg, device="cuda")).requires_grad_()
    kw = (1 + 0.1 * torch.randn(kg, device="cuda")).requires_grad_()
    pos = (torch.arange(t, device="cuda") % 256).to(torch.int32)
    inv = rope_inv_freq(d, 1e6, "cuda")
    q, k, v = qkv_norm_rope(qkv, qw, kw, pos, inv, hq, hkv, d, qg, kg, 1e-6)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    (q.float() * gq).sum().add_((k.float() * gk).sum()).add_((v.float() * gv).sum()).backward()
    qkv_r = qkv.detach().float().requires_grad_()
    qw_r = qw.detach().clone().requires_grad_()
    kw_r = kw.detach().clone().requires_grad_()
    qr, kr, vr = qkv_norm_rope(qkv_r.cpu(), qw_r.cpu(), kw_r.cpu(), pos.cpu(), inv.cpu(), hq, hkv, d, qg, kg, 1e-6)
    (qr * gq.float().cpu()).sum().add_((kr * gk.float().cpu()).sum()).add_((vr * gv.float().cpu()).sum()).backward()
    assert rel(q.cpu(), qr) < 1e-2 and rel(k.cpu(), kr) < 1e-2 and rel(v.cpu(), vr) < 1e-2
    assert rel(qkv.grad.cpu(), qkv_r.grad) < 2e-2
    assert rel(qw.main_grad.cpu(), qw_r.grad) < 2e-2
    assert rel(kw.main_grad.cpu(), kw_r.grad) < 2e-2


@pytest.mark.parametrize("e,k,renorm", [(64, 8, False), (128, 8, True), (16, 4, True)])
def test_router_topk(e, k, renorm):
    from placemoe_b200.ops import kernels
    from placemoe_b200.ops.moe import router_reference

    torch.manual_seed(2)
    t = 3000
    logits = torch.randn(t, e, device="cuda")
    bias = torch.randn(e, device="cuda")
    idx, w, ps, cnt = kernels().router_topk_fwd(logits, bias, k, renorm)
    ref = router_reference(logits, bias, k, renorm)
    assert torch.equal(idx.long().sort(-1).values, ref.idx.long().sort(-1).values)
    # same order (descending prob) as torch.topk for distinct values
    assert (w - ref.weight).abs().max().item() < 1e-5
    assert rel(ps, ref.prob_sum) < 1e-4 and torch.equal(cnt, ref.count)
    # backward: d(logits) of sum(dw * w) + sum(aux * p)
    dw = torch.randn(t, k, device="cuda")
    aux = torch.randn(e, device="cuda") * 0.01
    dl = kernels().router_topk_bwd(logits, bias, idx, dw, aux, renorm)
    z = (logits + bias).requires_grad_()
    p = torch.softmax(z, -1)
    wsel = p.gather(1, idx.long())
    if renorm:
        wsel = wsel / wsel.sum(-1, keepdim=True)
    ((wsel * dw).sum() + (p * aux).sum()).backward()
    assert rel(dl, z.grad) < 2e-2


def test_moe_plan_and_rows():
    from placemoe_b200.ops import kernels

    torch.manual_seed(3)
    t, k, s = 4000, 8, 64
    idx = torch.randint(0, s, (t, k), device="cuda", dtype=torch.int32)
    w = torch.rand(t, k, device="cuda")
    cap = t * k + s * 128
    offsets, counts, row_of, row_token, row_scale = kernels().moe_plan(idx, None, w, s, cap, 128)
    off = offsets.cpu()
    ref_counts = torch.bincount(idx.reshape(-1).long().cpu(), minlength=s)
    assert torch.equal(counts.cpu().long(), ref_counts)
    assert all(int(off[i + 1] - off[i]) % 128 == 0 for i in range(s))
    ro = row_of.cpu().long()
    flat = idx.reshape(-1).cpu().long()
    # every assignment lands inside its slot segment, in token order (stable)
    for e in range(0, s, 7):
        rows = ro[flat == e]
        assert bool((rows >= off[e]).all()) and bool((rows < off[e] + ref_counts[e]).all())
        assert bool((rows[1:] > rows[:-1]).all())
    assert torch.equal(row_token.cpu().long()[ro], torch.arange(t * k) // k)
    assert torch.allclose(row_scale.cpu()[ro], w.reshape(-1).cpu())
    # gather + sum round trip
    x = torch.randn(t, 256, device="cuda", dtype=torch.bfloat16)
    xd = torch.empty(cap, 256, device="cuda", dtype=torch.bfloat16)
    kernels().gather_rows(x, row_token, offsets[s:], xd)
    out = torch.empty_like(x)
    kernels().sum_rows(xd, row_of, out)
    assert rel(out, x.float() * k) < 1e-2


@pytest.mark.parametrize("cfg", [(64, 8, False, 2048, 1024), (128, 8, True, 2048, 768), (16, 4, True, 256, 256)])
def test_moe_block_matches_reference(cfg):
    from placemoe_b200.ops.moe import moe_block, moe_block_reference

    e, k, renorm, h, inter = cfg
    torch.manual_seed(4)
    t = 1024
    x = torch.randn(t, h, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    # bf16-representable router weights: reference and kernel see the same logits, no top-k flips
    wg = (torch.randn(e, h, device="cuda") * 0.02).bfloat16().float().requires_grad_()
    bias = torch.randn(e, device="cuda") * 0.5
    p1 = (torch.randn(e, 2 * inter, h, device="cuda") * 0.02).requires_grad_()
    p2 = (torch.randn(e, h, inter, device="cuda") * 0.02).requires_grad_()
    y, aux, _ = moe_block(x, wg, bias, p1.detach().bfloat16(), p2.detach().bfloat16(), p1, p2, k, renorm, e,
                          aux_coef=0.01)
    g = torch.randn_like(y)
    ((y.float() * g.float()).sum() + aux).backward()
    xr = x.detach().float().requires_grad_()
    wgr = wg.detach().clone().requires_grad_()
    p1r = p1.detach().clone().requires_grad_()
    p2r = p2.detach().clone().requires_grad_()
    yr, auxr = moe_block_reference(xr, wgr, bias, p1r, p2r, k, renorm, 0.01)
    ((yr.float() * g.float()).sum() + auxr).backward()
    assert rel(y, yr) < 3e-2
    assert abs(aux.item() - auxr.item()) < 1e-4
    assert rel(x.grad, xr.grad) < 5e-2
    assert rel(wg.main_grad, wgr.grad) < 5e-2
    assert rel(p1.main_grad, p1r.grad) < 5e-2
    assert rel(p2.main_grad, p2r.grad) < 5e-2


def test_fused_adamw_matches_torch():
    from placemoe_b200.ops.optim import FusedAdamW

    torch.manual_seed(5)
    ps = [torch.randn(n, device="cuda", requires_grad=True) for n in (1000, 65536 * 3 + 17, 4096)]
    ref = [p.detach().clone().requires_grad_() for p in ps]
    shadow = torch.empty(ps[1].shape, device="cuda", dtype=torch.bfloat16)
    ps[1].bf16_shadow = shadow
    opt = FusedAdamW(ps, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    topt = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(3):
        for p, r in zip(ps, ref):
            g = torch.randn_like(p)
            p.grad = g.clone()
            r.grad = g.clone()
        opt.step()
        topt.step()
    for p, r in zip(ps, ref):
        assert (p - r).abs().max().item() < 1e-5
    assert torch.equal(shadow, ps[1].detach().to(torch.bfloat16))


def test_fused_linear_ce():
    from placemoe_b200.ops.loss import fused_linear_cross_entropy

    torch.manual_seed(6)
    n, h, v = 3000, 512, 50304
    x = torch.randn(n, h, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(v, h, device="cuda") * 0.02).to(torch.bfloat16).requires_grad_()
    lab = torch.randint(0, v, (n,), device="cuda")
    lab[::7] = -100
    loss = fused_linear_cross_entropy(x, w, lab, chunk=1024)
    loss.backward()
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    lr_ = torch.nn.functional.cross_entropy(xr @ wr.t(), lab, ignore_index=-100)
    lr_.backward()
    assert abs(loss.item() - lr_.item()) / lr_.item() < 1e-2
    assert rel(x.grad, xr.grad) < 3e-2
    assert rel(w.grad, wr.grad) < 3e-2


@pytest.mark.parametrize("b,s,hq,hkv,d,qscale", [(1, 128, 1, 1, 128, 1.0), (2, 512, 4, 2, 128, 1.0),
                                                 (1, 1024, 16, 16, 128, 1.0), (2, 256, 8, 2, 64, 1.0),
                                                 (1, 1024, 2, 1, 128, 8.0), (1, 384, 2, 2, 64, 4.0),
                                                 (1, 512, 8, 1, 128, 1.0)])
def test_attention_fwd_bwd(b, s, hq, hkv, d, qscale):
    """qscale > 1 spreads the scores so that the running row max moves often (rescaling paths)."""
    from placemoe_b200.ops import kernels
    from placemoe_b200.ops.attention import attention_reference, causal_attention

    assert hasattr(kernels(), "attn_fwd"), "attention kernel must be built in"
    torch.manual_seed(7)
    t = b * s
    q = (torch.randn(t, hq, d, device="cuda") * qscale).to(torch.bfloat16).requires_grad_()
    k = torch.randn(t, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = causal_attention(q, k, v, s)
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (z.detach().float().requires_grad_() for z in (q, k, v))
    orf = attention_reference(qr, kr, vr, s)
    orf.backward(g.float())
    assert rel(o, orf) < 2e-2
    assert rel(q.grad, qr.grad) < 5e-2
    assert rel(k.grad, kr.grad) < 5e-2
    assert rel(v.grad, vr.grad) < 5e-2
    from placemoe_b200.ops import check_device_error

    torch.cuda.synchronize()
    check_device_error()
    assert math.isfinite(o.float().sum().item())


def test_sq_norm_matches_torch():
    from placemoe_b200.ops import kernels

    torch.manual_seed(6)
    gs = [torch.randn(n, device="cuda") for n in (1000, 65536 * 3 + 17, 7)]
    gs.append(torch.randn(12345, device="cuda").bfloat16())
    gs.append(torch.randn(20000, device="cuda").bfloat16()[1:])  # unaligned start
    gs[-1] = gs[-1].contiguous()
    weights = [1.0, 0.5, 2.0, 1.0, 0.25]
    table, meta = kernels().sq_norm_build_table(gs, weights)
    out = torch.zeros(1, device="cuda")
    kernels().sq_norm(table, meta, out)
    ref = sum(w * g.double().pow(2).sum() for g, w in zip(gs, weights))
    assert abs(out.item() - ref.item()) / ref.item() < 1e-5


@pytest.mark.parametrize("d,hq,hkv", [(128, 4, 2), (64, 2, 2)])
def test_attention_packed_documents(d, hq, hkv):
    """Several documents per row (boundaries inside and across tiles, 1-token documents): the
    document-masked kernels against the fp32 block-diagonal causal reference."""
    from placemoe_b200.ops.attention import attention_reference, causal_attention, doc_bounds

    torch.manual_seed(11)
    s, b = 512, 2
    t = b * s
    cuts = sorted({0, 1, 2, 130, 200, 255, 256, 400, 511, s} | {s + x for x in (0, 3, 128, 300, 301)} | {2 * s})
    cu = torch.tensor(cuts, dtype=torch.int32, device="cuda")
    docs = doc_bounds(cu, t, s)
    q = torch.randn(t, hq, d, device="cuda").to(torch.bfloat16).requires_grad_()
    k = torch.randn(t, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = causal_attention(q, k, v, s, docs)
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (z.detach().float().requires_grad_() for z in (q, k, v))
    orf = attention_reference(qr, kr, vr, s, docs)
    orf.backward(g.float())
    assert torch.isfinite(o.float()).all()
    assert rel(o, orf) < 2e-2
    assert rel(q.grad, qr.grad) < 5e-2
    assert rel(k.grad, kr.grad) < 5e-2
    assert rel(v.grad, vr.grad) < 5e-2
    from placemoe_b200.ops import check_device_error

    torch.cuda.synchronize()
    check_device_error()


@pytest.mark.gpu
def test_peer_barrier_times_out_and_status_is_sticky():
    """A bounded peer wait that runs out: one GPU, a two-entry peer table whose second flag is never
    written.  The kernel returns an error status (no trap); a later wait returns at once; the host raises."""
    import time

    from placemoe_b200.ops import check_device_error, kernels, p2p_status

    kn = kernels()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = p2p_status(dev)
    check_device_error()  # start clean
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    peers = torch.tensor([flags.data_ptr(), flags.data_ptr()], dtype=torch.int64, device=dev)
    t0 = time.perf_counter()
    kn.p2p_barrier(peers, 0, 0, 1, 0.3, st)
    torch.cuda.synchronize()
    first = time.perf_counter() - t0
    assert st.tolist()[:2] == [2, 1]  # peer wait timed out, in the p2p barrier
    t1 = time.perf_counter()
    kn.p2p_barrier(peers, 0, 0, 2, 5.0, st)  # sticky: returns without waiting out its budget
    torch.cuda.synchronize()
    second = time.perf_counter() - t1
    assert 0.25 < first < 5.0, first
    assert second < 1.0, second
    with pytest.raises(RuntimeError, match="peer wait timed out"):
        check_device_error()
    assert st.tolist()[0] == 0
    # the context stays usable
    x = torch.ones(1024, device=dev)
    assert float(x.sum()) == 1024.0
