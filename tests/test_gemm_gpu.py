"""Numerics of the tcgen05 GEMM family against fp32 PyTorch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().t()


def _close(out, ref, tol=2e-2):
    out, ref = out.detach().float().cpu(), ref.detach().float().cpu()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"relative error {err / scale:.3e}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (1000, 776, 304), (4096, 2048, 2048), (77, 64, 128)])
def test_dense_forward(M, N, K):
    from placemoe_b200.ops import gemm_nt, check_device_error

    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    out = gemm_nt(a, b)
    torch.cuda.synchronize()
    check_device_error()
    _close(out, _ref(a, b))
    out32 = gemm_nt(a, b, out_dtype=torch.float32)
    _close(out32, _ref(a, b), 1e-3)


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (1000, 776, 304), (2048, 2048, 4096)])
def test_dense_dgrad_wgrad(M, N, K):
    from placemoe_b200.ops import gemm_nn, gemm_tn, check_device_error

    torch.manual_seed(1)
    dy = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    _close(gemm_nn(dy, w), dy.float() @ w.float())
    x = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    # dW[K, N] = dy^T x  (contraction over M)
    _close(gemm_tn(dy, x), dy.float().t() @ x.float())
    acc = torch.randn(K, N, device="cuda", dtype=torch.float32)
    ref = acc + dy.float().t() @ x.float()
    gemm_tn(dy, x, out=acc, accumulate=True)
    torch.cuda.synchronize()
    check_device_error()
    _close(acc, ref, 1e-3)


def test_linear_autograd():
    from placemoe_b200.ops import linear

    torch.manual_seed(2)
    x = torch.randn(3, 100, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(768, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = xr @ wr.t()
    yr.backward(g.float())
    _close(y, yr.detach())
    _close(x.grad, xr.grad)
    _close(w.grad, wr.grad)


def _segments(counts, align=128):
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + align - 1) // align * align)
    return offs


@pytest.mark.parametrize("align", [128, 256])
@pytest.mark.parametrize("E,H,I", [(4, 256, 256), (8, 512, 384), (16, 2048, 1024)])
def test_grouped_fc1_fc2_and_backward(E, H, I, align):
    """align 256 runs the CTA-pair (cta_group::2) kernels."""
    from placemoe_b200.ops import kernels, check_device_error

    torch.manual_seed(3)
    counts = [int(c) for c in torch.randint(0, 300, (E,))]
    counts[0] = 0
    offs = _segments(counts, align)
    rows = offs[-1] + align  # capacity larger than used rows
    x = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    scale = torch.zeros(rows, device="cuda", dtype=torch.float32)
    for e in range(E):
        x[offs[e]: offs[e] + counts[e]] = torch.randn(counts[e], H, device="cuda", dtype=torch.bfloat16)
        scale[offs[e]: offs[e] + counts[e]] = torch.rand(counts[e], device="cuda")
    w1 = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device="cuda") * 0.05).to(torch.bfloat16)
    off_t = torch.tensor(offs, device="cuda", dtype=torch.int32)
    k = kernels()
    h = torch.zeros(rows, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.zeros(rows, 2 * I, device="cuda", dtype=torch.bfloat16)
    k.moe_fc1_swiglu(x, w1, off_t, scale, h, gu, align, None)
    y = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    k.moe_grouped_gemm(h, w2, off_t, y, False, align)
    dy = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    for e in range(E):
        dy[offs[e]: offs[e] + counts[e]] = torch.randn(counts[e], H, device="cuda", dtype=torch.bfloat16)
    dgu = torch.zeros(rows, 2 * I, device="cuda", dtype=torch.bfloat16)
    dscale = torch.zeros(rows, device="cuda", dtype=torch.float32)
    k.moe_fc2_dgrad_dswiglu(dy, w2, off_t, gu, scale, dgu, dscale, align)
    dx = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    k.moe_grouped_gemm(dgu, w1, off_t, dx, True, align)
    dw1 = torch.zeros(E, 2 * I, H, device="cuda", dtype=torch.float32)
    dw2 = torch.zeros(E, H, I, device="cuda", dtype=torch.float32)
    k.moe_wgrad(dgu, x, off_t, dw1, False, None)
    k.moe_wgrad(dy, h, off_t, dw2, True, None)
    torch.cuda.synchronize()
    check_device_error()
    for e in range(E):
        s, c = offs[e], counts[e]
        if c == 0:
            assert dw1[e].abs().max().item() == 0
            continue
        xe = x[s: s + c].float().requires_grad_()
        w1e = w1[e].float().requires_grad_()
        w2e = w2[e].float().requires_grad_()
        se = scale[s: s + c].clone().requires_grad_()
        g_u = xe @ w1e.t()
        g, u = g_u[:, :I], g_u[:, I:]
        he = torch.nn.functional.silu(g) * u * se[:, None]
        ye = he @ w2e.t()
        ye.backward(dy[s: s + c].float())
        _close(gu[s: s + c], g_u.detach())
        _close(h[s: s + c], he.detach())
        _close(y[s: s + c], ye.detach())
        _close(dx[s: s + c], xe.grad)
        _close(dscale[s: s + c], se.grad, 3e-2)
        _close(dw1[e], w1e.grad, 3e-2)
        _close(dw2[e], w2e.grad, 3e-2)


@pytest.mark.parametrize("align", [128, 256])
def test_gathered_fc1_and_wgrad_match_materialised_rows(align):
    """TMA row-gather operands give the same results as an explicit gather of the rows."""
    from placemoe_b200.ops import kernels, check_device_error

    torch.manual_seed(4)
    E, H, I, T = 8, 512, 256, 700
    counts = [int(c) for c in torch.randint(0, 400, (E,))]
    offs = _segments(counts, align)
    rows = offs[-1] + align
    tok = torch.full((rows,), -1, dtype=torch.int32)
    for e in range(E):
        tok[offs[e]: offs[e] + counts[e]] = torch.randint(0, T, (counts[e],), dtype=torch.int32)
    tok = tok.cuda()
    xt = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    xd = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    valid = tok >= 0
    xd[valid] = xt[tok[valid].long()]
    scale = torch.rand(rows, device="cuda") * valid.float()
    w1 = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).to(torch.bfloat16)
    off_t = torch.tensor(offs, device="cuda", dtype=torch.int32)
    k = kernels()
    h0 = torch.zeros(rows, I, device="cuda", dtype=torch.bfloat16)
    g0 = torch.zeros(rows, 2 * I, device="cuda", dtype=torch.bfloat16)
    k.moe_fc1_swiglu(xd, w1, off_t, scale, h0, g0, align, None)
    h1 = torch.zeros_like(h0)
    g1 = torch.zeros_like(g0)
    k.moe_fc1_swiglu(xt, w1, off_t, scale, h1, g1, align, tok)
    dgu = torch.randn(rows, 2 * I, device="cuda", dtype=torch.bfloat16) * valid[:, None].to(torch.bfloat16)
    dw0 = torch.zeros(E, 2 * I, H, device="cuda")
    dw1 = torch.zeros(E, 2 * I, H, device="cuda")
    k.moe_wgrad(dgu, xd, off_t, dw0, False, None)
    k.moe_wgrad(dgu, xt, off_t, dw1, False, tok)
    torch.cuda.synchronize()
    check_device_error()
    v = valid.cpu()
    assert torch.equal(h0.cpu()[v], h1.cpu()[v])
    assert torch.equal(g0.cpu()[v], g1.cpu()[v])
    _close(dw1, dw0, 1e-5)
