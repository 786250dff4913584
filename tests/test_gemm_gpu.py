"""tcgen05 GEMM (forward / dgrad / wgrad + fused epilogues) against fp32 torch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 64), (333, 776, 200), (1000, 1536, 1536), (4096, 512, 4096), (16, 1032, 1536),
          (5328, 4608, 1536)]


@pytest.fixture(scope="module")
def E():
    from verl_omni_b200.ops._ext import ext

    e = ext()
    e.gemm_error(True)
    yield e
    assert e.gemm_error(True) == 0, "GEMM kernel reported a barrier timeout"


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-6))


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_fwd_bias(E, M, N, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    b = torch.randn(N, device="cuda").bfloat16()
    out, _ = E.gemm_fwd(x, w, b, 1, None, None, 1)
    ref = x.float() @ w.float().t() + b.float()
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", SHAPES[:3])
def test_gemm_fwd_gelu_and_gate_res(E, M, N, K):
    torch.manual_seed(1)
    S = M // 2 if M % 2 == 0 else M
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    b = torch.randn(N, device="cuda").bfloat16()
    out, pre = E.gemm_fwd(x, w, b, 2, None, None, 1)
    lin = x.float() @ w.float().t() + b.float()
    assert _rel(pre, lin) < 1e-2
    assert _rel(out, torch.nn.functional.gelu(lin, approximate="tanh")) < 2e-2
    B = M // S
    gate = torch.randn(B, N, device="cuda").bfloat16()
    res = torch.randn(M, N, device="cuda").bfloat16()
    out, lin2 = E.gemm_fwd(x, w, b, 3, gate, res, S)
    ref = res.float() + (lin.view(B, S, N) * gate.float()[:, None]).view(M, N)
    assert _rel(lin2, lin) < 1e-2
    assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_dgrad(E, M, N, K):
    torch.manual_seed(2)
    dy = torch.randn(M, N, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / N ** 0.5).bfloat16()
    dx = E.gemm_dgrad(dy, w)
    assert _rel(dx, dy.float() @ w.float()) < 1e-2


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("accumulate", [False, True])
def test_gemm_wgrad(E, M, N, K, accumulate):
    torch.manual_seed(3)
    dy = torch.randn(M, N, device="cuda").bfloat16()
    x = torch.randn(M, K, device="cuda").bfloat16()
    out = torch.randn(N, K, device="cuda") if accumulate else torch.empty(N, K, device="cuda")
    base = out.clone()
    E.gemm_wgrad(dy, x, out, accumulate)
    ref = dy.float().t() @ x.float() + (base if accumulate else 0)
    assert _rel(out, ref) < 1e-2


def test_linear_layer_autograd_native_vs_torch():
    from verl_omni_b200.ops import linear as L

    torch.manual_seed(4)
    x = torch.randn(2, 300, 512, device="cuda").bfloat16().requires_grad_(True)
    w = (torch.randn(768, 512, device="cuda") / 512 ** 0.5).bfloat16().requires_grad_(True)
    b = torch.zeros(768, device="cuda").bfloat16().requires_grad_(True)
    w.main_grad = torch.zeros(768, 512, device="cuda")
    y = L.linear(x, w, b, epilogue="gelu")
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = torch.nn.functional.gelu(xr @ wr.t(), approximate="tanh")
    yr.backward(g.float())
    assert _rel(y, yr) < 2e-2
    assert _rel(x.grad, xr.grad) < 3e-2
    assert w.grad is None and _rel(w.main_grad, wr.grad) < 3e-2


@pytest.mark.parametrize("epilogue", ["none", "gelu", "gate_res"])
def test_fused_lora_linear_matches_unfused(E, epilogue):
    """Low-rank term folded into the base GEMM (extension operands): forward and adapter/input grads."""
    from verl_omni_b200.ops.linear import lora_linear

    torch.manual_seed(7)
    Bs, S, K, N, r, s = 2, 160, 256, 384, 16, 2.0
    x = torch.randn(Bs, S, K, device="cuda").bfloat16().requires_grad_(True)
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    b = torch.randn(N, device="cuda").bfloat16()
    A = (torch.randn(r, K, device="cuda") / K ** 0.5).bfloat16().requires_grad_(True)
    B = (torch.randn(N, r, device="cuda") * 0.1).bfloat16().requires_grad_(True)
    gate = torch.randn(Bs, N, device="cuda").bfloat16()
    res = torch.randn(Bs, S, N, device="cuda").bfloat16()
    kw = dict(gate=gate, res=res, S=S) if epilogue == "gate_res" else {}
    y = lora_linear(x, w, b, A, B, s, epilogue=epilogue, **kw)
    g = torch.randn_like(y)
    y.backward(g)
    xr, Ar, Br = (t.detach().float().requires_grad_(True) for t in (x, A, B))
    lin = xr @ w.float().t() + b.float() + s * (xr @ Ar.t()) @ Br.t()
    if epilogue == "gelu":
        yr = torch.nn.functional.gelu(lin, approximate="tanh")
    elif epilogue == "gate_res":
        yr = res.float() + lin * gate.float()[:, None]
    else:
        yr = lin
    yr.backward(g.float())
    assert _rel(y, yr) < 2e-2
    for a, ref in ((x, xr), (A, Ar), (B, Br)):
        assert _rel(a.grad, ref.grad) < 3e-2, (a.shape, _rel(a.grad, ref.grad))


PAIRS = [((16384, 1536, 1536), (5328, 1536, 1536)), ((1024, 4608, 1536), (333, 4608, 1536)),
         ((5328, 6144, 1536), (200, 6144, 1536)), ((640, 1536, 6144), (2048, 1536, 6144))]


@pytest.mark.parametrize("p0,p1", PAIRS)
@pytest.mark.parametrize("epi", [1, 2, 3])
def test_gemm_fwd_pair_matches_single(E, p0, p1, epi):
    """A grouped launch computes every tile exactly as the single launch of the same shape."""
    torch.manual_seed(5)
    args = []
    for (M, N, K) in (p0, p1):
        S = M // 2 if M % 2 == 0 else M
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
        b = torch.randn(N, device="cuda").bfloat16()
        gate = torch.randn(M // S, N, device="cuda").bfloat16() if epi == 3 else None
        res = torch.randn(M, N, device="cuda").bfloat16() if epi == 3 else None
        args.append((x, w, b, gate, res, S))
    outs = E.gemm_fwd_pair(*args[0], *args[1], epi)
    for i, (x, w, b, gate, res, S) in enumerate(args):
        two_sm_same = min(p0[0], p1[0]) >= 256 or x.shape[0] < 256
        o, s = E.gemm_fwd(x, w, b, epi, gate, res, S)
        if two_sm_same:  # same kernel variant as the single launch: bitwise identical
            assert torch.equal(outs[2 * i], o)
        lin = x.float() @ w.float().t() + b.float()
        if epi == 1:
            ref = lin
        elif epi == 2:
            ref = torch.nn.functional.gelu(lin, approximate="tanh")
        else:
            B = x.shape[0] // S
            ref = res.float() + (lin.view(B, S, -1) * gate.float()[:, None]).view_as(lin)
        assert _rel(outs[2 * i], ref) < 2e-2
        if epi in (2, 3):
            assert _rel(outs[2 * i + 1], lin) < 1e-2


@pytest.mark.parametrize("p0,p1", PAIRS)
def test_gemm_dgrad_wgrad_pair(E, p0, p1):
    torch.manual_seed(6)
    dys, ws, xs, gws = [], [], [], []
    for (M, N, K) in (p0, p1):
        dys.append(torch.randn(M, N, device="cuda").bfloat16())
        ws.append((torch.randn(N, K, device="cuda") / N ** 0.5).bfloat16())
        xs.append(torch.randn(M, K, device="cuda").bfloat16())
        gws.append(torch.randn(N, K, device="cuda"))
    dx0, dx1 = E.gemm_dgrad_pair(dys[0], ws[0], dys[1], ws[1])
    for dx, dy, w in ((dx0, dys[0], ws[0]), (dx1, dys[1], ws[1])):
        assert _rel(dx, dy.float() @ w.float()) < 1e-2
    init = [g.clone() for g in gws]
    E.gemm_wgrad_pair(dys[0], xs[0], gws[0], dys[1], xs[1], gws[1], True)
    for g, g0, dy, x in zip(gws, init, dys, xs):
        assert _rel(g, g0 + dy.float().t() @ x.float()) < 1e-3


def test_linear_pair_autograd_matches_two_linears(E):
    from verl_omni_b200.ops.linear import linear, linear_pair

    torch.manual_seed(7)
    B, Si, St, D = 4, 256, 77 + 3, 512
    mk = lambda *s: torch.randn(*s, device="cuda").bfloat16()
    for epi in ("none", "gelu", "gate_res"):
        x0, x1 = mk(B, Si, D).requires_grad_(), mk(B, St, D).requires_grad_()
        w0, w1 = (mk(2 * D, D) * 0.05).requires_grad_(), (mk(2 * D, D) * 0.05).requires_grad_()
        b0, b1 = mk(2 * D).requires_grad_(), mk(2 * D).requires_grad_()
        g0 = mk(B, 2 * D).requires_grad_() if epi == "gate_res" else None
        g1 = mk(B, 2 * D).requires_grad_() if epi == "gate_res" else None
        r0 = mk(B, Si, 2 * D).requires_grad_() if epi == "gate_res" else None
        r1 = mk(B, St, 2 * D).requires_grad_() if epi == "gate_res" else None
        leaves = [t for t in (x0, x1, w0, w1, b0, b1, g0, g1, r0, r1) if t is not None]
        y0, y1 = linear_pair(x0, w0, b0, x1, w1, b1, epilogue=epi, gate0=g0, res0=r0, S0=Si, gate1=g1, res1=r1,
                             S1=St)
        gy0, gy1 = mk(*y0.shape), mk(*y1.shape)
        gp = torch.autograd.grad((y0 * gy0).sum() + (y1 * gy1).sum(), leaves)
        z0 = linear(x0, w0, b0, epilogue=epi, gate=g0, res=r0, S=Si)
        z1 = linear(x1, w1, b1, epilogue=epi, gate=g1, res=r1, S=St)
        gs = torch.autograd.grad((z0 * gy0).sum() + (z1 * gy1).sum(), leaves)
        assert torch.equal(y0, z0) and torch.equal(y1, z1)
        for a, b in zip(gp, gs):
            assert _rel(a, b) < 1e-2, epi
