"""Expert-grouped tcgen05 GEMMs (forward / dgrad / weight gradient) and the MoE SwiGLU layer on them,
against fp32 torch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-6))


@pytest.fixture(scope="module")
def E_():
    from verl_omni_b200.ops._ext import ext

    e = ext()
    e.gemm_error(True)
    yield e
    assert e.gemm_error(True) == 0


def _layout(E, counts, dev="cuda"):
    """Padded expert segments for given per-expert row counts -> (seg int32 [E+1], tile_expert, rows)."""
    padded = [(c + 127) // 128 * 128 for c in counts]
    seg = torch.tensor([0] + list(torch.tensor(padded).cumsum(0).tolist()), dtype=torch.int32)
    rows = int(seg[-1]) + 256  # two unused tiles at the end
    te = []
    for t in range(rows // 128):
        r = t * 128
        e = -1
        for i in range(E):
            if seg[i] <= r < seg[i + 1]:
                e = i
        te.append(e)
    return seg.to(dev), torch.tensor(te, dtype=torch.int32, device=dev), rows


def test_moe_gemm_fwd_dgrad_wgrad(E_):
    torch.manual_seed(0)
    E, N, K = 6, 512, 384
    counts = [130, 0, 256, 1, 77, 300]
    seg, te, rows = _layout(E, counts)
    x = torch.zeros(rows, K, device="cuda")
    dy = torch.zeros(rows, N, device="cuda")
    for e in range(E):  # zero padding rows, as the dispatch leaves them
        s = int(seg[e])
        x[s:s + counts[e]] = torch.randn(counts[e], K, device="cuda")
        dy[s:s + counts[e]] = torch.randn(counts[e], N, device="cuda")
    x, dy = x.bfloat16(), dy.bfloat16()
    w = (torch.randn(E, N, K, device="cuda") / K ** 0.5).bfloat16()
    y = E_.moe_gemm_fwd(x, w, te)
    dx = E_.moe_gemm_dgrad(dy, w, te)
    gw = torch.randn(E, N, K, device="cuda")
    g0 = gw.clone()
    E_.moe_gemm_wgrad(dy, x, seg, gw, True)
    for e in range(E):
        s, c = int(seg[e]), counts[e]
        if c == 0:
            assert torch.equal(gw[e], g0[e])
            continue
        assert _rel(y[s:s + c], x[s:s + c].float() @ w[e].float().t()) < 1e-2
        assert _rel(dx[s:s + c], dy[s:s + c].float() @ w[e].float()) < 1e-2
        assert _rel(gw[e], g0[e] + dy[s:s + c].float().t() @ x[s:s + c].float()) < 1e-3


def test_moe_layer_forward_backward_matches_loop(E_):
    from verl_omni_b200.ops.moe import moe_ffn, moe_ffn_reference

    torch.manual_seed(1)
    T, K, E, D, Fh = 300, 2, 8, 256, 256
    h = torch.randn(T, D, device="cuda").bfloat16().requires_grad_()
    idx = torch.stack([torch.randperm(E)[:K] for _ in range(T)]).cuda()
    gates = torch.softmax(torch.randn(T, K, device="cuda"), -1).bfloat16().requires_grad_()
    wgu = (torch.randn(E, 2 * Fh, D, device="cuda") / D ** 0.5).bfloat16().requires_grad_()
    wd = (torch.randn(E, D, Fh, device="cuda") / Fh ** 0.5).bfloat16().requires_grad_()
    out = moe_ffn(h, idx, gates, wgu, wd)
    leaves = [t.detach().float().requires_grad_() for t in (h, gates, wgu, wd)]
    ref = moe_ffn_reference(leaves[0], idx, leaves[1], leaves[2], leaves[3])
    assert _rel(out, ref) < 2e-2
    gy = torch.randn(T, D, device="cuda")
    g_nat = torch.autograd.grad((out.float() * gy).sum(), [h, gates, wgu, wd])
    g_ref = torch.autograd.grad((ref * gy).sum(), leaves)
    for a, b, name in zip(g_nat, g_ref, ("h", "gates", "w_gate_up", "w_down")):
        assert _rel(a, b) < 3e-2, name


def test_moe_ffn_local_experts_only(E_):
    """This rank's experts' contribution with the other slots dropped on the device (sink tiles skipped by the
    grouped GEMM) equals the fp32 oracle restricted to those experts."""
    from verl_omni_b200.ops.moe import moe_ffn_local, moe_ffn_local_reference

    torch.manual_seed(0)
    E, El, e0, D, F, T, K = 16, 4, 8, 256, 128, 96, 4
    h = (torch.randn(T, D, device="cuda") * 0.5).bfloat16()
    idx = torch.randint(0, E, (T, K), device="cuda")
    gates = torch.rand(T, K, device="cuda")
    wgu = (torch.randn(El, 2 * F, D, device="cuda") * 0.05).bfloat16()
    wd = (torch.randn(El, D, F, device="cuda") * 0.05).bfloat16()
    with torch.no_grad():
        out = moe_ffn_local(h, idx, gates, wgu, wd, e0)
    ref = moe_ffn_local_reference(h, idx, gates, wgu, wd, e0)
    assert torch.isfinite(out).all()
    assert _rel(out, ref) < 2e-2
