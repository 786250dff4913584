"""tcgen05 flash attention against an fp32 torch reference."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [(2, 3, 333, 333, 64, False), (1, 2, 1357, 1357, 64, False), (2, 2, 200, 200, 128, False),
         (1, 2, 300, 300, 64, True), (2, 2, 100, 77, 64, False), (1, 1, 1024, 1024, 128, True)]


@pytest.fixture(scope="module")
def E():
    from verl_omni_b200.ops._ext import ext

    e = ext()
    e.fmha_error(True)
    yield e
    assert e.fmha_error(True) == 0, "FMHA kernel reported a barrier timeout"


def _ref(q, k, v, causal, scale):
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    if causal:
        Sq, Sk = s.shape[-2:]
        mask = torch.ones(Sq, Sk, dtype=torch.bool, device=s.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ v.float()
    return o, lse


@pytest.mark.parametrize("version", [1, 2, 3, 4, 5, 7])
@pytest.mark.parametrize("B,H,Sq,Skv,D,causal", CASES)
def test_fmha_fwd(E, B, H, Sq, Skv, D, causal, version):
    torch.manual_seed(0)
    q = torch.randn(B, H, Sq, D, device="cuda").bfloat16()
    k = torch.randn(B, H, Skv, D, device="cuda").bfloat16()
    v = torch.randn(B, H, Skv, D, device="cuda").bfloat16()
    scale = 1 / math.sqrt(D)
    o, lse = E.fmha_fwd(q, k, v, causal, scale, version)
    ro, rlse = _ref(q, k, v, causal, scale)
    torch.testing.assert_close(o.float(), ro.transpose(1, 2), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse, rlse, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("version", [1, 2, 3, 4, 5, 7])
@pytest.mark.parametrize("D", [64, 128])
def test_fmha_fwd_growing_max(E, D, version):
    """Later key blocks carry far larger scores: exercises the running-max rescale of O."""
    torch.manual_seed(3)
    B, H, S = 1, 2, 700
    q = torch.randn(B, H, S, D, device="cuda")
    k = torch.randn(B, H, S, D, device="cuda")
    k[:, :, 260:300] *= 6.0
    k[:, :, 600:640] *= 12.0
    q, k = q.bfloat16(), k.bfloat16()
    v = torch.randn(B, H, S, D, device="cuda").bfloat16()
    scale = 1 / math.sqrt(D)
    o, lse = E.fmha_fwd(q, k, v, False, scale, version)
    ro, rlse = _ref(q, k, v, False, scale)
    torch.testing.assert_close(o.float(), ro.transpose(1, 2), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse, rlse, rtol=1e-3, atol=1e-3)


def test_attention_op_autograd():
    from verl_omni_b200.ops.attention import attention

    torch.manual_seed(1)
    B, H, S, D = 2, 4, 257, 64
    q, k, v = (torch.randn(B, H, S, D, device="cuda").bfloat16().requires_grad_(True) for _ in range(3))
    o = attention(q, k, v)
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    orf = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr).transpose(1, 2).reshape(B, S, H * D)
    orf.backward(g.float())
    torch.testing.assert_close(o.float(), orf, rtol=2e-2, atol=2e-2)
    for a, b in ((q, qr), (k, kr), (v, vr)):
        torch.testing.assert_close(a.grad.float(), b.grad, rtol=5e-2, atol=5e-2)


@pytest.mark.parametrize("version", [1, 2, 3, 4, 5, 7])
@pytest.mark.parametrize("B,H,Sq,Skv,D,causal", CASES)
def test_fmha_bwd(E, B, H, Sq, Skv, D, causal, version):
    torch.manual_seed(2)
    q = torch.randn(B, H, Sq, D, device="cuda").bfloat16()
    k = torch.randn(B, H, Skv, D, device="cuda").bfloat16()
    v = torch.randn(B, H, Skv, D, device="cuda").bfloat16()
    scale = 1 / math.sqrt(D)
    o, lse = E.fmha_fwd(q, k, v, causal, scale)
    do = torch.randn(B, Sq, H, D, device="cuda").bfloat16()
    dq, dk, dv = E.fmha_bwd(q, k, v, o, lse, do, causal, scale, version)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _ref(qr, kr, vr, causal, scale)
    ro.backward(do.float().transpose(1, 2))
    for a, b in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        rel = float((a.float() - b).norm() / (b.norm() + 1e-6))
        assert rel < 2e-2, rel


@pytest.mark.parametrize("fwd,bwd", [(2, 1), (3, 2), (4, 2), (5, 2), (4, 3), (4, 4), (4, 5), (4, 7)])
@pytest.mark.parametrize("D", [64, 128])
def test_attention_split_matches_joint(E, fwd, bwd, D, monkeypatch):
    """Split outputs (image rows / text rows in separate tensors) equal slices of the joint output,
    forward and backward, on the kernel versions the split path uses."""
    import verl_omni_b200.ops.attention as A

    monkeypatch.setattr(A, "_FWD_VERSION", fwd)
    monkeypatch.setattr(A, "_BWD_VERSION", bwd)
    torch.manual_seed(5)
    B, H, Si, St = 2, 3, 256, 77
    q, k, v = (torch.randn(B, H, Si + St, D, device="cuda").bfloat16().requires_grad_(True) for _ in range(3))
    oa, ob = A.attention_split(q, k, v, Si)
    ga, gb = torch.randn_like(oa), torch.randn_like(ob)
    torch.autograd.backward([oa, ob], [ga, gb])
    qr, kr, vr = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    o = A.attention(qr, kr, vr)
    torch.testing.assert_close(oa, o[:, :Si])
    torch.testing.assert_close(ob, o[:, Si:])
    o.backward(torch.cat([ga, gb], 1))
    for a, b in ((q, qr), (k, kr), (v, vr)):
        torch.testing.assert_close(a.grad.float(), b.grad.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("D", [64, 128])
def test_split_attention_with_key_counts_matches_masked_sdpa(D):
    """Right-padded prompts: the tcgen05 forward with per-sequence key counts equals masked SDPA."""
    from verl_omni_b200.ops.attention import attention_split

    torch.manual_seed(0)
    B, H, Si, St = 3, 4, 256, 200
    S = Si + St
    q, k, v = (torch.randn(B, H, S, D, device="cuda").bfloat16() for _ in range(3))
    kv_len = torch.tensor([S, Si + 57, Si + 1], dtype=torch.int32, device="cuda")
    with torch.no_grad():
        oi, ot = attention_split(q, k, v, Si, kv_len=kv_len)
        keep = torch.arange(S, device="cuda")[None, :] < kv_len[:, None].long()
        ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                               attn_mask=keep[:, None, None, :])
        ref = ref.transpose(1, 2).reshape(B, S, H * D)
    torch.testing.assert_close(oi.float(), ref[:, :Si], rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(ot.float(), ref[:, Si:], rtol=2e-2, atol=2e-2)


def test_split_attention_with_key_counts_backward():
    """Gradients of the key-count path equal masked SDPA's; padded keys get zero dK / dV."""
    from verl_omni_b200.ops.attention import attention_split

    torch.manual_seed(1)
    B, H, Si, St, D = 2, 4, 256, 130, 64
    S = Si + St
    base = [torch.randn(B, H, S, D, device="cuda").bfloat16() for _ in range(3)]
    kv_len = torch.tensor([S, Si + 40], dtype=torch.int32, device="cuda")
    g_i, g_t = torch.randn(B, Si, H * D, device="cuda"), torch.randn(B, St, H * D, device="cuda")
    q, k, v = (t.clone().requires_grad_() for t in base)
    oi, ot = attention_split(q, k, v, Si, kv_len=kv_len)
    ((oi.float() * g_i).sum() + (ot.float() * g_t).sum()).backward()
    qr, kr, vr = (t.float().clone().requires_grad_() for t in base)
    keep = torch.arange(S, device="cuda")[None, :] < kv_len[:, None].long()
    ref = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr, attn_mask=keep[:, None, None, :])
    ref = ref.transpose(1, 2).reshape(B, S, H * D)
    ((ref[:, :Si] * g_i).sum() + (ref[:, Si:] * g_t).sum()).backward()
    rel = lambda a, b: float((a.float() - b).norm() / (b.norm() + 1e-6))  # noqa: E731
    for a, b in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert rel(a, b) < 3e-2
    assert float(k.grad[1, :, Si + 40:].abs().max()) == 0.0 and float(v.grad[1, :, Si + 40:].abs().max()) == 0.0


@pytest.mark.parametrize("version", [4, 5])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_fmha_fwd4_key_counts_and_wide_scores(E, D, causal, version):
    """Forward v4 with per-sequence key counts (and the causal mask), scores spanning a wide range so the
    FMA-pipe exponentials see large negative arguments, against the fp32 reference."""
    torch.manual_seed(7)
    B, H, S = 3, 2, 450
    q = (torch.randn(B, H, S, D, device="cuda") * 3).bfloat16()
    k = (torch.randn(B, H, S, D, device="cuda") * 3).bfloat16()
    v = torch.randn(B, H, S, D, device="cuda").bfloat16()
    kv_len = torch.tensor([S, 300, 65], dtype=torch.int32, device="cuda")
    scale = 1 / math.sqrt(D)
    if causal:
        o, lse = E.fmha_fwd(q, k, v, True, scale, version)
        ro, rlse = _ref(q, k, v, True, scale)
        torch.testing.assert_close(o.float(), ro.transpose(1, 2), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(lse, rlse, rtol=1e-3, atol=1e-3)
        return
    o, lse = E.fmha_fwd(q, k, v, False, scale, version, 0, kv_len=kv_len)
    for b in range(B):
        n = int(kv_len[b])
        ro, rlse = _ref(q[b:b + 1], k[b:b + 1, :, :n], v[b:b + 1, :, :n], False, scale)
        torch.testing.assert_close(o[b:b + 1].float(), ro.transpose(1, 2), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(lse[b:b + 1], rlse, rtol=1e-3, atol=1e-3)
