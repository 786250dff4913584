"""Fused linear-backward prologue (gelu'/gate scaling + gate grad + bias grad) vs an fp32 torch oracle."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def E():
    from verl_omni_b200.ops._ext import ext

    return ext()


def _gelu_grad(x):
    k0, k1 = 0.7978845608028654, 0.044715
    t = torch.tanh(k0 * (x + k1 * x ** 3))
    return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * k0 * (1 + 3 * k1 * x * x)


@pytest.mark.parametrize("B,S,N", [(2, 333, 1536), (3, 70, 520), (16, 1357, 64)])
@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("accumulate", [False, True])
def test_linear_bwd_prep(E, B, S, N, mode, accumulate):
    torch.manual_seed(B * N + mode)
    M = B * S
    dy = torch.randn(M, N, device="cuda").bfloat16()
    saved = torch.randn(M, N, device="cuda").bfloat16()
    mod = torch.randn(B, 3 * N, device="cuda").bfloat16()
    gate = mod.view(B, 3, N)[:, 1]  # strided view, as the AdaLN-Zero gate is used
    db = torch.randn(N, device="cuda") if accumulate else torch.zeros(N, device="cuda")
    db0 = db.clone()
    dy2, dg = E.linear_bwd_prep(dy, saved if mode else None, gate if mode == 2 else None, S, mode, db, accumulate)
    f, x = dy.float(), saved.float()
    if mode == 0:
        ref = f
        assert dy2.data_ptr() == dy.data_ptr()
    elif mode == 1:
        ref = f * _gelu_grad(x)
    else:
        ref = (f.view(B, S, N) * gate.float()[:, None]).view(M, N)
        dg_ref = (f.view(B, S, N) * x.view(B, S, N)).sum(1)
        torch.testing.assert_close(dg.float(), dg_ref, rtol=2e-2, atol=2e-2 * S ** 0.5)
    torch.testing.assert_close(dy2.float(), ref, rtol=1e-2, atol=1e-2)
    db_ref = dy2.float().sum(0) + (db0 if accumulate else 0)
    torch.testing.assert_close(db, db_ref, rtol=1e-4, atol=1e-3)


def test_linear_bwd_prep_deterministic(E):
    dy = torch.randn(4 * 1357, 1536, device="cuda").bfloat16()
    saved = torch.randn_like(dy)
    gate = torch.randn(4, 1536, device="cuda").bfloat16()
    outs = []
    for _ in range(2):
        db = torch.zeros(1536, device="cuda")
        _, dg = E.linear_bwd_prep(dy, saved, gate, 1357, 2, db, False)
        outs.append((dg.clone(), db.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
