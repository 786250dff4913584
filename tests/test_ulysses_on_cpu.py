"""Ulysses all-to-all on gloo ranks: SP attention == full attention (forward and gradients)."""

import torch

from tests._dist_util import run_ranks


def _check(rank, world):
    from verl_omni_b200.parallel import ulysses as U
    from verl_omni_b200.parallel import dist as D
    import torch.distributed as dist

    group = dist.group.WORLD
    torch.manual_seed(0)
    B, H, S, Dh = 2, 4, 12, 8
    q, k, v = (torch.randn(B, H, S, Dh) for _ in range(3))
    g = torch.randn(B, S, H * Dh)
    # reference on the full sequence
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr).transpose(1, 2).reshape(B, S, H * Dh)
    ref.backward(g)
    # SP: this rank holds tokens [r*S/sp, (r+1)*S/sp)
    sl = slice(rank * S // world, (rank + 1) * S // world)
    ql, kl, vl = (t[:, :, sl].clone().requires_grad_(True) for t in (q, k, v))
    out = U.ulysses_attention(ql, kl, vl, group)
    torch.testing.assert_close(out, ref[:, sl].detach(), rtol=1e-5, atol=1e-5)
    out.backward(g[:, sl])
    for a, b in ((ql, qr), (kl, kr), (vl, vr)):
        torch.testing.assert_close(a.grad, b.grad[:, :, sl], rtol=1e-5, atol=1e-5)
    # gather / shard round trip with gradient slicing
    x = torch.randn(B, S // world, 3, requires_grad=True)
    y = U.gather_sequence(x, group)
    assert y.shape == (B, S, 3)
    y.sum().backward()
    assert torch.equal(x.grad, torch.ones_like(x))


def test_ulysses_sp2_gloo():
    run_ranks(_check, 2)
