"""Tensor + sequence parallel linears (Megatron layout) on gloo ranks: a column-parallel -> row-parallel MLP
over TP=2 equals the single-rank MLP in outputs and gradients."""

import torch

from tests._dist_util import run_ranks


def _mlp_check(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.parallel.tensor_parallel import TPContext, column_parallel_linear, row_parallel_linear

    torch.manual_seed(0)
    S, D, Hd = 8, 16, 24
    x = torch.randn(S, D)
    w1, b1 = torch.randn(Hd, D) * 0.2, torch.randn(Hd) * 0.1
    w2, b2 = torch.randn(D, Hd) * 0.2, torch.randn(D) * 0.1
    gy = torch.randn(S, D)
    # single-rank reference
    leaves = [t.clone().requires_grad_() for t in (x, w1, b1, w2, b2)]
    ref = torch.nn.functional.linear(torch.nn.functional.gelu(torch.nn.functional.linear(leaves[0], leaves[1],
                                                                                         leaves[2])), leaves[3], leaves[4])
    (ref * gy).sum().backward()
    # TP = world: rows of the sequence, output columns of w1, input columns of w2
    tp = TPContext(dist.group.WORLD)
    sl, hl = S // world, Hd // world
    xs = x[rank * sl:(rank + 1) * sl].clone().requires_grad_()
    w1s = w1[rank * hl:(rank + 1) * hl].clone().requires_grad_()
    b1s = b1[rank * hl:(rank + 1) * hl].clone().requires_grad_()
    w2s = w2[:, rank * hl:(rank + 1) * hl].clone().requires_grad_()
    b2r = b2.clone().requires_grad_()
    h = torch.nn.functional.gelu(column_parallel_linear(xs, w1s, b1s, tp))  # [S, Hd/world]
    y = row_parallel_linear(h, w2s, b2r, tp)  # [S/world, D]
    torch.testing.assert_close(y, ref[rank * sl:(rank + 1) * sl].detach(), rtol=1e-5, atol=1e-5)
    (y * gy[rank * sl:(rank + 1) * sl]).sum().backward()
    torch.testing.assert_close(xs.grad, leaves[0].grad[rank * sl:(rank + 1) * sl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(w1s.grad, leaves[1].grad[rank * hl:(rank + 1) * hl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(b1s.grad, leaves[2].grad[rank * hl:(rank + 1) * hl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(w2s.grad, leaves[3].grad[:, rank * hl:(rank + 1) * hl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(b2r.grad, leaves[4].grad, rtol=1e-4, atol=1e-5)


def test_tp_mlp_world2_gloo():
    run_ranks(_mlp_check, 2)
