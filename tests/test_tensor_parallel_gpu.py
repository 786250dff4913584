"""Tensor + sequence parallel linears on 2 B200s: both fused paths (all-gather by copy-engine pulls
overlapped with the GEMMs, or inside the GEMM's TMA producer; reduce-scatter inside the GEMM epilogue)
equal the NCCL collective path."""

import pytest
import torch

from tests._dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _run(rank, world):
    import os

    import torch.distributed as dist

    from verl_omni_b200.parallel.tensor_parallel import TPContext, column_parallel_linear, row_parallel_linear

    torch.manual_seed(0)
    S, Dm, Hd = 512, 256, 512
    sl, hl = S // world, Hd // world
    g = torch.Generator().manual_seed(1)
    x = torch.randn(S, Dm, generator=g).cuda().bfloat16()
    w1 = (torch.randn(Hd, Dm, generator=g) * 0.06).cuda().bfloat16()
    b1 = (torch.randn(Hd, generator=g) * 0.1).cuda().bfloat16()
    w2 = (torch.randn(Dm, Hd, generator=g) * 0.04).cuda().bfloat16()
    gy = torch.randn(S, Dm, generator=g).cuda()
    tp = TPContext(dist.group.WORLD)
    res = {}
    for fused in ("0", "1", "kernel"):
        os.environ["VO_TP_FUSED"] = fused
        xs = x[rank * sl:(rank + 1) * sl].clone().requires_grad_()
        w1s = w1[rank * hl:(rank + 1) * hl].clone().requires_grad_()
        b1s = b1[rank * hl:(rank + 1) * hl].clone().requires_grad_()
        w2s = w2[:, rank * hl:(rank + 1) * hl].contiguous().requires_grad_()
        for _ in range(2):  # second pass reuses the alternate buffers
            h = torch.nn.functional.gelu(column_parallel_linear(xs, w1s, b1s, tp))
            y = row_parallel_linear(h.contiguous(), w2s, None, tp)
        (y.float() * gy[rank * sl:(rank + 1) * sl]).sum().backward()
        res[fused] = [t.float().clone() for t in (y, xs.grad, w1s.grad, b1s.grad, w2s.grad)]
    rel = lambda a, b: float((a - b).norm() / (b.norm() + 1e-6))  # noqa: E731
    for mode in ("1", "kernel"):
        for name, a, b in zip(("y", "dx", "dw1", "db1", "dw2"), res[mode], res["0"]):
            assert rel(a, b) < 2e-2, (mode, name, rel(a, b))
    from verl_omni_b200.ops._ext import ext

    assert ext().gemm_error(True) == 0
    tp.release()


def test_tp_fused_matches_nccl_sp2():
    run_ranks(_run, 2, device="cuda")
