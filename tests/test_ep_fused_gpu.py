"""Fused expert-parallel exchange (peer row copies around the expert-grouped GEMMs) on 2 B200s equals the
NCCL all-to-all path in outputs and in the gradients of tokens, gates and the local experts' weights."""

import pytest
import torch

from tests._dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _run(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.models.moe_llm import _ffn_grouped
    from verl_omni_b200.parallel.expert_parallel import ExpertParallel, FusedExpertParallel

    E, D, Fh, K = 8, 256, 256, 2
    g = torch.Generator().manual_seed(0)
    wgu0 = (torch.randn(E, 2 * Fh, D, generator=g) / D ** 0.5).cuda().bfloat16()
    wd0 = (torch.randn(E, D, Fh, generator=g) / Fh ** 0.5).cuda().bfloat16()
    g = torch.Generator().manual_seed(10 + rank)
    T = 300 + 37 * rank
    h0 = torch.randn(T, D, generator=g).cuda().bfloat16()
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).cuda()
    gates0 = torch.softmax(torch.randn(T, K, generator=g), -1).cuda().bfloat16()
    gy = torch.randn(T, D, generator=g).cuda()
    res = {}
    fused = FusedExpertParallel(E, dist.group.WORLD)
    for name in ("nccl", "fused"):
        h, gates, wgu, wd = (t.clone().requires_grad_() for t in (h0, gates0, wgu0, wd0))
        if name == "nccl":
            out = ExpertParallel(E, dist.group.WORLD).dispatch_combine(
                h, idx, gates, lambda t, e: _ffn_grouped(t, e, wgu, wd))
        else:
            assert fused.fused_ok(h, wgu, wd)
            out = fused.dispatch_combine_fused(h, idx, gates, wgu, wd)
            out = fused.dispatch_combine_fused(h, idx, gates, wgu, wd)  # second call reuses the buffer pairs
        (out.float() * gy).sum().backward()
        lo, hi = rank * (E // world), (rank + 1) * (E // world)
        res[name] = [out.float(), h.grad.float(), gates.grad.float(), wgu.grad[lo:hi].float(), wd.grad[lo:hi].float()]
    rel = lambda a, b: float((a - b).norm() / (b.norm() + 1e-6))  # noqa: E731
    for nm, a, b in zip(("out", "dh", "dgates", "dw_gate_up", "dw_down"), res["fused"], res["nccl"]):
        assert rel(a, b) < (4e-2 if nm.startswith("dw") else 2e-2), (nm, rel(a, b))
    fused.release()


def test_fused_expert_parallel_matches_nccl_ep2():
    run_ranks(_run, 2, device="cuda")

