"""Ulysses sequence parallelism on 2 B200s over NCCL: native-path model sizes, SP=2 vs one rank."""

import pytest
import torch

from tests._dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _run(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT

    torch.manual_seed(0)
    cfg = QwenImageConfig(in_channels=4, hidden=256, heads=4, depth=2, joint_attention_dim=64)
    m = QwenImageDiT(cfg).cuda().bfloat16()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 4, 32, 32, generator=g).cuda()
    t = torch.tensor([900.0, 300.0]).cuda()
    c = torch.randn(2, 256, 64, generator=g).cuda()
    gy = torch.randn(x.shape, generator=torch.Generator().manual_seed(2)).cuda()
    ref = m(x, t, c)
    (ref * gy).sum().backward()
    ref_g = {n: p.grad.float().clone() for n, p in m.named_parameters() if p.grad is not None}
    m.zero_grad(set_to_none=True)
    m.sp_group = dist.group.WORLD
    out = m(x, t, c)
    torch.testing.assert_close(out, ref.detach(), rtol=3e-2, atol=3e-2)
    (out * gy).sum().backward()
    for n, p in m.named_parameters():
        if p.grad is None:
            continue
        gs = p.grad.float().clone()
        dist.all_reduce(gs)
        err = float((gs - ref_g[n]).norm() / (ref_g[n].norm() + 1e-6))
        assert err < 5e-2, (n, err)


def test_qwen_image_ulysses_sp2_nccl():
    run_ranks(_run, 2, device="cuda")
