"""Ulysses sequence parallelism on 2 B200s over NCCL: native-path model sizes, SP=2 vs one rank."""

import pytest
import torch

from tests._dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _grads(m, x, t, c, gy):
    out = m(x, t, c)
    (out.float() * gy).sum().backward()
    g = {n: p.grad.float().clone() for n, p in m.named_parameters() if p.grad is not None}
    m.zero_grad(set_to_none=True)
    return out.float().detach(), g


def _run(rank, world):
    import copy

    import torch.distributed as dist

    from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT

    torch.manual_seed(0)
    cfg = QwenImageConfig(in_channels=4, hidden=256, heads=4, depth=2, joint_attention_dim=64,
                                          axes_dim=(8, 28, 28))
    m32 = QwenImageDiT(cfg)
    m = copy.deepcopy(m32).cuda().bfloat16()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 4, 32, 32, generator=g)
    t = torch.tensor([900.0, 300.0])
    c = torch.randn(2, 256, 64, generator=g)
    gy = torch.randn(x.shape, generator=torch.Generator().manual_seed(2))
    ref32, g32 = _grads(m32, x, t, c, gy)  # fp32 oracle on the CPU
    g32 = {n: v.cuda() for n, v in g32.items()}
    x, t, c, gy = x.cuda(), t.cuda(), c.cuda(), gy.cuda()
    ref16, g16 = _grads(m, x, t, c, gy)    # bf16 native kernels, one rank
    m.sp_group = dist.group.WORLD
    out, gsp = _grads(m, x, t, c, gy)      # bf16 native kernels, SP=2
    torch.testing.assert_close(out, ref16, rtol=3e-2, atol=3e-2)
    rel = lambda a, b: float((a - b).norm() / (b.norm() + 1e-6))  # noqa: E731
    for n, gs in gsp.items():
        dist.all_reduce(gs)
        if n not in g32:  # discarded last-block text outputs: the grouped GEMM reports zero gradients
            assert float(gs.abs().max()) == 0.0, n
            continue
        e16, esp = rel(g16[n], g32[n]), rel(gs, g32[n])
        # the SP gradient is as close to the fp32 oracle as the one-rank bf16 gradient is
        assert esp <= max(5e-2, 1.5 * e16 + 2e-2), (n, esp, e16)
    from verl_omni_b200.parallel import peer_a2a as PA

    PA.release_all()


def test_qwen_image_ulysses_sp2_nccl():
    run_ranks(_run, 2, device="cuda")


def _run_masked(rank, world):
    """Right-padded prompts under SP: gathered keys reordered image-first, native key-count attention."""
    import torch.distributed as dist

    from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT

    torch.manual_seed(0)
    m = QwenImageDiT(QwenImageConfig(in_channels=4, hidden=256, heads=4, depth=2, joint_attention_dim=64,
                                     axes_dim=(8, 28, 28))).cuda().bfloat16()
    g = torch.Generator().manual_seed(1)
    x, c = torch.randn(2, 4, 32, 32, generator=g).cuda(), torch.randn(2, 256, 64, generator=g).cuda()
    t = torch.tensor([900.0, 300.0]).cuda()
    mask = torch.ones(2, 256, device="cuda")
    mask[0, 150:] = 0
    mask[1, 40:] = 0
    gy = torch.randn(x.shape, generator=torch.Generator().manual_seed(2)).cuda()
    outs, grads = [], []
    for sp in (None, dist.group.WORLD):
        m.sp_group = sp
        out = m(x, t, c, mask)
        (out.float() * gy).sum().backward()
        outs.append(out.float().detach())
        grads.append({n: p.grad.float().clone() for n, p in m.named_parameters() if p.grad is not None})
        m.zero_grad(set_to_none=True)
    torch.testing.assert_close(outs[1], outs[0], rtol=3e-2, atol=3e-2)
    rel = lambda a, b: float((a - b).norm() / (b.norm() + 1e-6))  # noqa: E731
    for n, gs in grads[1].items():
        dist.all_reduce(gs)
        assert rel(gs, grads[0][n]) < 5e-2, (n, rel(gs, grads[0][n]))


def test_qwen_image_ulysses_sp2_padded_prompts_nccl():
    run_ranks(_run_masked, 2, device="cuda")


def _fused(rank, world):
    import os

    import torch.distributed as dist

    from verl_omni_b200.models.dit import DiT, DiTConfig
    from verl_omni_b200.models.mmdit import MMDiT, MMDiTConfig
    from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT
    from verl_omni_b200.parallel import ulysses_fused as UF

    torch.manual_seed(0)  # every rank builds the same weights
    g = torch.Generator().manual_seed(1)
    cases = [
        ("qwen", QwenImageDiT(QwenImageConfig(in_channels=4, hidden=256, heads=4, depth=2, joint_attention_dim=64,
                                          axes_dim=(8, 28, 28))),
         (torch.randn(2, 4, 32, 32, generator=g), torch.tensor([900.0, 300.0]), torch.randn(2, 256, 64, generator=g))),
        ("mmdit", MMDiT(MMDiTConfig(in_channels=4, out_channels=4, hidden=256, heads=4, depth=2, joint_attention_dim=64,
                                    pooled_projection_dim=32, dual_attention_layers=1, sample_size=32,
                                    pos_embed_max_size=32)),
         (torch.randn(2, 4, 32, 32, generator=g), torch.tensor([900.0, 300.0]), torch.randn(2, 256, 64, generator=g),
          torch.randn(2, 32, generator=g))),
        ("wan", DiT(DiTConfig(in_channels=4, out_channels=4, hidden=256, heads=2, depth=2, ffn=512, text_dim=64)),
         (torch.randn(2, 4, 4, 16, 16, generator=g), torch.tensor([900.0, 300.0]), torch.randn(2, 64, 64, generator=g))),
    ]
    for name, m, inputs in cases:
        m = m.cuda().bfloat16().eval()
        inputs = [t.cuda() for t in inputs]
        with torch.no_grad():
            ref = m(*inputs)
            m.sp_group = dist.group.WORLD
            os.environ["VO_ULYSSES_FUSED"] = "0"
            nccl = m(*inputs)
            os.environ["VO_ULYSSES_FUSED"] = "1"
            assert UF.enabled(m.sp_group, torch.empty(1, device="cuda", dtype=torch.bfloat16),
                              4 if name != "wan" else 2, 256)
            fused = m(*inputs)
            fused2 = m(*inputs)  # buffers reused across calls
        torch.testing.assert_close(nccl, ref, rtol=3e-2, atol=3e-2, msg=lambda s: f"{name} nccl: {s}")
        torch.testing.assert_close(fused, nccl, rtol=2e-2, atol=2e-2, msg=lambda s: f"{name} fused: {s}")
        assert torch.equal(fused, fused2), name
        del m.sp_group
    from verl_omni_b200.ops._ext import ext

    assert ext().gemm_error(True) == 0 and ext().fmha_error(True) == 0
    UF.release_all()


def test_ulysses_fused_exchange_matches_nccl_sp2():
    """QKV-GEMM scatter + attention peer output (both exchanges inside kernels) == NCCL all-to-all path."""
    run_ranks(_fused, 2, device="cuda")


def _peer_exchange(rank, world):
    import os

    from verl_omni_b200.parallel import peer_a2a as PA
    from verl_omni_b200.parallel import ulysses as U

    import torch.distributed as dist

    grp = dist.group.WORLD
    torch.manual_seed(10 + rank)
    B, H, Sl, Dh = 2, 8, 40, 64
    xs = [torch.randn(B, H, Sl, Dh, device="cuda").bfloat16().requires_grad_(True) for _ in range(3)]
    o = torch.randn(B, world * Sl, (H // world) * Dh, device="cuda").bfloat16().requires_grad_(True)
    gh = [torch.randn(B, H // world, world * Sl, Dh, device="cuda").bfloat16() for _ in range(3)]
    gt = torch.randn(B, Sl, H * Dh, device="cuda").bfloat16()

    def run(peer: bool):
        os.environ["VO_ULYSSES_PEER"] = "1" if peer else "0"
        assert PA.applies(grp, xs) == peer
        hs = U.seq_to_head_many(xs, grp)
        t = U.head_to_seq(o, grp, Dh)
        loss = sum((h.float() * g.float()).sum() for h, g in zip(hs, gh)) + (t.float() * gt.float()).sum()
        grads = torch.autograd.grad(loss, xs + [o])
        return [h.detach() for h in hs] + [t.detach()] + list(grads)

    ref = run(False)
    for _ in range(3):  # both receive slots, reused
        got = run(True)
        for a, b in zip(got, ref):
            assert torch.equal(a, b)  # pure data movement: bit-exact
    os.environ["VO_ULYSSES_PEER"] = "1"
    PA.release_all()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ulysses_peer_exchange_matches_nccl(world):
    """Sequence <-> head exchanges as one peer-memory kernel each == NCCL all-to-all, forward and backward."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    run_ranks(_peer_exchange, world, device="cuda")
