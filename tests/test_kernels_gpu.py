"""sm_100a kernel numerics against fp32 torch references of the same op (B200 only)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _ext():
    from verl_omni_b200.ops._ext import ext

    ext()  # fail loudly when the extension is missing on a GPU box


@pytest.mark.parametrize("sde_type", ["sde", "cps", "dance_sde"])
@pytest.mark.parametrize("mode", ["prev", "noise", "seed"])
def test_sde_step_matches_reference(sde_type, mode):
    from verl_omni_b200.ops.sde import philox_normal, sde_step, sde_step_reference

    torch.manual_seed(0)
    B, shape = 5, (16, 24, 24)
    x = torch.randn(B, *shape, device="cuda")
    v = torch.randn(B, *shape, device="cuda")
    sig = torch.tensor([1.0, 0.9, 0.5, 0.3, 0.1], device="cuda")
    sigp = torch.tensor([0.9, 0.7, 0.3, 0.1, 0.05], device="cuda")
    kw = dict(sigma_max=0.95, noise_level=0.7, sde_type=sde_type)
    prev = noise = None
    if mode == "prev":
        prev = torch.randn(B, *shape, device="cuda")
    elif mode == "noise":
        noise = torch.randn(B, *shape, device="cuda")
    seed = 1234
    p, lp, mean, std = sde_step(x, v, sig, sigp, prev_sample=prev, noise=noise, seed=seed if mode == "seed" else None,
                                noise_offset=3, **kw)
    ref_noise = noise
    if mode == "seed":
        ref_noise = philox_normal(seed, B, x[0].numel(), 3).reshape(x.shape).cuda()
    rp, rlp, rmean, rstd = sde_step_reference(x.double(), v.double(), sig.double(), sigp.double(),
                                              prev_sample=None if prev is None else prev.double(),
                                              noise=None if ref_noise is None else ref_noise.double(), **kw)
    torch.testing.assert_close(mean.double(), rmean, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(p.double(), rp, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(std.double(), rstd.double(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lp.double(), rlp, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("sde_type", ["sde", "cps", "dance_sde"])
def test_sde_step_backward(sde_type):
    from verl_omni_b200.ops.sde import sde_step, sde_step_reference

    torch.manual_seed(1)
    B = 3
    x = torch.randn(B, 4, 16, 16, device="cuda")
    v = torch.randn(B, 4, 16, 16, device="cuda", requires_grad=True)
    prev = torch.randn(B, 4, 16, 16, device="cuda")
    sig = torch.tensor([0.9, 0.5, 0.3], device="cuda")
    sigp = torch.tensor([0.7, 0.3, 0.1], device="cuda")
    kw = dict(sigma_max=0.95, noise_level=0.7, sde_type=sde_type, prev_sample=prev)
    _, lp, mean, _ = sde_step(x, v, sig, sigp, **kw)
    gm = torch.randn_like(mean)
    (lp.sum() * 0.3 + (mean * gm).sum()).backward()
    v2 = v.detach().double().requires_grad_(True)
    _, rlp, rmean, _ = sde_step_reference(x.double(), v2, sig.double(), sigp.double(), sigma_max=0.95,
                                          noise_level=0.7, sde_type=sde_type, prev_sample=prev.double())
    (rlp.sum() * 0.3 + (rmean * gm.double()).sum()).backward()
    torch.testing.assert_close(v.grad.double(), v2.grad, rtol=1e-4, atol=1e-5)


def test_ppo_clip_fwd_bwd():
    from verl_omni_b200.ops.losses import ppo_clip_loss, ppo_clip_reference

    torch.manual_seed(0)
    B = 300
    lp = (torch.randn(B, device="cuda") * 0.3).requires_grad_(True)
    old = torch.randn(B, device="cuda") * 0.3
    adv = torch.randn(B, device="cuda")
    w = torch.rand(B, device="cuda")
    loss, st = ppo_clip_loss(lp, old, adv, 0.2, w)
    loss.backward()
    lp2 = lp.detach().clone().requires_grad_(True)
    rl, rst = ppo_clip_reference(lp2, old, adv, 0.2, w)
    rl.backward()
    torch.testing.assert_close(loss, rl, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(torch.stack(list(st.values())), rst, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(lp.grad, lp2.grad, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("shape", [(3, 16, 128, 128), (7, 4), (2, 1 << 20)])
def test_sq_dist_fwd_bwd(shape):
    from verl_omni_b200.ops.losses import _SqDist

    torch.manual_seed(0)
    a = torch.randn(*shape, device="cuda").requires_grad_(True)
    b = torch.randn(*shape, device="cuda").requires_grad_(True)
    d = _SqDist.apply(a, b)
    g = torch.randn_like(d)
    (d * g).sum().backward()
    a2 = a.detach().double().requires_grad_(True)
    b2 = b.detach().double().requires_grad_(True)
    rd = ((a2 - b2) ** 2).flatten(1).mean(1)
    (rd * g.double()).sum().backward()
    torch.testing.assert_close(d.double(), rd, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(a.grad.double(), a2.grad, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(b.grad.double(), b2.grad, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("D", [128, 1536])
def test_affine_layernorm_fwd_bwd(D):
    from verl_omni_b200.ops.norm import layer_norm

    torch.manual_seed(0)
    x = torch.randn(2, 333, D, device="cuda").bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16().requires_grad_(True)
    b = (0.1 * torch.randn(D, device="cuda")).bfloat16().requires_grad_(True)
    y = layer_norm(x, w, b, 1e-6)
    gy = torch.randn_like(y)
    (y.float() * gy.float()).sum().backward()
    x2, w2, b2 = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    y2 = torch.nn.functional.layer_norm(x2, (D,), w2, b2, 1e-6)
    (y2 * gy.float()).sum().backward()
    torch.testing.assert_close(y.float(), y2, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), x2.grad, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(w.grad.float(), w2.grad, rtol=2e-2, atol=0.5)
    torch.testing.assert_close(b.grad.float(), b2.grad, rtol=2e-2, atol=0.5)


@pytest.mark.parametrize("D", [256, 1536])
def test_adaln_layernorm_fwd_bwd(D):
    from verl_omni_b200.ops.norm import adaln_layernorm

    torch.manual_seed(0)
    B, S = 3, 77
    x = torch.randn(B, S, D, device="cuda").bfloat16().requires_grad_(True)
    mod = (torch.randn(B, 6 * D, device="cuda") * 0.5).bfloat16().requires_grad_(True)
    y = adaln_layernorm(x, mod, 3, 4, 6)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr = x.detach().float().requires_grad_(True)
    mr = mod.detach().float().requires_grad_(True)
    m = mr.view(B, 6, D)
    yr = torch.nn.functional.layer_norm(xr, (D,), eps=1e-6) * (1 + m[:, 4, None]) + m[:, 3, None]
    yr.backward(gy.float())
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(mod.grad.float(), mr.grad, rtol=3e-2, atol=0.5)


@pytest.mark.parametrize("dh", [32, 64, 128])
@pytest.mark.parametrize("rope", [False, True])
def test_qk_norm_split_fwd_bwd(dh, rope):
    from verl_omni_b200.models.layers import rope_table
    from verl_omni_b200.ops.norm import qk_norm_split_into

    torch.manual_seed(0)
    B, H, Si, St = 2, 3, 40, 13
    D = H * dh
    S = Si + St
    qkv_i = torch.randn(B * Si, 3 * D, device="cuda").bfloat16().requires_grad_(True)
    qkv_t = torch.randn(B * St, 3 * D, device="cuda").bfloat16().requires_grad_(True)
    wq = (1 + 0.1 * torch.randn(dh, device="cuda")).bfloat16().requires_grad_(True)
    wk = (1 + 0.1 * torch.randn(dh, device="cuda")).bfloat16().requires_grad_(True)
    rp = None
    if rope:
        c, s = rope_table(torch.arange(S), dh)
        rp = (c.cuda(), s.cuda())

    def run(qi, qt, a, b, device, rope_t):
        mk = lambda: torch.empty(B, H, S, dh, device=device, dtype=qi.dtype)  # noqa: E731
        q, k, v = qk_norm_split_into(mk(), mk(), mk(), qi, a, b, Si, 0, rope=rope_t)
        q, k, v = qk_norm_split_into(q, k, v, qt, a, b, St, Si, rope=rope_t)
        return q, k, v

    q, k, v = run(qkv_i, qkv_t, wq, wk, "cuda", rp)
    g = [torch.randn_like(t) for t in (q, k, v)]
    torch.autograd.backward([q, k, v], g)
    leaves = [t.detach().cpu().float().requires_grad_(True) for t in (qkv_i, qkv_t, wq, wk)]
    rq, rk, rv = run(*leaves, "cpu", (rp[0].cpu(), rp[1].cpu()) if rope else None)
    torch.autograd.backward([rq, rk, rv], [t.cpu().float() for t in g])
    for a, b in zip((q, k, v), (rq, rk, rv)):
        torch.testing.assert_close(a.float().cpu(), b, rtol=2e-2, atol=2e-2)
    for a, b in zip((qkv_i, qkv_t), leaves[:2]):
        torch.testing.assert_close(a.grad.float().cpu(), b.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(wq.grad.float().cpu(), leaves[2].grad, rtol=3e-2, atol=0.5)


def test_adamw_matches_torch():
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.workers.engine.base import _adamw_torch

    torch.manual_seed(0)
    n = 100_003
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda") * 3
    m = torch.randn(n, device="cuda").abs() * 0.1
    v = torch.rand(n, device="cuda") * 0.1
    p2, m2, v2 = p.clone(), m.clone(), v.clone()
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    sq = ext().sq_norm(g)
    torch.testing.assert_close(sq, (g.double() ** 2).sum().float().reshape(1), rtol=1e-5, atol=1e-3)
    ext().adamw_flat(p, g, m, v, p16, 1e-3, 0.9, 0.999, 1e-8, 0.01, 7, 1.0, sq, 1.0)
    coef = min(1.0, 1.0 / (float(sq.sqrt()) + 1e-6))
    _adamw_torch(p2, g * coef, m2, v2, 1e-3, 0.9, 0.999, 1e-8, 0.01, 7)
    torch.testing.assert_close(p, p2, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m, m2, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(p16.float(), p2, rtol=1e-2, atol=1e-2)
    before = p.clone()
    bad = torch.tensor([float("inf")], device="cuda")
    ext().adamw_flat(p, g, m, v, p16, 1e-3, 0.9, 0.999, 1e-8, 0.01, 8, 1.0, bad, 1.0)
    assert torch.equal(p, before)
    # views starting one element in (not 16-byte aligned): the scalar kernel takes the whole range
    p3, m3, v3 = p2.clone(), m2.clone(), v2.clone()
    p4, m4, v4 = p2.clone(), m2.clone(), v2.clone()
    ext().adamw_flat(p3[1:], g[1:], m3[1:], v3[1:], p16[1:], 1e-3, 0.9, 0.999, 1e-8, 0.01, 9, 1.0, None, 1.0)
    _adamw_torch(p4[1:], g[1:], m4[1:], v4[1:], 1e-3, 0.9, 0.999, 1e-8, 0.01, 9)
    torch.testing.assert_close(p3, p4, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(v3, v4, rtol=1e-4, atol=1e-6)  # fused multiply-add vs addcmul_ rounding


def test_tiny_mmdit_gpu_matches_cpu():
    from verl_omni_b200.models.mmdit import MMDiT, MMDiTConfig

    torch.manual_seed(0)
    m = MMDiT(MMDiTConfig.tiny())
    x = torch.randn(2, 4, 8, 8)
    t = torch.tensor([900.0, 300.0])
    c = torch.randn(2, 12, 48)
    pooled = torch.randn(2, 32)
    ref = m(x, t, c, pooled)
    mg = m.cuda().bfloat16()
    out = mg(x.cuda(), t.cuda(), c.cuda(), pooled.cuda())
    torch.testing.assert_close(out.cpu(), ref, rtol=5e-2, atol=5e-2)


def test_trainer_step_gpu_sd35_tiny():
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cuda", "actor_rollout_ref.model.architecture=sd35_tiny", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.pipeline.num_inference_steps=4",
        "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.ppo_mini_batch_size=2",
        "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=8", "actor_rollout_ref.actor.use_kl_loss=true",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=2"])
    D.init_distributed(device="cuda")
    t = PolicyGradientTrainer(cfg)
    m1 = t.step()
    m2 = t.step()
    for m in (m1, m2):
        assert math.isfinite(m["actor/grad_norm"]) and math.isfinite(m["actor/pg_loss"])
    assert abs(m1["actor/ppo_kl"]) < 1e-4


def test_row_seeded_noise_matches_cpu_stream():
    """Per-row Philox keys: GPU initial noise and SDE noise equal the CPU oracle and ignore row order."""
    from verl_omni_b200.ops.sde import normal_rows, philox_normal, sde_step, sde_step_reference

    seeds = torch.tensor([5, -7, 123456789012345, 5], dtype=torch.int64)
    z_gpu = normal_rows(seeds, (4, 8, 8), 0x7FFFFFFF, "cuda").cpu()
    z_cpu = normal_rows(seeds, (4, 8, 8), 0x7FFFFFFF, "cpu")
    torch.testing.assert_close(z_gpu, z_cpu, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(z_gpu[0], z_gpu[3])  # same seed, same noise
    B = 4
    x = torch.randn(B, 4, 8, 8, device="cuda")
    v = torch.randn_like(x)
    sig = torch.full((B,), 0.6, device="cuda")
    sigp = torch.full((B,), 0.5, device="cuda")
    prev, lp, mean, std = sde_step(x, v, sig, sigp, sigma_max=0.95, noise_level=0.7, seed=0, noise_offset=3,
                                   row_seeds=seeds)
    z = philox_normal(0, B, 4 * 8 * 8, 3, row_seeds=seeds).reshape(x.shape).cuda()
    ref_prev, _, _, _ = sde_step_reference(x, v, sig, sigp, sigma_max=0.95, noise_level=0.7, sde_type="sde", noise=z)
    torch.testing.assert_close(prev, ref_prev, rtol=1e-4, atol=1e-4)
    perm = torch.tensor([2, 0, 3, 1])
    prev_p, _, _, _ = sde_step(x[perm], v[perm], sig, sigp, sigma_max=0.95, noise_level=0.7, seed=0, noise_offset=3,
                               row_seeds=seeds[perm])
    torch.testing.assert_close(prev_p, prev[perm])


@pytest.mark.parametrize("renorm", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cfg_combine_matches_reference(renorm, dtype):
    from verl_omni_b200.ops.cfg import cfg_combine, cfg_combine_reference

    pos = torch.randn(3, 16, 12, 10, device="cuda").to(dtype)
    neg = torch.randn_like(pos)
    with torch.no_grad():
        out = cfg_combine(pos, neg, 4.5, renorm)
    torch.testing.assert_close(out, cfg_combine_reference(pos, neg, 4.5, renorm), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("silu", [False, True])
@pytest.mark.parametrize("C,H", [(128, 64), (512, 16), (256, 33)])
def test_group_norm_nhwc_matches_reference(C, H, silu):
    from verl_omni_b200.ops.norm import group_norm_act

    torch.manual_seed(0)
    x = (torch.randn(3, C, H, H + 5, device="cuda") * 2 + 0.5).bfloat16().contiguous(memory_format=torch.channels_last)
    w = (1 + 0.1 * torch.randn(C, device="cuda")).bfloat16()
    b = (0.1 * torch.randn(C, device="cuda")).bfloat16()
    with torch.no_grad():
        y = group_norm_act(x, w, b, 32, 1e-6, silu)
    ref = torch.nn.functional.group_norm(x.float(), 32, w.float(), b.float(), 1e-6)
    if silu:
        ref = torch.nn.functional.silu(ref)
    assert y.is_contiguous(memory_format=torch.channels_last)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


def test_qwen_image_gpu_matches_cpu():
    """Qwen-Image-shaped blocks at sizes that take the native paths (grouped image/text GEMMs, split joint
    attention with 256 image rows, head_dim 128) against the fp32 CPU model; then a masked prompt."""
    from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT

    torch.manual_seed(0)
    cfg = QwenImageConfig(in_channels=4, hidden=256, heads=2, depth=2, joint_attention_dim=64)
    m = QwenImageDiT(cfg)
    x = torch.randn(2, 4, 32, 32)
    t = torch.tensor([900.0, 300.0])
    c = torch.randn(2, 128, 64)
    ref = m(x, t, c)
    mask = torch.ones(2, 128)
    mask[1, 100:] = 0
    ref_m = m(x, t, c, mask)
    mg = m.cuda().bfloat16()
    out = mg(x.cuda(), t.cuda(), c.cuda())
    torch.testing.assert_close(out.cpu(), ref, rtol=5e-2, atol=5e-2)
    out_m = mg(x.cuda(), t.cuda(), c.cuda(), mask.cuda())
    torch.testing.assert_close(out_m.cpu(), ref_m, rtol=5e-2, atol=5e-2)
    out_m.square().mean().backward()
    assert all(torch.isfinite(p.grad).all() for p in mg.parameters() if p.grad is not None)


def test_wan_dit_gpu_matches_cpu():
    """Wan-style DiT (self attention, then cross attention whose q-only and k/v-only projections go through
    the q/k-norm split with absent destinations) in bf16 on the native kernels against the fp32 CPU model,
    then a backward pass."""
    from verl_omni_b200.models.dit import DiT, DiTConfig

    torch.manual_seed(0)
    m = DiT(DiTConfig(in_channels=4, out_channels=4, hidden=256, heads=2, depth=2, ffn=512, text_dim=64))
    x = torch.randn(2, 4, 4, 16, 16)
    t = torch.tensor([900.0, 300.0])
    c = torch.randn(2, 64, 64)
    ref = m(x, t, c)
    mg = m.cuda().bfloat16()
    out = mg(x.cuda(), t.cuda(), c.cuda())
    torch.testing.assert_close(out.float().cpu(), ref, rtol=5e-2, atol=5e-2)
    out.float().square().mean().backward()
    assert all(torch.isfinite(p.grad).all() for p in mg.parameters() if p.grad is not None)


def test_peer_row_copy_skips_out_of_range_rows():
    """One GPU, this rank's own buffer as the only peer: rows whose destination rank, destination row or
    source row is out of range are skipped and counted; the others land."""
    from verl_omni_b200.ops._ext import ext

    D, R = 64, 8
    src = torch.randn(5, D, device="cuda").bfloat16()
    dst = torch.zeros(R, D, device="cuda").bfloat16()
    src_idx = torch.tensor([0, 1, 2, 3, 7], dtype=torch.int64, device="cuda")
    dst_rank = torch.tensor([0, 1, 0, 0, 0], dtype=torch.int32, device="cuda")
    dst_row = torch.tensor([2, 3, 5, R + 4, 1], dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext().peer_row_copy(src, src_idx, dst_rank, dst_row, [dst.data_ptr()], R, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 3  # rank 1 absent, row R + 4 past the buffer, source row 7 past src
    exp = torch.zeros_like(dst)
    exp[2], exp[5] = src[0], src[2]
    assert torch.equal(dst, exp)


@pytest.mark.parametrize("V,chunk", [(151936, 32768), (5000, 1024)])
def test_chunked_vocab_logprob_matches_fp32(V, chunk):
    """tcgen05 GEMM chunks + online log-sum-exp kernel against an fp32 log_softmax over bf16 logits; the
    backward's hidden-state gradient and the weight gradient accumulated into main_grad."""
    from verl_omni_b200.ops.vocab_logprob import token_logprobs_from_hidden

    torch.manual_seed(0)
    N, D, T = 384, 256, 0.9
    h = (torch.randn(N, D, device="cuda") * 0.5).bfloat16().requires_grad_(True)
    w = (torch.randn(V, D, device="cuda") * 0.05).bfloat16().requires_grad_(True)
    w.main_grad = torch.zeros(V, D, device="cuda")
    t = torch.randint(0, V, (N,), device="cuda")
    lp = token_logprobs_from_hidden(h, w, t, T, chunk=chunk)
    z = (h.float() @ w.float().t()).bfloat16().float() / T
    ref = torch.log_softmax(z, -1).gather(1, t[:, None])[:, 0]
    torch.testing.assert_close(lp, ref, rtol=1e-3, atol=2e-3)
    g = torch.randn(N, device="cuda")
    (lp * g).sum().backward()
    hr = h.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    rr = torch.log_softmax((hr @ wr.t()) / T, -1).gather(1, t[:, None])[:, 0]
    (rr * g).sum().backward()
    rel = lambda a, b: float((a.float() - b).norm() / (b.norm() + 1e-12))  # noqa: E731
    assert rel(h.grad, hr.grad) < 2e-2
    assert rel(w.main_grad, wr.grad) < 2e-2


def test_llm_row_ops_match_fp32():
    """RMSNorm, SwiGLU, router top-k and per-head q/k RMSNorm + RoPE kernels (forward and backward) against
    fp32 torch."""
    from verl_omni_b200.models.layers import rope_table
    from verl_omni_b200.ops import llm

    torch.manual_seed(0)
    rel = lambda a, b: float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))  # noqa: E731
    # RMSNorm
    x = torch.randn(300, 2048, device="cuda").bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(2048, device="cuda")).bfloat16().requires_grad_(True)
    y = llm.rms_norm(x, w, 1e-6)
    xr, wr = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    assert rel(y, yr) < 1e-2
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    assert rel(x.grad, xr.grad) < 2e-2 and rel(w.grad, wr.grad) < 2e-2
    # SwiGLU
    gu = torch.randn(257, 2 * 768, device="cuda").bfloat16().requires_grad_(True)
    a = llm.swiglu(gu)
    gr = gu.detach().float().requires_grad_(True)
    g_, u_ = gr.chunk(2, -1)
    ar = torch.nn.functional.silu(g_) * u_
    assert rel(a, ar) < 1e-2
    da = torch.randn_like(ar)
    a.backward(da.bfloat16())
    ar.backward(da)
    assert rel(gu.grad, gr.grad) < 2e-2
    # router
    logits = torch.randn(1000, 128, device="cuda", requires_grad=True)
    gates, idx, probs = llm.router_topk(logits, 8)
    lr = logits.detach().clone().requires_grad_(True)
    pr = torch.softmax(lr, -1)
    gv, ir = torch.topk(pr, 8, -1)
    gvr = gv / gv.sum(-1, keepdim=True)
    assert torch.equal(idx, ir)
    torch.testing.assert_close(gates, gvr, rtol=1e-5, atol=1e-6)
    dg = torch.randn_like(gvr)
    gates.backward(dg)
    gvr.backward(dg)
    torch.testing.assert_close(logits.grad, lr.grad, rtol=1e-4, atol=1e-6)
    # per-head norm + RoPE over a column slice of a projection output
    B, S, H, Dh = 2, 77, 4, 128
    proj = torch.randn(B, S, (H + 2) * Dh, device="cuda").bfloat16().requires_grad_(True)
    wn = (1 + 0.1 * torch.randn(Dh, device="cuda")).bfloat16().requires_grad_(True)
    cos, sin = (t.cuda() for t in rope_table(torch.arange(S), Dh, 1e6))
    out = llm.head_norm_rope(proj, Dh, H, wn, cos, sin)
    pr2, wr2 = proj.detach().float().requires_grad_(True), wn.detach().float().requires_grad_(True)
    ref = llm.head_norm_rope_reference(pr2[..., Dh:Dh + H * Dh].reshape(B, S, H, Dh), wr2, cos, sin, 1e-6)
    assert rel(out, ref) < 1e-2
    go = torch.randn_like(ref)
    out.backward(go.bfloat16())
    ref.backward(go)
    assert rel(proj.grad, pr2.grad) < 2e-2 and rel(wn.grad, wr2.grad) < 2e-2


@pytest.mark.parametrize("Dh,H,S", [(64, 3, 45), (128, 5, 33), (256, 2, 19)])
def test_head_norm_rope_vector_kernel_widths(Dh, H, S):
    """The vectorised per-head RMSNorm + RoPE (16-byte lanes, rotate-half partner one shuffle away) at each
    head width, with a head count that leaves the last CTA partly empty; and RMSNorm on the warp-per-row widths
    and the CTA-per-row fallback."""
    from verl_omni_b200.models.layers import rope_table
    from verl_omni_b200.ops import llm

    torch.manual_seed(1)
    rel = lambda a, b: float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))  # noqa: E731
    B = 3
    proj = torch.randn(B, S, (H + 3) * Dh, device="cuda").bfloat16().requires_grad_(True)
    wn = (1 + 0.1 * torch.randn(Dh, device="cuda")).bfloat16().requires_grad_(True)
    cos, sin = (t.cuda() for t in rope_table(torch.arange(S) + 5, Dh, 1e6))
    out = llm.head_norm_rope(proj, 2 * Dh, H, wn, cos, sin)
    pr, wr = proj.detach().float().requires_grad_(True), wn.detach().float().requires_grad_(True)
    ref = llm.head_norm_rope_reference(pr[..., 2 * Dh:(2 + H) * Dh].reshape(B, S, H, Dh), wr, cos, sin, 1e-6)
    assert out.shape == (B, H, S, Dh) and rel(out, ref) < 1e-2
    go = torch.randn_like(ref)
    out.backward(go.bfloat16())
    ref.backward(go)
    assert rel(proj.grad, pr.grad) < 2e-2 and rel(wn.grad, wr.grad) < 2e-2
    for D in (1024, 1536, 2048, 1000):
        x = torch.randn(37, D, device="cuda").bfloat16()
        w = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
        with torch.no_grad():
            y = llm.rms_norm(x, w, 1e-6)
        yr = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
        assert rel(y, yr) < 1e-2, D
