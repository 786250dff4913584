"""Grouped-query decode attention over a preallocated KV cache, and the device sampler, against fp32
references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hd,rep,Hk", [(128, 8, 4), (128, 1, 8), (64, 4, 2), (64, 2, 4)])
@pytest.mark.parametrize("splits", [1, 3])
def test_decode_attention_matches_reference(hd, rep, Hk, splits):
    from verl_omni_b200.ops.decode import decode_attention, decode_attention_reference

    torch.manual_seed(0)
    B, Lmax = 3, 700
    q = torch.randn(B, Hk * rep, hd, device="cuda").bfloat16()
    kc = torch.randn(B, Hk, Lmax, hd, device="cuda").bfloat16()
    vc = torch.randn(B, Hk, Lmax, hd, device="cuda").bfloat16()
    lens = torch.tensor([1, 333, 700], dtype=torch.int32, device="cuda")
    out = decode_attention(q, kc, vc, lens, splits=splits)
    ref = decode_attention_reference(q, kc, vc, lens, hd ** -0.5)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("hd,rep,Hk", [(128, 4, 2), (64, 8, 1)])
@pytest.mark.parametrize("splits", [1, 4])
def test_paged_decode_attention_matches_contiguous(hd, rep, Hk, splits):
    """Block-table reads from a shuffled block pool equal the contiguous-cache oracle."""
    from verl_omni_b200.ops.decode import decode_attention, decode_attention_reference, gather_paged

    torch.manual_seed(0)
    B, bs, nb = 3, 16, 120
    lens = torch.tensor([5, 300, 640], dtype=torch.int32, device="cuda")
    width = (int(lens.max()) + bs - 1) // bs
    table = torch.randperm(nb)[:B * width].view(B, width).to(torch.int32).cuda()
    kp = torch.randn(nb, Hk, bs, hd, device="cuda").bfloat16()
    vp = torch.randn(nb, Hk, bs, hd, device="cuda").bfloat16()
    q = torch.randn(B, Hk * rep, hd, device="cuda").bfloat16()
    out = decode_attention(q, kp, vp, lens, splits=splits, block_table=table)
    ref = decode_attention_reference(q, gather_paged(kp, table, lens), gather_paged(vp, table, lens), lens, hd ** -0.5)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_device_sampler_distribution_and_logprobs():
    from verl_omni_b200.ops.decode import sample_tokens

    torch.manual_seed(0)
    logits = torch.randn(4, 50, device="cuda") * 2
    g = torch.Generator(device="cuda").manual_seed(1)
    counts = torch.zeros(4, 50, device="cuda")
    for _ in range(4000):
        ids, lp = sample_tokens(logits, 1.0, 0, 1.0, g)
        counts[torch.arange(4), ids] += 1
    freq = counts / 4000
    torch.testing.assert_close(freq, torch.softmax(logits, -1), rtol=0, atol=0.03)
    torch.testing.assert_close(lp, torch.log_softmax(logits, -1).gather(-1, ids[:, None]).squeeze(-1))
    ids, _ = sample_tokens(logits, 1.0, 5, 1.0, g)  # top-k keeps the 5 largest
    top5 = torch.topk(logits, 5, -1).indices
    assert bool((top5 == ids[:, None]).any(-1).all())


def test_decode_attention_clamps_lengths_and_block_ids():
    """A length beyond the cache reads as the full cache; a paged table id outside the pool reads zeros."""
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.ops.decode import decode_attention_reference

    torch.manual_seed(0)
    B, Hk, rep, hd, Lmax = 2, 2, 4, 64, 96
    q = torch.randn(B, Hk * rep, hd, device="cuda").bfloat16()
    kc = torch.randn(B, Hk, Lmax, hd, device="cuda").bfloat16()
    vc = torch.randn(B, Hk, Lmax, hd, device="cuda").bfloat16()
    too_long = torch.tensor([Lmax + 50, 10 ** 6], dtype=torch.int32, device="cuda")
    full = torch.full((B,), Lmax, dtype=torch.int32, device="cuda")
    out = ext().decode_attention(q, kc, vc, too_long, hd ** -0.5, 2, None)
    ref = decode_attention_reference(q, kc, vc, full, hd ** -0.5)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
    # paged: block 1 of sequence 0 names a block past the pool -> its keys score 0 and its values are 0
    bs, nb = 16, 4
    kp = torch.randn(nb, Hk, bs, hd, device="cuda").bfloat16()
    vp = torch.randn(nb, Hk, bs, hd, device="cuda").bfloat16()
    table = torch.tensor([[0, 999], [2, 3]], dtype=torch.int32, device="cuda")
    lens = torch.tensor([2 * bs, 2 * bs], dtype=torch.int32, device="cuda")
    out = ext().decode_attention(q, kp, vp, lens, hd ** -0.5, 1, table)
    k0 = torch.cat([kp[0], torch.zeros_like(kp[0])], 1)[None]
    v0 = torch.cat([vp[0], torch.zeros_like(vp[0])], 1)[None]
    ref0 = decode_attention_reference(q[:1], k0, v0, lens[:1], hd ** -0.5)
    torch.testing.assert_close(out[:1].float(), ref0.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("rep,Hk", [(8, 4), (16, 2), (1, 8), (4, 1)])
@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("block", [0, 8, 32, 128])
def test_decode_tcgen05_matches_reference(rep, Hk, splits, block):
    """head_dim 128 runs the tcgen05 kernel (TMA tiles, tensor-core QK^T / PV): contiguous and paged caches,
    partial last tiles, empty key splits, zero-length sequences."""
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.ops.decode import decode_attention, decode_attention_reference, gather_paged

    torch.manual_seed(0)
    hd, B = 128, 4
    lens = torch.tensor([1, 129, 700, 0], dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hk * rep, hd, device="cuda").bfloat16()
    if block == 0:
        Lmax = 768
        kc = torch.randn(B, Hk, Lmax, hd, device="cuda").bfloat16()
        vc = torch.randn(B, Hk, Lmax, hd, device="cuda").bfloat16()
        # rows past each length hold non-finite garbage: they must not leak into the result
        for bi, L in enumerate(lens.tolist()):
            vc[bi, :, L:] = float("nan")
            kc[bi, :, L:] = float("inf")
        out = decode_attention(q, kc, vc, lens, splits=splits)
        ref = decode_attention_reference(q, kc, vc, lens, hd ** -0.5)
    else:
        width = (int(lens.max()) + block - 1) // block
        nb = B * width + 3
        table = torch.randperm(nb)[:B * width].view(B, width).to(torch.int32).cuda()
        kp = torch.randn(nb, Hk, block, hd, device="cuda").bfloat16()
        vp = torch.randn(nb, Hk, block, hd, device="cuda").bfloat16()
        out = decode_attention(q, kp, vp, lens, splits=splits, block_table=table)
        ref = decode_attention_reference(q, gather_paged(kp, table, lens), gather_paged(vp, table, lens), lens,
                                         hd ** -0.5)
    assert ext().decode_tc_error(True) == 0
    ref = torch.where(lens[:, None, None] > 0, ref.float(), torch.zeros_like(ref.float()))
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


def test_decode_tcgen05_equals_cuda_core_path(monkeypatch):
    """The tensor-core kernel and the CUDA-core kernel agree, including out-of-pool block ids (zero rows)."""
    from verl_omni_b200.ops._ext import ext

    torch.manual_seed(1)
    B, Hk, rep, hd, bs, nb = 3, 4, 8, 128, 16, 40
    q = torch.randn(B, Hk * rep, hd, device="cuda").bfloat16()
    kp = torch.randn(nb, Hk, bs, hd, device="cuda").bfloat16()
    vp = torch.randn(nb, Hk, bs, hd, device="cuda").bfloat16()
    table = torch.randint(0, nb, (B, 12), dtype=torch.int32, device="cuda")
    table[0, 3] = 9999  # outside the pool: reads as zero keys and values on both paths
    lens = torch.tensor([100, 192, 37], dtype=torch.int32, device="cuda")
    tc = ext().decode_attention(q, kp, vp, lens, hd ** -0.5, 0, table)
    monkeypatch.setenv("VO_DECODE_TC", "0")
    cc = ext().decode_attention(q, kp, vp, lens, hd ** -0.5, 0, table)
    assert ext().decode_tc_error(True) == 0
    torch.testing.assert_close(tc.float(), cc.float(), rtol=2e-2, atol=2e-2)


def test_llm_rollout_cuda_graph_decode_matches_eager(monkeypatch):
    """The thinker's decode step captured once as a CUDA graph and replayed at every position produces the
    same greedy tokens and log-probs as eager steps, and the launch counter advances on replays."""
    from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.utils.dataproto import DataProto
    from verl_omni_b200.workers.rollout.llm_rollout import LLMRolloutEngine

    torch.manual_seed(0)
    cfg = MoEConfig(vocab=2048, hidden=512, layers=2, q_heads=16, kv_heads=2, head_dim=128, experts=8, top_k=2,
                    expert_ffn=256, audio_layers=1, audio_dim=128, audio_mel=16, vision_layers=1, vision_dim=128,
                    vision_patch_dim=48, audio_token=2046, image_token=2047)
    m = MoELLM(cfg).to("cuda", torch.bfloat16).eval()
    ids = torch.randint(0, 2000, (4, 37))
    batch = DataProto({"input_ids": ids}, {})
    eng = LLMRolloutEngine(m, max_new_tokens=12, temperature=0.0, device=torch.device("cuda"))
    monkeypatch.setenv("VO_DECODE_GRAPH", "0")
    n0 = ext().launch_count()
    a = eng.generate(batch, seed=0)
    n_eager = ext().launch_count() - n0
    monkeypatch.setenv("VO_DECODE_GRAPH", "1")
    n0 = ext().launch_count()
    b = eng.generate(batch, seed=0)
    torch.cuda.synchronize()
    assert n_eager > 10 * cfg.layers and ext().launch_count() - n0 == n_eager
    assert torch.equal(a.batch["responses"], b.batch["responses"])
    torch.testing.assert_close(b.batch["rollout_log_probs"], a.batch["rollout_log_probs"], rtol=1e-4, atol=1e-4)
