"""Omni MoE thinker on CPU: KV-cached decode == full forward, grouped experts, GRPO/GSPO/DPO steps, EP=2."""

import copy
import math

import pytest
import torch

from tests._dist_util import run_ranks
from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM, grouped_expert_ffn
from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig


def test_decode_matches_full_forward():
    torch.manual_seed(0)
    m = MoELLM(MoEConfig.tiny())
    ids = torch.randint(0, 500, (2, 7))
    full = m(ids)
    caches = [dict() for _ in m.layers]
    a = m(ids[:, :5], caches=caches, pos0=0)
    b = m(ids[:, 5:6], caches=caches, pos0=5)
    c = m(ids[:, 6:7], caches=caches, pos0=6)
    torch.testing.assert_close(a, full[:, :5], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(b[:, 0], full[:, 5], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(c[:, 0], full[:, 6], rtol=1e-4, atol=1e-4)


def test_paged_cache_decode_matches_full_forward():
    from verl_omni_b200.ops.decode import PagedKVCache

    torch.manual_seed(0)
    m = MoELLM(MoEConfig.tiny())
    cfg = m.cfg
    ids = torch.randint(0, 500, (2, 7))
    full = m(ids)
    caches = []
    for _ in m.layers:
        pool = PagedKVCache(8, cfg.kv_heads, 2, cfg.head_dim, "cpu", torch.float32)
        caches.append(pool.view([pool.add_sequence(), pool.add_sequence()]))
    a = m(ids[:, :5], caches=caches, pos0=0)
    b = m(ids[:, 5:6], caches=caches, pos0=5)
    c = m(ids[:, 6:7], caches=caches, pos0=6)
    torch.testing.assert_close(a, full[:, :5], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(b[:, 0], full[:, 5], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(c[:, 0], full[:, 6], rtol=1e-4, atol=1e-4)


def test_device_position_decode_matches_host_position():
    """One-token steps with the position held in a device tensor (the CUDA-graph decode form) give the same
    logits as steps with the host position."""
    from verl_omni_b200.ops.decode import KVCache

    torch.manual_seed(0)
    m = MoELLM(MoEConfig.tiny())
    cfg = m.cfg
    ids = torch.randint(0, 500, (2, 8))
    mk = lambda: [KVCache(2, cfg.kv_heads, 8, cfg.head_dim, "cpu", torch.float32) for _ in m.layers]
    ca, cb = mk(), mk()
    m(ids[:, :5], caches=ca, pos0=0)
    m(ids[:, :5], caches=cb, pos0=0)
    m.rope(0, 8, "cpu")
    pos = torch.zeros(1, dtype=torch.long)
    for t in range(5, 8):
        a = m(ids[:, t:t + 1], caches=ca, pos0=t)[:, -1]
        pos.fill_(t)
        b = m(ids[:, t:t + 1], caches=cb, pos_t=pos)[:, -1]
        for c in cb:
            c.len = t + 1
        torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
    for x, y in zip(ca, cb):
        torch.testing.assert_close(y.k, x.k)
        torch.testing.assert_close(y.v, x.v)


def test_rollout_paged_cache_same_tokens():
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer

    t = OmniGRPOTrainer(MoEConfig.tiny(), DiffusionActorConfig(), device=torch.device("cpu"), n=1)
    p = t.make_prompts(2, seed=3)
    a = t.rollout.generate(p, seed=1)
    t.rollout.kv_block_size = 4
    b = t.rollout.generate(p, seed=1)
    assert torch.equal(a.batch["responses"], b.batch["responses"])


def test_grouped_experts_match_dense_loop():
    torch.manual_seed(1)
    E, D, F = 4, 8, 6
    wgu, wd = torch.randn(E, 2 * F, D), torch.randn(E, D, F)
    h = torch.randn(10, D)
    idx = torch.randint(0, E, (10, 2))
    gates = torch.rand(10, 2)
    out = grouped_expert_ffn(h, idx, gates, wgu, wd)
    ref = torch.zeros_like(h)
    for t in range(10):
        for k in range(2):
            e = idx[t, k]
            g, u = (wgu[e] @ h[t]).chunk(2)
            ref[t] += gates[t, k] * (wd[e] @ (torch.nn.functional.silu(g) * u))
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("mode", ["grpo", "gspo"])
def test_omni_policy_steps(mode):
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer

    ac = DiffusionActorConfig()
    ac.optim.lr = 1e-3
    t = OmniGRPOTrainer(MoEConfig.tiny(), ac, device=torch.device("cpu"), n=4, loss_mode=mode)
    for _ in range(2):
        m = t.step(num_prompts=2)
        assert math.isfinite(m["actor/pg_loss"]) and math.isfinite(m["actor/grad_norm"])
    # rollout log-probs (KV-cached decode) match the trainer's recompute
    assert m["rollout_corr/logprob_abs_diff_mean"] < 1e-3


def test_omni_dpo_step():
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer

    t = OmniGRPOTrainer(MoEConfig.tiny(), DiffusionActorConfig(), device=torch.device("cpu"), n=1)
    ref = copy.deepcopy(t.model)
    p = t.make_prompts(2, seed=3)
    a = t.rollout.generate(p, seed=1)
    b = t.rollout.generate(p, seed=2)
    m = t.dpo_step(a, b, ref)
    assert math.isfinite(m["dpo_loss"]) and abs(m["dpo_loss"] - math.log(2)) < 1e-3  # policy == reference


def _ep_check(rank, world):
    from verl_omni_b200.parallel.expert_parallel import ExpertParallel
    import torch.distributed as dist

    torch.manual_seed(0)
    E, D, F = 4, 8, 6
    wgu, wd = torch.randn(E, 2 * F, D), torch.randn(E, D, F)
    torch.manual_seed(10 + rank)
    h = torch.randn(6, D, requires_grad=True)
    idx = torch.randint(0, E, (6, 2))
    gates = torch.rand(6, 2)
    ref = grouped_expert_ffn(h.detach(), idx, gates, wgu, wd)
    ep = ExpertParallel(E, dist.group.WORLD)
    from verl_omni_b200.models.moe_llm import _ffn_grouped

    out = ep.dispatch_combine(h, idx, gates, lambda t, e: _ffn_grouped(t, e, wgu, wd))
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    out.sum().backward()
    h2 = h.detach().clone().requires_grad_(True)
    grouped_expert_ffn(h2, idx, gates, wgu, wd).sum().backward()
    torch.testing.assert_close(h.grad, h2.grad, rtol=1e-5, atol=1e-5)


def test_expert_parallel_ep2_gloo():
    run_ranks(_ep_check, 2)


def _ep_decode_check(rank, world):
    from verl_omni_b200.parallel.expert_parallel import ExpertParallel
    import torch.distributed as dist

    torch.manual_seed(0)
    E, D, F = 4, 8, 6
    wgu, wd = torch.randn(E, 2 * F, D), torch.randn(E, D, F)
    torch.manual_seed(10 + rank)
    h = torch.randn(5, D)
    idx = torch.randint(0, E, (5, 2))
    gates = torch.rand(5, 2)
    ref = grouped_expert_ffn(h, idx, gates, wgu, wd)
    ep = ExpertParallel(E, dist.group.WORLD)
    El = E // world
    lo = rank * El
    with torch.no_grad():
        out = ep.decode_combine(h, idx, gates, wgu[lo:lo + El], wd[lo:lo + El], lo)
    # tokens / gates travel as bf16 through the gather: compare with the oracle on the rounded inputs
    ref16 = grouped_expert_ffn(h.bfloat16().float(), idx, gates.bfloat16().float(), wgu, wd)
    torch.testing.assert_close(out, ref16, rtol=1e-4, atol=1e-4)
    assert float((out - ref).abs().max()) < 0.1 * float(ref.abs().max()) + 1e-3


def test_expert_parallel_decode_gather_ep2_gloo():
    """One-token decode steps: tokens all-gathered, local experts, reduce-scatter (no host-synchronised
    variable all-to-all) equals the unsharded expert layer."""
    run_ranks(_ep_decode_check, 2)


def test_chunked_vocab_logprob_matches_full_log_softmax():
    """Chunked log-sum-exp over the vocabulary (chunk not dividing V) equals log_softmax().gather, values and
    gradients of the hidden states and head weight."""
    from verl_omni_b200.ops.vocab_logprob import token_logprobs_from_hidden

    torch.manual_seed(0)
    N, D, V, T = 37, 16, 1000, 0.7
    h = torch.randn(N, D, requires_grad=True)
    w = torch.randn(V, D, requires_grad=True)
    t = torch.randint(0, V, (N,))
    lp = token_logprobs_from_hidden(h, w, t, T, chunk=96)
    ref = torch.log_softmax((h @ w.t()) / T, -1).gather(1, t[:, None])[:, 0]
    torch.testing.assert_close(lp, ref, rtol=1e-5, atol=1e-5)
    g = torch.randn(N)
    gh, gw = torch.autograd.grad((lp * g).sum(), (h, w))
    rh, rw = torch.autograd.grad((ref * g).sum(), (h, w))
    torch.testing.assert_close(gh, rh, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(gw, rw, rtol=1e-4, atol=1e-5)


def _omni_ep_step(rank, world, outdir, ep):
    import torch.distributed as dist

    from verl_omni_b200.models.moe_llm import MoEConfig
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer
    from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig

    ac = DiffusionActorConfig()
    ac.optim.lr = 1e-3
    t = OmniGRPOTrainer(MoEConfig.tiny(), ac, device=torch.device("cpu"), n=4,
                        ep_group=dist.group.WORLD if ep > 1 else None)
    blk = t.model.layers[0]
    m = t.step(num_prompts=2)
    torch.save({"wgu": blk.w_gate_up.detach().clone(), "e0": blk.e0, "loss": m["actor/pg_loss"],
                "n_expert_params": sum(p.numel() for p in t.model.parameters() if getattr(p, "_vo_expert", False)),
                "gn": m["actor/grad_norm"]}, f"{outdir}/ep{ep}_r{rank}.pt")


def test_expert_sharded_grpo_step_matches_unsharded(tmp_path):
    """Two gloo ranks, same data: with EP=2 each rank holds half of every layer's experts (weights, grads,
    optimizer state) and one GRPO step leaves them equal to the matching slices of the replicated-expert
    (data-parallel only) step."""
    run_ranks(_omni_ep_step, 2, (str(tmp_path), 1))
    run_ranks(_omni_ep_step, 2, (str(tmp_path), 2))
    full = torch.load(tmp_path / "ep1_r0.pt")
    E = full["wgu"].shape[0]
    for r in range(2):
        part = torch.load(tmp_path / f"ep2_r{r}.pt")
        assert part["wgu"].shape[0] == E // 2 and part["e0"] == r * E // 2
        assert part["n_expert_params"] > 0
        torch.testing.assert_close(part["wgu"], full["wgu"][r * E // 2:(r + 1) * E // 2], rtol=1e-3, atol=5e-5)


def _main_omni(rank, world, ckpt, steps, par="actor_rollout_ref.actor.megatron.expert_model_parallel_size=2"):
    from verl_omni_b200.trainer.main_omni import run_omni
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("omni_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=qwen3_omni_tiny", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.response_length=6",
        "data.prompt_text_tokens=5", "data.prompt_audio_tokens=3", "data.prompt_image_tokens=3",
        "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=3",
        *((par,) if isinstance(par, str) else tuple(par)), f"trainer.total_training_steps={steps}",
        "trainer.save_freq=1", f"trainer.default_local_dir={ckpt}", "trainer.logger=[]"])
    hist = run_omni(cfg)
    if rank == 0:
        import json

        with open(f"{ckpt}/hist_{steps}.json", "w") as f:
            json.dump([{k: v for k, v in m.items() if isinstance(v, (int, float))} for m in hist], f)


def test_main_omni_ep2_checkpoint_resume(tmp_path):
    """The omni entry point from its config tree on two gloo ranks with EP=2 and micro-batches: one step,
    a checkpoint (dense shards + expert slices), then a resumed run that continues at step 2."""
    import json

    run_ranks(_main_omni, 2, (str(tmp_path), 1))
    assert (tmp_path / "global_step_1" / "actor" / "expert_world_size_2_rank_1.pt").exists()
    run_ranks(_main_omni, 2, (str(tmp_path), 2))
    h1 = json.load(open(tmp_path / "hist_1.json"))
    h2 = json.load(open(tmp_path / "hist_2.json"))
    assert len(h1) == 1 and len(h2) == 1 and h2[0]["training/global_step"] == 2
    assert all(abs(v) < 1e6 for v in h2[0].values())


def test_pipeline_with_expert_parallel_matches_ep_only(tmp_path):
    """4 gloo ranks as 2 pipeline stages x EP=2 (experts sharded inside each stage, expert data-parallel groups
    stage-local): the step equals the 2-rank EP=2 step without stages (losses, norm, every parameter of each
    stage against the same expert shard)."""
    run_ranks(_omni_pp_step, 2, (str(tmp_path), 1, 2))
    run_ranks(_omni_pp_step, 4, (str(tmp_path), 2, 2))
    for r in range(4):
        ref = torch.load(tmp_path / f"pp1_ep2_r{r % 2}.pt")
        part = torch.load(tmp_path / f"pp2_ep2_r{r}.pt")
        for k, v in ref["m"].items():
            assert abs(part["m"][k] - v) <= 1e-5 * max(1.0, abs(v)), (r, k, part["m"][k], v)
        for n, p in part["params"].items():
            torch.testing.assert_close(p, ref["params"][n], rtol=1e-4, atol=1e-6, msg=lambda s: f"{r} {n}: {s}")


def test_main_omni_rollout_tp2(tmp_path):
    """The omni entry point with the rollout decoding tensor-parallel over both ranks: the rollout's log-probs
    agree with the trainer's (replicated-weight) recompute."""
    import json

    run_ranks(_main_omni, 2, (str(tmp_path), 1, "actor_rollout_ref.rollout.tensor_model_parallel_size=2"))
    h1 = json.load(open(tmp_path / "hist_1.json"))
    assert len(h1) == 1 and all(abs(v) < 1e6 for v in h1[0].values())
    assert h1[0]["rollout_corr/logprob_abs_diff_mean"] < 1e-4


def test_main_omni_ep2_hf_export_loads_into_unsharded_thinker(tmp_path):
    """save_contents with hf_model: the EP ranks write disjoint safetensors files (dense tensors once, each
    rank its experts) in the hub layout; together they load strictly into an unsharded thinker and equal the
    trained ranks' weights."""
    from verl_omni_b200.models.hf_omni_io import load_thinker

    run_ranks(_main_omni, 2, (str(tmp_path), 1, ("actor_rollout_ref.actor.megatron.expert_model_parallel_size=2",
                                                 "actor_rollout_ref.actor.checkpoint.save_contents=[model,optimizer,extra,hf_model]")))
    hf_dir = tmp_path / "global_step_1" / "actor" / "huggingface"
    files = sorted(p.name for p in hf_dir.glob("*.safetensors"))
    assert len(files) == 2, files
    m = MoELLM(MoEConfig.tiny())
    n = load_thinker(m, str(hf_dir))
    assert n == len([k for k, _ in m.named_parameters() if not k.startswith(("audio_tower.", "visual."))])
    from safetensors import safe_open

    with safe_open(str(hf_dir / files[1]), framework="pt") as h:  # rank 1: experts 4..7 of every layer
        assert "thinker.model.layers.0.mlp.experts.7.down_proj.weight" in h.keys()
        torch.testing.assert_close(h.get_tensor("thinker.model.layers.0.mlp.experts.7.down_proj.weight").float(),
                                   m.layers[0].w_down[7].float())


def test_main_omni_pp2_checkpoint_resume(tmp_path):
    """The omni entry point with pipeline_model_parallel_size=2: each stage writes its shards under
    ``actor/pp_rank_XX`` and a resumed run continues at step 2."""
    import json

    pp = "actor_rollout_ref.actor.megatron.pipeline_model_parallel_size=2"
    run_ranks(_main_omni, 2, (str(tmp_path), 1, pp))
    for s in range(2):
        assert (tmp_path / "global_step_1" / "actor" / f"pp_rank_{s:02d}" / "model_world_size_1_rank_0.pt").exists()
    run_ranks(_main_omni, 2, (str(tmp_path), 2, pp))
    h2 = json.load(open(tmp_path / "hist_2.json"))
    assert len(h2) == 1 and h2[0]["training/global_step"] == 2
    assert all(abs(v) < 1e6 for v in h2[0].values())


def _pp_check(rank, world, outdir):
    from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM, rms_norm
    from verl_omni_b200.ops.vocab_logprob import token_logprobs_from_hidden
    from verl_omni_b200.parallel.pipeline import PipelineStage

    torch.manual_seed(0)
    cfg = MoEConfig.tiny()
    cfg.layers = 4
    m = MoELLM(cfg)
    M, B, S = 4, 2, 9
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 500, (M, B, S + 1), generator=g)
    cos, sin = m.rope(0, S, ids.device)

    def loss_of(h, i):
        lp = token_logprobs_from_hidden(rms_norm(h, m.norm, cfg.eps), m.lm_head.weight, ids[i, :, 1:])
        return -lp.mean() / M

    # reference: the whole model on this rank
    ref = 0.0
    for i in range(M):
        x = m.embed_tokens(ids[i, :, :-1])
        for blk in m.layers:
            x = blk(x, cos, sin)
        ref_l = loss_of(x, i)
        ref_l.backward()
        ref += float(ref_l)
    ref_g = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
    m.zero_grad(set_to_none=True)
    # two stages: layers [0, 2) with the embedding on rank 0, layers [2, 4) with the head on rank 1
    lo, hi = (0, 2) if rank == 0 else (2, 4)

    def fn(x, i):
        if rank == 0:
            x = m.embed_tokens(ids[i, :, :-1])
        for blk in m.layers[lo:hi]:
            x = blk(x, cos, sin)
        return loss_of(x, i) if rank == 1 else x

    st = PipelineStage(fn, rank, 2, [0, 1], (B, S, cfg.hidden), (B, S, cfg.hidden), torch.float32,
                       torch.device("cpu"))
    losses = st.run(M)
    for n, p in m.named_parameters():
        if p.grad is not None:
            torch.testing.assert_close(p.grad, ref_g[n], rtol=1e-4, atol=1e-6, msg=lambda s: f"{n}: {s}")
    if rank == 1:
        assert abs(sum(float(x) for x in losses) - ref) < 1e-5


def test_pipeline_1f1b_two_stages_match_single_rank():
    """1F1B over 2 gloo stages (4 micro-batches) gives the single-rank loss and every parameter's gradient."""
    run_ranks(_pp_check, 2, ("",))


def _omni_pp_step(rank, world, outdir, pp, ep=1):
    import torch.distributed as dist

    from verl_omni_b200.models.moe_llm import MoEConfig
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer
    from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig

    ac = DiffusionActorConfig()
    ac.optim.lr = 1e-3
    cfg = MoEConfig.tiny()
    cfg.layers = 3
    ep_group = None
    if ep > 1:
        from verl_omni_b200.parallel import dist as D

        ep_group = D.make_hsdp_groups(ep)[0]
    t = OmniGRPOTrainer(cfg, ac, device=torch.device("cpu"), n=4, response_len=5, micro_batch_size=3,
                        pp_size=pp, ep_group=ep_group)
    m = t.step(num_prompts=2)
    out = {"m": {k: m[k] for k in ("actor/pg_loss", "actor/grad_norm", "critic/rewards/mean",
                                   "rollout_corr/logprob_abs_diff_mean")},
           "params": {f"{n}" if pp == 1 else _full_name(n, t.model): p.detach().clone()
                      for n, p in t.model.named_parameters()}}
    torch.save(out, f"{outdir}/pp{pp}_ep{ep}_r{rank}.pt")


def _full_name(n, stage):
    if n.startswith("layers."):
        i, rest = n.split(".", 2)[1:]
        return f"layers.{int(i) + stage.lo}.{rest}"
    return n


def test_pipeline_parallel_grpo_step_matches_single_rank(tmp_path):
    """The omni GRPO step with the model split into 2 pipeline stages (gloo ranks: layers [0, 2) + embedding
    and towers, layer 2 + head): pipelined decode, forward-only old log-probs, 1F1B update over uneven
    micro-batches (3 + 3 + 2 sequences) and the cross-stage gradient norm give the single-rank step's
    losses, norm and updated parameters."""
    run_ranks(_omni_pp_step, 1, (str(tmp_path), 1))
    run_ranks(_omni_pp_step, 2, (str(tmp_path), 2))
    ref = torch.load(tmp_path / "pp1_ep1_r0.pt")
    seen = set()
    for r in range(2):
        part = torch.load(tmp_path / f"pp2_ep1_r{r}.pt")
        for k, v in ref["m"].items():
            assert abs(part["m"][k] - v) <= 1e-5 * max(1.0, abs(v)), (k, part["m"][k], v)
        for n, p in part["params"].items():
            torch.testing.assert_close(p, ref["params"][n], rtol=1e-4, atol=1e-6, msg=lambda s: f"{n}: {s}")
            seen.add(n)
    assert seen == set(ref["params"])


def _tp_rollout_check(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.parallel.tensor_parallel import TPContext
    from verl_omni_b200.utils.dataproto import DataProto
    from verl_omni_b200.workers.rollout.llm_rollout import LLMRolloutEngine

    torch.manual_seed(0)
    cfg = MoEConfig.tiny()
    m = MoELLM(cfg)
    g = torch.Generator().manual_seed(100 + rank)
    n, P = 3, 6
    ids = torch.cat([torch.randint(0, 500, (n, P - 2), generator=g), torch.full((n, 1), cfg.audio_token),
                     torch.full((n, 1), cfg.image_token)], 1)
    batch = DataProto({"input_ids": ids, "audio_feats": torch.randn(n, 1, cfg.audio_mel, generator=g),
                       "image_patches": torch.randn(n, 1, cfg.vision_patch_dim, generator=g)}, {})
    tp = LLMRolloutEngine(m, max_new_tokens=5, temperature=0.0, device=torch.device("cpu"),
                          tp=TPContext(dist.group.WORLD))
    ref = LLMRolloutEngine(m, max_new_tokens=5, temperature=0.0, device=torch.device("cpu"))
    a, b = tp.generate(batch, seed=1), ref.generate(batch, seed=1)
    assert torch.equal(a.batch["responses"], b.batch["responses"])
    assert torch.equal(a.batch["prompts"], ids)
    torch.testing.assert_close(a.batch["rollout_log_probs"], b.batch["rollout_log_probs"], rtol=1e-4, atol=1e-5)
    # sampled decode: both ranks of the group draw the same tokens for the group's whole batch
    import verl_omni_b200.workers.rollout.llm_rollout as LR

    drawn, orig = [], LR.sample_tokens

    def rec(*a, **k):
        out = orig(*a, **k)
        drawn.append(out[0].clone())
        return out

    LR.sample_tokens = rec
    try:
        tp.temperature = 1.0
        tp.generate(batch, seed=3)
    finally:
        LR.sample_tokens = orig
    mine = torch.stack(drawn)  # [steps, group batch]
    both = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(both, mine)
    assert mine.shape[1] == world * n and torch.equal(both[0], both[1])


def test_tensor_parallel_rollout_tp2_gloo():
    """Rollout decode with attention heads (and KV caches) split over a TP=2 group: greedy tokens and log-probs
    equal the replicated-weight decode of the same prompts."""
    run_ranks(_tp_rollout_check, 2)


def _main_omni_parquet(rank, world, root):
    from verl_omni_b200.trainer.main_omni import run_omni
    from verl_omni_b200.utils.config import load_config

    for name in ("with_feats", "text_only"):
        cfg = load_config("omni_trainer", [
            "trainer.device=cpu", "actor_rollout_ref.model.architecture=qwen3_omni_tiny", "data.train_batch_size=2",
            "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.response_length=4",
            f"data.train_files={root}/{name}.parquet", "data.max_prompt_length=10", "trainer.total_training_steps=1",
            "trainer.save_freq=0", f"trainer.default_local_dir={root}/ck_{name}", "trainer.logger=[]"])
        hist = run_omni(cfg)
        assert len(hist) == 1 and hist[0]["actor/grad_norm"] == hist[0]["actor/grad_norm"]


def test_main_omni_reads_parquet_prompts(tmp_path):
    """data.train_files: omni prompts from parquet (token ids with audio / image placeholders and their
    feature arrays, or plain text), left-padded to max_prompt_length, through the entry point on 2 gloo ranks."""
    import pandas as pd

    from verl_omni_b200.utils.datasets_parquet import ParquetOmniRLDataset

    cfg = MoEConfig.tiny()
    rows = []
    for i in range(5):
        rows.append({"prompt_ids": [3 + i, 7, cfg.audio_token, cfg.audio_token, cfg.image_token],
                     "audio_feats": torch.randn(2, cfg.audio_mel).tolist(),
                     "image_patches": torch.randn(1, cfg.vision_patch_dim).tolist(), "data_source": "synthetic"})
    pd.DataFrame(rows).to_parquet(tmp_path / "with_feats.parquet")
    pd.DataFrame([{"prompt": f"describe sound number {i}"} for i in range(3)]).to_parquet(tmp_path / "text_only.parquet")
    ds = ParquetOmniRLDataset(str(tmp_path / "with_feats.parquet"), vocab=cfg.vocab, max_prompt_length=8)
    b = ds.get_batch([4, 5])  # index 5 wraps to row 0
    assert b.batch["input_ids"].shape == (2, 8) and b.batch["audio_feats"].shape == (2, 2, cfg.audio_mel)
    assert b.batch["input_ids"][0, :3].tolist() == [0, 0, 0] and b.batch["input_ids"][1, 3].item() == 3
    run_ranks(_main_omni_parquet, 2, (str(tmp_path),))


def _main_omni_dpo(rank, world, root, steps):
    import json

    from verl_omni_b200.trainer.main_omni import run_omni
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("omni_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=qwen3_omni_tiny", "data.train_batch_size=4",
        "algorithm.trainer_type=direct_preference", "algorithm.dpo_beta=0.2", f"data.train_files={root}/pairs.parquet",
        "actor_rollout_ref.actor.megatron.expert_model_parallel_size=2", "actor_rollout_ref.actor.optim.lr=1e-3",
        f"trainer.total_training_steps={steps}", "trainer.save_freq=1", f"trainer.default_local_dir={root}/ck",
        "trainer.logger=[]"])
    hist = run_omni(cfg)
    if rank == 0:
        with open(f"{root}/dpo_{steps}.json", "w") as f:
            json.dump(hist, f)


def test_main_omni_offline_dpo_ep2_and_resume(tmp_path):
    """algorithm.trainer_type=direct_preference: offline omni DPO from parquet pairs through the entry point on 2
    gloo ranks with EP=2; the first step sits at log 2 (policy == frozen reference), a resumed run continues."""
    import json

    import pandas as pd

    cfg = MoEConfig.tiny()
    g = torch.Generator().manual_seed(0)
    rows = [{"prompt_ids": torch.randint(0, 500, (6,), generator=g).tolist(),
             "chosen_ids": torch.randint(0, 500, (4,), generator=g).tolist(),
             "rejected_ids": torch.randint(0, 500, (3 + i % 2,), generator=g).tolist()} for i in range(8)]
    pd.DataFrame(rows).to_parquet(tmp_path / "pairs.parquet")
    run_ranks(_main_omni_dpo, 2, (str(tmp_path), 2))
    h = json.load(open(tmp_path / "dpo_2.json"))
    assert len(h) == 2 and abs(h[0]["dpo_loss"] - math.log(2)) < 1e-4
    assert abs(h[1]["dpo_loss"] - math.log(2)) > 1e-6  # the first update moved the policy off the reference
    run_ranks(_main_omni_dpo, 2, (str(tmp_path), 3))
    h3 = json.load(open(tmp_path / "dpo_3.json"))
    assert len(h3) == 1 and h3[0]["training/global_step"] == 3
