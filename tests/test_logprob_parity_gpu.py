"""Rollout vs recomputed log-probs on the native path at the SD3.5-Medium block shape.

The PPO ratio exp(logp - old_logp) is clipped at 1 +- 1e-4 in FlowGRPO, so the log-probs the rollout records
and the ones the trainer recomputes for the same trajectory must agree far inside 1e-4: the rollout and the
trainer run the same adapter, kernels and reduction orders, with different batch compositions (rollout
batches of 6 samples, recompute micro-batches of 2).  Checked with 4 joint blocks of the full width (hidden
1536, 24 heads of 64, 1024 image + 333 text tokens) on the tcgen05 GEMM / FMHA / AdaLN / q-k-norm / SDE
kernels."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_rollout_recompute_logprob_parity_sd35_medium_blocks():
    from verl_omni_b200.models.mmdit import MMDiT, MMDiTConfig
    from verl_omni_b200.models.registry import ARCHS, ArchSpec
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    spec = ARCHS["sd35_medium"]
    ARCHS["sd35_medium_4blk"] = ArchSpec("sd35_medium_4blk", "SD3MMDiT",
                                         lambda: MMDiT(MMDiTConfig(depth=4, dual_attention_layers=2)),
                                         spec.latent_shape, spec.cond_shapes, reward="mlp", image_size=512)
    cfg = load_config("diffusion_trainer", [
        "trainer.device=cuda", "actor_rollout_ref.model.architecture=sd35_medium_4blk", "data.train_batch_size=3",
        "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=4",
        "actor_rollout_ref.rollout.max_num_seqs=6", "actor_rollout_ref.rollout.algo.noise_level=0.7",
        "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=2", "trainer.resume_mode=disable", "trainer.logger=[]"])
    D.init_distributed(device="cuda")
    t = PolicyGradientTrainer(cfg)
    out, _, _ = t.generate(t.local_prompt_ids(t.sampler.next_batch()))
    old = t.actor.infer_batch(out, keys=("log_probs",)).batch["log_probs"]
    roll = out.batch["rollout_log_probs"]
    diff = (old - roll).abs().max().item()
    assert torch.isfinite(old).all() and diff < 1e-5, diff
    ratio = torch.exp(old - roll)
    assert float((ratio - 1).abs().max()) < 1e-4


def test_rollout_and_recompute_are_bitwise_reproducible():
    """Deterministic-mode check on the native path: the same rollout (same seed) twice gives bit-identical
    latents, log-probs and rewards, and the same recompute twice gives bit-identical log-probs (no atomics
    or run-to-run reduction orders in the forward kernels)."""
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cuda", "actor_rollout_ref.model.architecture=sd35_tiny", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.pipeline.num_inference_steps=4",
        "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4",
        "trainer.resume_mode=disable", "trainer.logger=[]"])
    D.init_distributed(device="cuda")
    t = PolicyGradientTrainer(cfg)
    ids = t.local_prompt_ids(t.sampler.next_batch())
    (a, sa, _), (b, sb, _) = t.generate(ids, seed_step=1), t.generate(ids, seed_step=1)
    for k in ("latents", "rollout_log_probs"):
        assert torch.equal(a.batch[k], b.batch[k]), k
    assert torch.equal(sa, sb)
    la = t.actor.infer_batch(a, keys=("log_probs",)).batch["log_probs"]
    lb = t.actor.infer_batch(a, keys=("log_probs",)).batch["log_probs"]
    assert torch.equal(la, lb)
