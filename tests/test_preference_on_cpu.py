"""Direct-preference trainers on CPU: DiffusionNFT (LoRA old adapter and full-FT EMA copy) and DPO."""

import math

import pytest
import torch

BASE = ["trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.pipeline.num_inference_steps=3",
        "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.ppo_mini_batch_size=2",
        "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4", "trainer.logger=[]", "trainer.resume_mode=disable",
        "actor_rollout_ref.actor.optim.lr=1e-4", "algorithm.trainer_type=direct_preference"]


def _trainer(extra):
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.preference_trainer import DirectPreferenceTrainer
    from verl_omni_b200.utils.config import load_config

    D.init_distributed(device="cpu")
    return DirectPreferenceTrainer(load_config("diffusion_trainer", BASE + extra))


@pytest.mark.parametrize("lora", [True, False])
def test_diffusion_nft_steps(lora):
    extra = ["actor_rollout_ref.model.algorithm=diffusion_nft", "algorithm.old_policy_decay_schedule=linear_to_0_5",
             "algorithm.timestep_fraction=0.67"]
    if lora:
        extra += ["actor_rollout_ref.model.lora_rank=8", "actor_rollout_ref.model.lora_alpha=16",
                  "actor_rollout_ref.model.policy_state_adapters=[default,old]"]
    t = _trainer(extra)
    for _ in range(2):
        m = t.step()
        assert math.isfinite(m["actor/policy_loss"]) and math.isfinite(m["actor/grad_norm"])
    assert 0.0 <= m["actor/reward_prob_mean"] <= 1.0


def test_dpo_online_and_offline():
    from verl_omni_b200.trainer.diffusion.preference_trainer import OfflineDPODataset

    t = _trainer(["actor_rollout_ref.model.algorithm=dpo", "actor_rollout_ref.model.lora_rank=8"])
    m = t.step()
    assert math.isfinite(m["actor/dpo_loss"]) and "actor/implicit_acc" in m
    t.algo_cfg.sample_source = "offline"
    ds = OfflineDPODataset(t, num_pairs=8)
    m2 = t.step(offline_batch=ds.get_batch([0, 1]))
    assert math.isfinite(m2["actor/dpo_loss"])


def test_diffusion_nft_minimax_h3_tiny():
    """DiffusionNFT (the reference's objective for MiniMax-H3) on the packed audio-video model."""
    extra = ["actor_rollout_ref.model.algorithm=diffusion_nft", "algorithm.old_policy_decay_schedule=linear_to_0_5",
             "algorithm.timestep_fraction=0.67"]
    base = [b for b in BASE if not b.startswith("actor_rollout_ref.model.architecture")]
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.preference_trainer import DirectPreferenceTrainer
    from verl_omni_b200.utils.config import load_config

    D.init_distributed(device="cpu")
    t = DirectPreferenceTrainer(load_config("diffusion_trainer", base + extra + [
        "actor_rollout_ref.model.architecture=minimax_h3_tiny"]))
    m = t.step()
    assert math.isfinite(m["actor/policy_loss"]) and math.isfinite(m["actor/grad_norm"])
