"""Host offload in the sharded engine: with ``optimizer_offload`` the fp32 master shard and AdamW moments live in
pinned host memory between updates, with ``param_offload`` the fp32 gradient buffer is released between updates
and the frozen reference model waits on the host; two FlowGRPO steps (KL against the reference) give the same
losses and norms as the resident run."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(offload: bool):
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    flag = "true" if offload else "false"
    cfg = load_config("diffusion_trainer", [
        "trainer.device=cuda", "actor_rollout_ref.model.architecture=sd35_tiny", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.pipeline.num_inference_steps=4",
        "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.ppo_mini_batch_size=2",
        "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=8", "actor_rollout_ref.actor.use_kl_loss=true",
        f"actor_rollout_ref.actor.fsdp_config.param_offload={flag}",
        f"actor_rollout_ref.actor.fsdp_config.optimizer_offload={flag}",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=2"])
    t = PolicyGradientTrainer(cfg)
    hist = [t.step(), t.step()]
    return t, hist


def test_optimizer_and_param_offload_match_resident():
    from verl_omni_b200.parallel import dist as D

    D.init_distributed(device="cuda")
    _, ref = _run(False)
    t, off = _run(True)
    fp = t.actor.engine.flat
    assert not fp.master.is_cuda and fp.master.is_pinned() and not fp.exp_avg.is_cuda
    assert fp.main_grad is None
    assert t.ref is not None and all(not p.is_cuda for p in t.ref.module.parameters())
    for a, b in zip(ref, off):
        for k in ("actor/pg_loss", "actor/grad_norm", "actor/ppo_kl"):
            assert math.isfinite(b[k])
            assert abs(a[k] - b[k]) <= 1e-5 * max(1.0, abs(a[k])), (k, a[k], b[k])
