"""Plumbing config on CPU/gloo, world_size=2: tiny DiT FlowGRPO end to end + checkpoint/resume."""

import json
import os

import pytest
import torch

from tests._dist_util import run_ranks

OVR = ["trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=8",
       "actor_rollout_ref.rollout.n=4", "actor_rollout_ref.rollout.pipeline.num_inference_steps=8",
       "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.use_kl_loss=true",
       "actor_rollout_ref.actor.kl_loss_coef=0.04", "actor_rollout_ref.actor.diffusion_loss.clip_ratio=1e-4",
       "actor_rollout_ref.actor.optim.lr=1e-4", "actor_rollout_ref.actor.ppo_mini_batch_size=8",
       "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=8", "trainer.logger=[]"]


def _train(rank, world, outdir):
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", OVR + [f"trainer.default_local_dir={outdir}", "trainer.total_training_steps=2",
                                                  "trainer.save_freq=2", "trainer.resume_mode=disable"])
    t = PolicyGradientTrainer(cfg)
    hist = t.fit()
    assert len(hist) == 2
    for m in hist:
        assert torch.isfinite(torch.tensor(m["actor/grad_norm"]))
        assert m["perf/total_num_samples"] == 32
    # every rank ends with identical weights (all-gathered bf16/fp32 flat buffer)
    w = t.actor.engine.flat.flat.clone()
    from verl_omni_b200.parallel import dist as D

    ws = D.all_gather_object(w)
    assert torch.equal(ws[0], ws[1])
    if rank == 0:
        with open(os.path.join(outdir, "final.json"), "w") as f:
            json.dump({"sum": float(w.double().sum()), "step": t.global_step}, f)
    # resume into a fresh trainer: weights and step restored
    cfg2 = load_config("diffusion_trainer", OVR + [f"trainer.default_local_dir={outdir}", "trainer.total_training_steps=3",
                                                   "trainer.resume_mode=auto"])
    t2 = PolicyGradientTrainer(cfg2)
    assert t2.maybe_resume()
    assert t2.global_step == 2
    torch.testing.assert_close(t2.actor.engine.flat.master, t.actor.engine.flat.master)
    m = t2.step()
    assert m["training/global_step"] == 3


def test_tiny_flowgrpo_gloo_world2(tmp_path):
    run_ranks(_train, 2, (str(tmp_path),))
    with open(tmp_path / "final.json") as f:
        d = json.load(f)
    assert d["step"] == 2
    assert os.path.exists(tmp_path / "global_step_2" / "actor" / "model_world_size_2_rank_1.pt")
    assert os.path.exists(tmp_path / "global_step_2" / "actor" / "fsdp_config.json")
    assert (tmp_path / "latest_checkpointed_iteration.txt").read_text() == "2"
    # the world-2 checkpoint (flat master slices, no gather at save) re-shards into a world-1 engine
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config
    from verl_omni_b200.workers.engine.base import read_full_state

    state = read_full_state(str(tmp_path / "global_step_2" / "actor"))
    cfg = load_config("diffusion_trainer", OVR + [f"trainer.default_local_dir={tmp_path}", "trainer.resume_mode=auto",
                                                  "trainer.total_training_steps=3"])
    t = PolicyGradientTrainer(cfg)
    assert t.maybe_resume() and t.global_step == 2
    fp = t.actor.engine.flat
    for n, view in fp.param_views(fp.master):
        torch.testing.assert_close(view, state[n].float(), rtol=0, atol=0)
    assert abs(float(fp.flat.double().sum()) - d["sum"]) < 1e-3 * max(1.0, abs(d["sum"]))


def _hsdp(rank, world, outdir):
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", OVR + [f"trainer.default_local_dir={outdir}", "trainer.total_training_steps=1",
                                                  "trainer.save_freq=1", "trainer.resume_mode=disable",
                                                  "actor_rollout_ref.actor.fsdp_config.fsdp_size=2"])
    t = PolicyGradientTrainer(cfg)
    eng = t.actor.engine
    assert eng.world == 2 and eng.n_replicas == 2
    t.fit()
    # every rank (both shard groups, both replicas) ends with identical full weights
    ws = D.all_gather_object(eng.flat.flat.clone())
    for w in ws[1:]:
        assert torch.equal(ws[0], w)


def test_hsdp_world4_fsdp2(tmp_path):
    """HSDP (2 shard groups x 2 replicas) on 4 gloo ranks: replicas stay identical, checkpoint written once."""
    run_ranks(_hsdp, world=4, args=(str(tmp_path),))
    step_dir = [d for d in os.listdir(tmp_path) if d.startswith("global_step")]
    assert step_dir
    actor = os.path.join(tmp_path, step_dir[0], "actor")
    files = sorted(os.listdir(actor))
    assert "model_world_size_2_rank_0.pt" in files and "model_world_size_2_rank_1.pt" in files


def test_validation_pass_with_test_freq():
    """trainer.test_freq runs the validation pass (val_kwargs sampling settings, fixed prompt set) and logs
    val-core / val-aux reward metrics; the pass is deterministic for fixed weights."""
    import torch

    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=3",
        "actor_rollout_ref.actor.ppo_mini_batch_size=2", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=2", "trainer.test_freq=2",
        "data.val_num_prompts=3", "actor_rollout_ref.rollout.val_kwargs.n=2",
        "actor_rollout_ref.rollout.val_kwargs.pipeline.num_inference_steps=4"])
    D.init_distributed(device="cpu")
    t = PolicyGradientTrainer(cfg)
    hist = t.fit()
    assert "val-core/synthetic/reward/mean@2" not in hist[0]
    v = hist[1]["val-core/synthetic/reward/mean@2"]
    assert v == v and "val-aux/synthetic/reward/std@2" in hist[1] and "timing_s/testing" in hist[1]
    again = t.validate()
    assert abs(again["val-core/synthetic/reward/mean@2"] - v) < 1e-6


@pytest.mark.parametrize("mode", ["distill_kl", "distill_fm_mse"])
def test_on_policy_distillation_teacher(mode):
    """distillation.enabled builds a frozen teacher whose reverse-SDE means / velocities feed the distill
    losses; the student's loss picks up the distill term."""
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=2", "actor_rollout_ref.rollout.pipeline.num_inference_steps=3",
        "actor_rollout_ref.actor.ppo_mini_batch_size=2", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=4",
        "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.total_training_steps=1",
        "distillation.enabled=true", "actor_rollout_ref.actor.use_distill_loss=true",
        f"actor_rollout_ref.actor.distill_loss_mode={mode}"])
    D.init_distributed(device="cpu")
    t = PolicyGradientTrainer(cfg)
    assert t.teacher is not None and not any(p.requires_grad for p in t.teacher.module.parameters())
    m = t.step()
    key = "actor/distill_kl_loss" if mode == "distill_kl" else "actor/distill_fm_mse_loss"
    assert m[key] > 0 and "timing_s/teacher" in m


def _veomni(rank, world, outdir):
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", ["diffusion/model_engine=veomni_diffusion"] + OVR + [
        f"trainer.default_local_dir={outdir}", "trainer.total_training_steps=1", "trainer.resume_mode=disable",
        "actor_rollout_ref.actor.veomni_config.fsdp_size=2"])
    assert cfg.model_engine == "veomni_diffusion" and cfg.actor_rollout_ref.actor.strategy == "veomni"
    t = PolicyGradientTrainer(cfg)
    eng = t.actor.engine
    assert eng.world == 2 and eng.n_replicas == 2  # dp_shard 2 x dp_replicate 2
    t.fit()


def test_veomni_engine_selection_world4(tmp_path):
    """``diffusion/model_engine=veomni_diffusion`` picks the VeOmni actor config; its fsdp_size sets the
    dp_shard x dp_replicate layout of the sharded engine."""
    run_ranks(_veomni, world=4, args=(str(tmp_path),))
