"""Agent loops + request-packing rollout server on CPU (tiny DiT)."""

import numpy as np
import pytest
import torch

from verl_omni_b200.utils.config import load_config

OVR = ["trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=4",
       "actor_rollout_ref.rollout.n=3", "actor_rollout_ref.rollout.pipeline.num_inference_steps=4",
       "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.actor.ppo_mini_batch_size=4",
       "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=6", "trainer.logger=[]",
       "trainer.total_training_steps=1", "trainer.resume_mode=disable"]


@pytest.fixture(scope="module")
def trainer():
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer

    torch.manual_seed(0)
    return PolicyGradientTrainer(load_config("diffusion_trainer", OVR))


def _gen_batch(t, ids, step=1, seed=777):
    cond = t.encode_prompts(t.dataset.get_batch(ids))
    cond.non_tensor_batch["uid"] = np.array([f"u{i}" for i in ids], dtype=object)
    gen = cond.repeat(t.n, interleave=True)
    gen.meta_info.update({"global_steps": step, "rollout_seed": seed})
    gen.non_tensor_batch["_rollout_seed_global_idx"] = np.array([i * t.n + j for i in ids for j in range(t.n)])
    return gen


def _manager(t, workers, max_num_seqs):
    from verl_omni_b200.workers.agent_loop import DiffusionAgentLoopManager
    from verl_omni_b200.workers.rollout.server import DiffusionRolloutServer

    srv = DiffusionRolloutServer(t.rollout, max_num_seqs=max_num_seqs)
    return DiffusionAgentLoopManager(srv, t.config.actor_rollout_ref.rollout, t.reward_fn,
                                     cond_keys=tuple(t.adapter.cond_keys()), num_workers=workers), srv


def test_seed_derivation_matches_formula():
    from verl_omni_b200.workers.agent_loop.utils import derive_rollout_seed, maybe_per_rollout_seeds

    assert derive_rollout_seed(5, 3) == 5 * 1_000_003 + 3
    assert maybe_per_rollout_seeds({}, 4) is None
    assert maybe_per_rollout_seeds({"rollout_seed": 2}, 3, [7, 8, 9]) == [2 * 1_000_003 + i for i in (7, 8, 9)]
    with pytest.raises(ValueError):
        maybe_per_rollout_seeds({"rollout_seed": 2}, 3, [1, 2])


def test_packing_and_worker_split_do_not_change_samples(trainer):
    gen = _gen_batch(trainer, [0, 1, 2, 3])
    a_mgr, a_srv = _manager(trainer, workers=1, max_num_seqs=16)
    b_mgr, b_srv = _manager(trainer, workers=3, max_num_seqs=2)
    a = a_mgr.generate_sequences(gen)
    b = b_mgr.generate_sequences(gen)
    assert len(a) == len(b) == 12
    assert b_srv.num_engine_calls > a_srv.num_engine_calls  # different packing really happened
    for k in ("latents", "final_latents", "rollout_log_probs"):
        torch.testing.assert_close(a.batch[k], b.batch[k], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(a.batch["rm_scores"], b.batch["rm_scores"], rtol=1e-5, atol=1e-5)
    # rows of one prompt differ (distinct per-row seeds); same seed -> same sample
    assert not torch.allclose(a.batch["final_latents"][0], a.batch["final_latents"][1])
    assert list(a.non_tensor_batch["uid"][:3]) == ["u0"] * 3
    assert len(a.meta_info["metrics"]) == 12


def test_agent_loop_matches_direct_engine_with_row_seeds(trainer):
    from verl_omni_b200.workers.agent_loop.utils import maybe_per_rollout_seeds

    gen = _gen_batch(trainer, [5, 6])
    mgr, _ = _manager(trainer, workers=2, max_num_seqs=4)
    out = mgr.generate_sequences(gen)
    seeds = torch.tensor(maybe_per_rollout_seeds(gen.meta_info, len(gen), gen.non_tensor_batch["_rollout_seed_global_idx"]))
    direct = trainer.rollout.generate(gen, seed=777, global_step=1, row_seeds=seeds)
    torch.testing.assert_close(out.batch["final_latents"], direct.batch["final_latents"], rtol=1e-5, atol=1e-5)


def test_tq_worker_streams_groups_into_replay_buffer(trainer):
    from verl_omni_b200.trainer.diffusion.v1.replay_buffer import ReplayBuffer
    from verl_omni_b200.workers.agent_loop.tq_agent_loop import DiffusionAgentLoopWorkerTQ
    from verl_omni_b200.workers.rollout.server import DiffusionRolloutServer

    buf = ReplayBuffer(max_off_policy_threshold=2)
    srv = DiffusionRolloutServer(trainer.rollout, max_num_seqs=4)
    w = DiffusionAgentLoopWorkerTQ(srv, trainer.config.actor_rollout_ref.rollout, trainer.reward_fn,
                                   cond_keys=tuple(trainer.adapter.cond_keys()), replay_buffer=buf,
                                   version_fn=lambda: 1)
    try:
        fut = w.submit(_gen_batch(trainer, [0, 1]), n=trainer.n)
        assert fut.result(timeout=300) == 6
        batch, m = buf.sample(global_steps=1, batch_size=2)
        assert len(batch) == 6 and m["training/rollout_failure/evicted_groups"] == 0
    finally:
        w.shutdown()


def test_trainer_step_through_agent_loop():
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer

    torch.manual_seed(0)
    t = PolicyGradientTrainer(load_config("diffusion_trainer", OVR + ["actor_rollout_ref.rollout.agent.enable=true",
                                                                     "actor_rollout_ref.rollout.agent.num_workers=2"]))
    assert t.agent_manager is not None
    m = t.step()
    assert np.isfinite(m["actor/grad_norm"])


def test_stepwise_batching_matches_request_batching():
    """Step-level continuous batching (requests joining while others are mid-trajectory, at most 3 rows per
    forward) reproduces the per-request trajectories and log-probs of whole-batch generation with the same
    per-row seeds."""
    import numpy as np
    import torch

    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config
    from verl_omni_b200.workers.rollout.dit_rollout import StepwiseBatcher

    cfg = load_config("diffusion_trainer", [
        "trainer.device=cpu", "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2",
        "actor_rollout_ref.rollout.n=1", "actor_rollout_ref.rollout.pipeline.num_inference_steps=4",
        "trainer.resume_mode=disable", "trainer.logger=[]"])
    D.init_distributed(device="cpu")
    t = PolicyGradientTrainer(cfg)
    cond = t.encode_prompts(t.dataset.get_batch([0, 1, 2, 3, 4]))
    seeds = torch.tensor([11, 22, 33, 44, 55])
    ref = t.rollout.generate(cond, row_seeds=seeds, decode=False)
    sb = StepwiseBatcher(t.rollout, max_num_seqs=3)
    for i in range(2):  # two requests first, the rest arrive after one iteration
        sb.submit(i, {k: v[i:i + 1] for k, v in cond.batch.items()}, int(seeds[i]))
    sb.step()
    for i in range(2, 5):
        sb.submit(i, {k: v[i:i + 1] for k, v in cond.batch.items()}, int(seeds[i]))
    out = sb.run()
    assert max(sb.rows_per_iteration) == 3 and len(out) == 5
    for i in range(5):
        torch.testing.assert_close(out[i].batch["latents"][0], ref.batch["latents"][i], rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(out[i].batch["rollout_log_probs"][0], ref.batch["rollout_log_probs"][i],
                                   rtol=1e-4, atol=1e-3)
