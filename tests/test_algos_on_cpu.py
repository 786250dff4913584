"""CPU oracles for the scheduler, advantage, losses and rollout correction."""

import math
from collections import defaultdict
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from verl_omni_b200.ops.sde import philox_normal, sde_step_reference
from verl_omni_b200.pipelines.schedulers.flow_match_sde import FlowMatchSDEDiscreteScheduler, build_scheduler
from verl_omni_b200.trainer.diffusion import diffusion_algos as algos
from verl_omni_b200.trainer.diffusion.rollout_correction import (
    apply_bypass_mode_to_diffusion_batch, apply_rollout_correction_to_diffusion_batch,
    compute_rollout_corr_metrics_from_logprobs)
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig


def _loop_advantage(scores, index, eps=1e-4, norm=True, global_std=True):
    """Straight per-sample restatement of the GRPO group normalisation."""
    scores = scores.clone()
    id2 = defaultdict(list)
    bstd = torch.std(scores)
    for i in range(scores.shape[0]):
        id2[index[i]].append(scores[i])
    mean, std = {}, {}
    for k, v in id2.items():
        if len(v) == 1:
            mean[k] = v[0]
            std[k] = bstd if global_std else torch.tensor(1.0)
        else:
            st = torch.stack(v)
            mean[k] = st.mean()
            std[k] = bstd if global_std else st.std()
    for i in range(scores.shape[0]):
        scores[i] = (scores[i] - mean[index[i]]) / (std[index[i]] + eps) if norm else scores[i] - mean[index[i]]
    return scores


@pytest.mark.parametrize("global_std", [True, False])
@pytest.mark.parametrize("norm", [True, False])
def test_grpo_advantage_matches_loop(global_std, norm):
    torch.manual_seed(0)
    r = torch.randn(12)
    index = np.array(["a"] * 4 + ["b"] * 4 + ["c"] * 3 + ["d"], dtype=object)
    rew = r[:, None].expand(12, 5).clone()
    adv, ret = algos.compute_flow_grpo_outcome_advantage(rew, index, norm_adv_by_std_in_grpo=norm, global_std=global_std)
    ref = _loop_advantage(rew, index, norm=norm, global_std=global_std)
    torch.testing.assert_close(adv, ref, rtol=1e-5, atol=1e-6)
    assert torch.equal(adv, ret)
    assert algos.get_diffusion_adv_estimator_fn("flow_grpo") is algos.compute_flow_grpo_outcome_advantage


def test_scheduler_sigmas_sd3():
    s = build_scheduler("sd3", 10)
    assert s.sigmas.shape == (11,)
    assert float(s.sigmas[0]) == pytest.approx(1.0)
    assert float(s.sigmas[-1]) == 0.0
    assert torch.all(s.sigmas[:-1] > s.sigmas[1:])
    torch.testing.assert_close(s.timesteps, s.sigmas[:-1] * 1000)


@pytest.mark.parametrize("sde_type", ["sde", "cps", "dance_sde"])
def test_sde_logprob_is_gaussian(sde_type):
    torch.manual_seed(0)
    sch = build_scheduler("sd3", 10)
    x = torch.randn(3, 4, 8, 8)
    v = torch.randn(3, 4, 8, 8)
    out = sch.sample_previous_step(x, v, step_index=3, noise_level=0.7, sde_type=sde_type, seed=123, return_sqrt_dt=True)
    # recompute with the drawn sample => identical log-prob
    out2 = sch.sample_previous_step(x, v, step_index=3, noise_level=0.7, sde_type=sde_type, prev_sample=out.prev_sample)
    torch.testing.assert_close(out.log_prob, out2.log_prob)
    if sde_type != "cps":
        sig, sigp = float(sch.sigmas[3]), float(sch.sigmas[4])
        scale = float(out.std_dev_t.reshape(-1)[0]) * (math.sqrt(sig - sigp) if sde_type == "sde" else 1.0)
        ref = torch.distributions.Normal(out.prev_sample_mean, scale).log_prob(out.prev_sample).mean(dim=(1, 2, 3))
        torch.testing.assert_close(out.log_prob, ref, rtol=1e-4, atol=1e-4)


def test_sde_first_step_sigma_one_uses_sigma_max():
    sch = build_scheduler("sd3", 10)
    x, v = torch.randn(2, 4, 4, 4), torch.randn(2, 4, 4, 4)
    out = sch.sample_previous_step(x, v, step_index=0, noise_level=0.7, sde_type="sde", seed=1)
    sm = float(sch.sigmas[1])
    expect = math.sqrt(1.0 / (1 - sm)) * 0.7
    assert float(out.std_dev_t.reshape(-1)[0]) == pytest.approx(expect, rel=1e-5)
    assert torch.isfinite(out.log_prob).all()


def test_philox_stream_stable_and_normal():
    z = philox_normal(7, 4, 40000, offset=3)
    assert z.shape == (4, 40000)
    assert abs(float(z.mean())) < 0.02 and abs(float(z.std()) - 1.0) < 0.02
    torch.testing.assert_close(z, philox_normal(7, 4, 40000, offset=3))
    assert not torch.allclose(z, philox_normal(7, 4, 40000, offset=4))


def _actor_cfg(**kw):
    c = DiffusionActorConfig()
    for k, v in kw.items():
        setattr(c.diffusion_loss, k, v)
    return c


def test_flow_grpo_loss_values():
    cfg = _actor_cfg(clip_ratio=0.2)
    lp = torch.tensor([0.0, 0.5, -0.5, 0.1], requires_grad=True)
    old = torch.zeros(4)
    adv = torch.tensor([1.0, 1.0, -1.0, -2.0])
    loss, m = algos.FlowGRPOLoss.compute_loss(old_log_prob=old, log_prob=lp, advantages=adv, config=cfg)
    r = torch.exp(lp.detach())
    per = torch.maximum(-adv * r, -adv * r.clamp(0.8, 1.2))
    assert float(loss) == pytest.approx(float(per.mean()), rel=1e-6)
    assert float(m["actor/pg_clipfrac"]) == pytest.approx(0.5)
    loss.backward()
    assert lp.grad is not None


def test_dppo_guard_nft_dpo_kl_run():
    torch.manual_seed(0)
    cfg = _actor_cfg()
    b = 4
    lp, old, adv = torch.randn(b), torch.randn(b), torch.randn(b)
    m1, m0 = torch.randn(b, 4, 8), torch.randn(b, 4, 8)
    std = torch.rand(b, 1, 1) + 0.5
    sqdt = torch.rand(b) + 0.1
    l1, _ = algos.FlowDPPOLoss.compute_loss(old_log_prob=old, log_prob=lp, advantages=adv, config=cfg,
                                            old_prev_sample_mean=m0, prev_sample_mean=m1, std_dev_t=std, sqrt_dt=sqdt)
    l2, _ = algos.GRPOGuardLoss.compute_loss(old_log_prob=old, log_prob=lp, advantages=adv, config=cfg,
                                             old_prev_sample_mean=m0, prev_sample_mean=m1, std_dev_t=std, sqrt_dt=sqdt)
    x = torch.randn(b, 4, 8)
    l3, _ = algos.DiffusionNFTLoss.compute_loss(forward_prediction=x, old_prediction=x + 0.1, ref_forward_prediction=x,
                                                x0=torch.randn(b, 4, 8), xt=torch.randn(b, 4, 8),
                                                t_expanded=torch.rand(b, 1, 1), reward_prob=torch.rand(b), config=cfg)
    rew = torch.tensor([2.0, 1.0, 3.0, 0.0])
    l4, m4 = algos.DPOLoss.compute_loss(torch.randn(b, 4), torch.randn(b, 4), torch.randn(b, 4), torch.randn(b, 4), rew,
                                        cfg, index=np.array(["a", "a", "b", "b"], dtype=object))
    l5, _ = algos.KLLoss.compute_loss(prev_sample_mean=m1, ref_prev_sample_mean=m0, std_dev_t=std)
    for l in (l1, l2, l3, l4, l5):
        assert torch.isfinite(l)
    # KL closed form
    torch.testing.assert_close(l5, (((m1 - m0) ** 2).mean(dim=(1, 2)) / (2 * std.reshape(-1) ** 2)).mean())
    with pytest.raises(ValueError):
        algos.DPOLoss.compute_loss(torch.randn(b, 4), torch.randn(b, 4), torch.randn(b, 4), torch.randn(b, 4),
                                   torch.tensor([0.0, 1.0, 3.0, 0.0]), cfg)


def test_loss_registry_and_validation():
    fn = algos.get_diffusion_loss_fn("flow_grpo")
    with pytest.raises(KeyError, match="old_log_probs"):
        fn.validate_inputs(loss_name="flow_grpo", model_output={"log_probs": 1}, data={"advantages": 1})
    with pytest.raises(ValueError):
        algos.get_diffusion_loss_fn("nope")
    for name in ("flow_grpo", "dance_grpo", "flow_dppo", "grpo_guard", "dpo", "diffusion_nft", "kl", "distill_kl",
                 "distill_fm_mse"):
        assert name in algos.DIFFUSION_LOSS_REGISTRY


def test_online_dpo_pairs_and_nft_prepare():
    uids = np.array(["a", "a", "a", "b", "b", "c"], dtype=object)
    scores = torch.tensor([1.0, 3.0, 2.0, 0.0, 5.0, 1.0])
    assert algos.DPOLoss.build_online_dpo_pair_indices(uids=uids, scores=scores) == [1, 0, 4, 3]
    rp = algos.DiffusionNFTLoss._advantage_to_reward_prob(torch.tensor([-10.0, 0.0, 2.5]), 5.0, "continuous")
    torch.testing.assert_close(rp, torch.tensor([0.0, 0.5, 0.75]))


def test_rollout_correction_modes():
    torch.manual_seed(0)
    old = torch.randn(6, 3) * 0.1
    roll = old + torch.randn(6, 3) * 0.5
    b = DataProto({"old_log_probs": old.clone(), "rollout_log_probs": roll})
    cfg = {"rollout_is": "sequence", "rollout_is_threshold": 2.0, "rollout_rs": "seq_mean_k1",
           "rollout_rs_threshold": "0.5_2.0"}
    b, m = apply_rollout_correction_to_diffusion_batch(b, cfg)
    w = b.batch["rollout_is_weights"]
    assert w.shape == (6, 3) and float(w.max()) <= 2.0
    lr = (old - roll).mean(-1)
    rejected = (lr < math.log(0.5)) | (lr > math.log(2.0))
    assert torch.all(w[rejected] == 0)
    assert "rollout_corr/kl" in m
    b2 = DataProto({"rollout_log_probs": roll})
    apply_bypass_mode_to_diffusion_batch(b2)
    assert torch.equal(b2.batch["old_log_probs"], roll)
    mm = compute_rollout_corr_metrics_from_logprobs(old, roll, timesteps=torch.arange(3).expand(6, 3))
    assert "rollout_corr/logprob_abs_diff/ts_0" in mm


def test_true_cfg_renorm_matches_per_token_norm_form():
    """Channel-axis renorm on [B, C, H, W] equals the reference's last-axis form on packed [B, L, C]."""
    from verl_omni_b200.ops.cfg import cfg_combine

    torch.manual_seed(0)
    pos, neg = torch.randn(2, 8, 4, 5), torch.randn(2, 8, 4, 5)
    out = cfg_combine(pos, neg, 3.0, renorm=True)
    p, n = pos.flatten(2).transpose(1, 2), neg.flatten(2).transpose(1, 2)  # [B, L, C]
    comb = n + 3.0 * (p - n)
    ref = comb * (torch.norm(p, dim=-1, keepdim=True) / torch.norm(comb, dim=-1, keepdim=True))
    torch.testing.assert_close(out.flatten(2).transpose(1, 2), ref)
