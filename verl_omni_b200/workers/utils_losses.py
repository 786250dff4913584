"""Worker-side loss composition (``verl_omni/workers/utils/losses.py:26-153``).

``diffusion_loss`` picks the policy loss by ``loss_mode``; applies bypass-mode rejection
sampling per SDE step; adds ``kl_loss_coef * KL(ref)`` and ``distill_loss_coef * distill``;
divides by the gradient-accumulation count (micro-batches x timesteps) and multiplies by the
Ulysses degree (each SP rank back-propagates the full loss of its sequence shard).
"""

from __future__ import annotations

import torch

from verl_omni_b200.trainer.diffusion.diffusion_algos import get_diffusion_loss_fn
from verl_omni_b200.trainer.diffusion.rollout_correction import compute_rollout_correction_and_rejection_mask


def _apply_bypass_rc(log_prob, old_log_prob, rc_cfg, data: dict, metrics: dict) -> None:
    lp = log_prob.detach().unsqueeze(-1)
    rl = old_log_prob.unsqueeze(-1)
    _, keep, rc_metrics = compute_rollout_correction_and_rejection_mask(
        old_log_prob=lp, rollout_log_prob=rl, response_mask=torch.ones_like(lp), rollout_is=rc_cfg.rollout_is,
        rollout_is_threshold=rc_cfg.rollout_is_threshold, rollout_is_batch_normalize=rc_cfg.rollout_is_batch_normalize,
        rollout_rs=rc_cfg.rollout_rs, rollout_rs_threshold=rc_cfg.rollout_rs_threshold)
    if rc_cfg.rollout_rs:
        w = keep.squeeze(-1).to(log_prob.dtype)
        prev = data.get("rollout_is_weights")
        data["rollout_is_weights"] = w if prev is None else prev * w
    for k, v in rc_metrics.items():
        metrics[f"actor/rollout_corr/{k}"] = v


def diffusion_loss(config, model_output: dict, data: dict, dp_group=None):
    metrics: dict = {}
    config.global_batch_info["loss_scale_factor"] = config.loss_scale_factor
    mode = config.diffusion_loss.loss_mode
    fn = get_diffusion_loss_fn(mode)
    if "log_probs" in fn.required_model_output_keys and config.rollout_correction.bypass_mode:
        _apply_bypass_rc(model_output["log_probs"], data["old_log_probs"], config.rollout_correction, data, metrics)
    fn.validate_inputs(loss_name=mode, model_output=model_output, data=data)
    res = fn(config=config, model_output=model_output, data=data)
    loss = res.loss
    metrics.update(res.metrics)
    if res.add_loss_metric:
        metrics["actor/loss"] = loss.detach()
    if config.use_kl_loss:
        kfn = get_diffusion_loss_fn("kl")
        kfn.validate_inputs(loss_name="kl", model_output=model_output, data=data)
        kr = kfn(config=config, model_output=model_output, data=data)
        loss = loss + kr.loss * config.kl_loss_coef
        metrics.update(kr.metrics)
        metrics["kl_coef"] = config.kl_loss_coef
    if config.use_distill_loss:
        dfn = get_diffusion_loss_fn(config.distill_loss_mode)
        dfn.validate_inputs(loss_name=config.distill_loss_mode, model_output=model_output, data=data)
        dr = dfn(config=config, model_output=model_output, data=data)
        loss = loss + dr.loss * config.distill_loss_coef
        metrics.update(dr.metrics)
        metrics["distill_coef"] = config.distill_loss_coef
    gas = data.get("gradient_accumulation_steps") or 1
    loss = loss / gas
    sp = data.get("sp_size") or 1
    if sp > 1:
        loss = loss * sp
    return loss, metrics
