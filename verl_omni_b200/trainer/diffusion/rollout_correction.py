"""Rollout correction (importance sampling + rejection sampling) between rollout and trainer policies.

Diffusion entry points match ``verl_omni/trainer/diffusion/rollout_correction.py:64-217``
(bypass mode, decoupled mode, off-policy diagnostics).  The generic IS/RS helper that the
reference imports from verl is implemented here from its documented behaviour:

* IS: ``rollout_is`` ``token`` -> ``w = exp(old - rollout)`` per step; ``sequence`` -> the product over
  the row.  ``rollout_is_threshold`` float -> upper truncation (TIS); ``"lo_hi"`` string -> weights
  outside ``[lo, hi]`` are zeroed (IcePop).  Optional batch normalisation to mean 1.
* RS: comma-separated modes ``{token,seq_mean,seq_sum,seq_max}_{k1,k2,k3}``; k1 is the log-ratio
  checked against ``[log lo, log hi]`` of a ``"lo_hi"`` threshold, k2 = ``0.5*lr^2`` and
  k3 = ``exp(-lr)-1+lr`` are checked against a single upper bound.  Rejected entries get mask 0.
"""

from __future__ import annotations

import logging
import math
from typing import Optional

import torch

from verl_omni_b200.utils.dataproto import DataProto

_log = logging.getLogger(__name__)
_warned = False


def _warn_once():
    global _warned
    if not _warned:
        _warned = True
        _log.warning("Rollout Correction for diffusion is an EXPERIMENTAL feature.")


def rollout_correction_enabled(cfg) -> bool:
    if cfg is None:
        return False
    return bool(cfg.get("rollout_is", None)) or bool(cfg.get("rollout_rs", None))


def _parse_band(spec) -> tuple[Optional[float], Optional[float]]:
    if spec is None:
        return None, None
    if isinstance(spec, (int, float)):
        return None, float(spec)
    s = str(spec)
    if "_" in s:
        lo, hi = s.split("_", 1)
        return float(lo), float(hi)
    return None, float(s)


def compute_offpolicy_metrics(old_log_prob: torch.Tensor, rollout_log_prob: torch.Tensor,
                              response_mask: torch.Tensor) -> dict:
    m = response_mask.float()
    n = m.sum().clamp_min(1)
    lr = (old_log_prob - rollout_log_prob) * m  # log(pi_old / pi_rollout)
    kl = (-lr).sum() / n  # KL(rollout || old) estimated on rollout samples
    k3 = ((torch.exp(lr) - 1 - lr) * m).sum() / n
    seq_len = m.sum(-1).clamp_min(1)
    log_ppl_old = -(old_log_prob * m).sum(-1) / seq_len
    log_ppl_roll = -(rollout_log_prob * m).sum(-1) / seq_len
    ppl_diff = (log_ppl_roll - log_ppl_old)
    ratio = torch.exp(lr) * m
    chi2_tok = ((ratio ** 2) * m).sum() / n - 1
    seq_ratio = torch.exp((lr).sum(-1))
    chi2_seq = (seq_ratio ** 2).mean() - 1
    return {
        "kl": kl.item(), "k3_kl": k3.item(), "log_ppl_diff": ppl_diff.mean().item(),
        "log_ppl_abs_diff": ppl_diff.abs().mean().item(), "chi2_token": chi2_tok.item(), "chi2_seq": chi2_seq.item(),
    }


def compute_rollout_correction_and_rejection_mask(*, old_log_prob: torch.Tensor, rollout_log_prob: torch.Tensor,
                                                  response_mask: torch.Tensor, rollout_is=None,
                                                  rollout_is_threshold=2.0, rollout_is_batch_normalize=False,
                                                  rollout_rs=None, rollout_rs_threshold=None):
    """Returns ``(is_weights DataProto or None, keep_mask [B,T], metrics)``."""
    mask = response_mask.float()
    lr = (old_log_prob - rollout_log_prob).float()
    metrics: dict = {}
    weights = None
    if rollout_is:
        if rollout_is == "token":
            logw = lr
        elif rollout_is == "sequence":
            logw = (lr * mask).sum(-1, keepdim=True).expand_as(lr)
        else:
            raise ValueError(f"rollout_is must be token or sequence, got {rollout_is!r}")
        w = torch.exp(logw.clamp(max=20.0))
        lo, hi = _parse_band(rollout_is_threshold)
        if lo is not None:
            w = torch.where((w >= lo) & (w <= hi), w, torch.zeros_like(w))
        elif hi is not None:
            w = w.clamp(max=hi)
        if rollout_is_batch_normalize:
            w = w / (w * mask).sum().div(mask.sum().clamp_min(1)).clamp_min(1e-8)
        w = w * mask
        weights = w
        sel = w[mask > 0]
        metrics.update({
            "rollout_is_mean": sel.mean().item(), "rollout_is_max": sel.max().item(),
            "rollout_is_min": sel.min().item(),
            "rollout_is_eff_sample_size": ((sel.sum() ** 2) / (sel.pow(2).sum() * sel.numel()).clamp_min(1e-12)).item(),
        })
    keep = mask.clone()
    if rollout_rs:
        lo, hi = _parse_band(rollout_rs_threshold)
        for mode in str(rollout_rs).split(","):
            mode = mode.strip()
            level, _, k = mode.rpartition("_")
            if k == "k1":
                stat = lr
            elif k == "k2":
                stat = 0.5 * lr ** 2
            elif k == "k3":
                stat = torch.exp(-lr) - 1 + lr
            else:
                raise ValueError(f"unknown rollout_rs mode {mode!r}")
            denom = mask.sum(-1, keepdim=True).clamp_min(1)
            if level == "token":
                s = stat
            elif level == "seq_mean":
                s = ((stat * mask).sum(-1, keepdim=True) / denom).expand_as(stat)
            elif level == "seq_sum":
                s = (stat * mask).sum(-1, keepdim=True).expand_as(stat)
            elif level == "seq_max":
                s = (stat * mask).max(-1, keepdim=True).values.expand_as(stat)
            else:
                raise ValueError(f"unknown rollout_rs mode {mode!r}")
            if k == "k1":
                lo_l = math.log(lo) if lo is not None else -float("inf")
                hi_l = math.log(hi) if hi is not None else float("inf")
                ok = (s >= lo_l) & (s <= hi_l)
            else:
                ok = s <= (hi if hi is not None else float("inf"))
            keep = keep * ok.float()
        rej = 1 - keep[mask > 0]
        metrics["rollout_rs_masked_fraction"] = rej.mean().item()
        metrics["rollout_rs_seq_masked_fraction"] = ((keep * mask).sum(-1) < mask.sum(-1)).float().mean().item()
    metrics.update(compute_offpolicy_metrics(old_log_prob, rollout_log_prob, mask))
    is_proto = DataProto({"rollout_is_weights": weights}) if weights is not None else None
    return is_proto, keep, metrics


def apply_bypass_mode_to_diffusion_batch(batch: DataProto) -> None:
    _warn_once()
    if "rollout_log_probs" not in batch.batch:
        raise ValueError("rollout_correction.bypass_mode=True requires `rollout_log_probs` in the batch. "
                         "Ensure the rollout backend records log probs (calculate_log_probs=true).")
    batch.batch["old_log_probs"] = batch.batch["rollout_log_probs"]


def apply_rollout_correction_to_diffusion_batch(batch: DataProto, cfg) -> tuple[DataProto, dict]:
    _warn_once()
    if "old_log_probs" not in batch.batch or "rollout_log_probs" not in batch.batch:
        raise ValueError("Rollout Correction requires both 'old_log_probs' and 'rollout_log_probs' in the batch.")
    old, roll = batch.batch["old_log_probs"], batch.batch["rollout_log_probs"]
    if old.shape != roll.shape:
        raise ValueError(f"old_log_probs and rollout_log_probs must have identical shapes; got "
                         f"{tuple(old.shape)} vs {tuple(roll.shape)}.")
    if old.dim() != 2:
        raise ValueError(f"Rollout Correction expects 2D log-prob tensors (batch, sde_window); got {tuple(old.shape)}.")
    is_proto, keep, metrics = compute_rollout_correction_and_rejection_mask(
        old_log_prob=old, rollout_log_prob=roll, response_mask=torch.ones_like(old),
        rollout_is=cfg.get("rollout_is", None), rollout_is_threshold=cfg.get("rollout_is_threshold", 2.0),
        rollout_is_batch_normalize=cfg.get("rollout_is_batch_normalize", False),
        rollout_rs=cfg.get("rollout_rs", None), rollout_rs_threshold=cfg.get("rollout_rs_threshold", None))
    eff = None
    if is_proto is not None:
        eff = is_proto.batch["rollout_is_weights"]
    if cfg.get("rollout_rs", None):
        eff = keep if eff is None else eff * keep
    if eff is not None:
        batch.batch["rollout_is_weights"] = eff.to(old.dtype)
    return batch, {f"rollout_corr/{k}": v for k, v in metrics.items()}


def compute_rollout_corr_metrics_from_logprobs(log_prob: torch.Tensor, rollout_log_prob: torch.Tensor,
                                               timesteps: Optional[torch.Tensor] = None) -> dict:
    if log_prob.dim() == 1:
        log_prob, rollout_log_prob = log_prob.unsqueeze(-1), rollout_log_prob.unsqueeze(-1)
    out = {f"rollout_corr/{k}": v for k, v in
           compute_offpolicy_metrics(log_prob, rollout_log_prob, torch.ones_like(log_prob)).items()}
    d = (log_prob - rollout_log_prob).abs()
    out["rollout_corr/logprob_abs_diff_mean"] = d.mean().item()
    out["rollout_corr/logprob_abs_diff_max"] = d.max().item()
    if timesteps is not None and timesteps.shape == log_prob.shape:
        for ts in torch.unique(timesteps):
            out[f"rollout_corr/logprob_abs_diff/ts_{ts.item():.4g}"] = d[timesteps == ts].mean().item()
    return out


def compute_rollout_corr_metrics_from_batch(batch: DataProto, *, bypass_mode: bool) -> dict:
    if bypass_mode or "old_log_probs" not in batch.batch or "rollout_log_probs" not in batch.batch:
        return {}
    return compute_rollout_corr_metrics_from_logprobs(batch.batch["old_log_probs"], batch.batch["rollout_log_probs"],
                                                      timesteps=batch.batch.get("all_timesteps"))
