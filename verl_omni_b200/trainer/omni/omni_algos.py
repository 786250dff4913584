"""Token-level policy losses for the omni thinker and the omni DPO loss.

* ``grpo``: PPO-clip on token log-ratios, token-mean over response tokens (verl ``compute_policy_loss``
  with ``loss_agg_mode=token-mean``).
* ``gspo``: sequence-level importance ratio ``s_i = exp(mean_t(logp - old))`` clipped with
  ``clip_ratio_low/high``; gradient flows per token through ``s_i * pi / sg(pi)`` (GSPO).
* ``dpo`` (``verl_omni/trainer/omni/omni_algos.py:61-205``): Bradley-Terry (sigmoid, with label
  smoothing) or IPO on sequence log-prob differences against the reference, optionally length-averaged.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

OMNI_LOSSES: dict = {}


def register_omni_loss(name: str):
    def deco(fn):
        OMNI_LOSSES[name] = fn
        return fn

    return deco


def get_omni_loss_fn(name: str):
    if name not in OMNI_LOSSES:
        raise ValueError(f"unknown omni loss {name!r}; known {sorted(OMNI_LOSSES)}")
    return OMNI_LOSSES[name]


def masked_mean(x, mask):
    return (x * mask).sum() / mask.sum().clamp_min(1)


@register_omni_loss("grpo")
def grpo_loss(logp, old_logp, adv, mask, clip_low: float = 0.2, clip_high: float = 0.2):
    ratio = torch.exp(logp - old_logp)
    a = adv[:, None] if adv.ndim == 1 else adv
    loss = torch.maximum(-a * ratio, -a * torch.clamp(ratio, 1 - clip_low, 1 + clip_high))
    with torch.no_grad():
        cf = masked_mean(((ratio - 1).abs() > max(clip_low, clip_high)).float(), mask)
        kl = masked_mean(old_logp - logp, mask)
    return masked_mean(loss, mask), {"actor/pg_clipfrac": float(cf), "actor/ppo_kl": float(kl)}


@register_omni_loss("gspo")
def gspo_loss(logp, old_logp, adv, mask, clip_low: float = 3e-4, clip_high: float = 4e-4):
    n = mask.sum(-1).clamp_min(1)
    seq_lr = ((logp - old_logp) * mask).sum(-1) / n
    s = torch.exp(seq_lr.detach())[:, None] * torch.exp(logp - logp.detach())
    a = adv[:, None] if adv.ndim == 1 else adv
    loss = torch.maximum(-a * s, -a * torch.clamp(s, 1 - clip_low, 1 + clip_high))
    with torch.no_grad():
        cf = (((torch.exp(seq_lr) - 1).abs() > clip_high).float()).mean()
    return masked_mean(loss, mask), {"actor/pg_clipfrac": float(cf), "actor/seq_ratio_mean": float(torch.exp(seq_lr).mean())}


@register_omni_loss("dpo")
def omni_dpo_loss(policy_chosen, policy_rejected, ref_chosen, ref_rejected, beta: float = 0.1,
                  label_smoothing: float = 0.0, loss_type: str = "sigmoid"):
    logits = (policy_chosen - policy_rejected) - (ref_chosen - ref_rejected)
    if loss_type == "ipo":
        losses = (logits - 1 / (2 * beta)) ** 2
    else:
        losses = -F.logsigmoid(beta * logits) * (1 - label_smoothing) - F.logsigmoid(-beta * logits) * label_smoothing
    cr = beta * (policy_chosen - ref_chosen).detach()
    rr = beta * (policy_rejected - ref_rejected).detach()
    loss = losses.mean()
    return loss, {"dpo_loss": float(loss.detach()), "chosen_rewards": float(cr.mean()),
                  "rejected_rewards": float(rr.mean()), "reward_accuracy": float((cr > rr).float().mean()),
                  "reward_margin": float((cr - rr).mean())}


def sequence_logps(token_logps, labels_mask, average: bool = False):
    s = (token_logps * labels_mask).sum(-1)
    return s / labels_mask.sum(-1).clamp_min(1) if average else s
