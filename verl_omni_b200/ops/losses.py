"""Fused clipped policy-gradient objective (FlowGRPO / DanceGRPO / MixGRPO).

``loss = mean_b( w_b * max(-A_b r_b, -A_b clip(r_b, 1-eps, 1+eps)) )`` with
``r_b = exp(logp_b - old_b)`` (``verl_omni/trainer/diffusion/diffusion_algos.py:307-342``), plus the
ppo_kl / clip-fraction / ratio statistics.  On CUDA one single-block kernel computes the loss,
the six statistics and (in backward) d loss / d logp; statistics stay on the device as a tensor
so the training loop does not synchronise per timestep.
"""

from __future__ import annotations

from typing import Optional

import torch

from verl_omni_b200.ops._ext import ext

STAT_NAMES = ("ppo_kl", "clipfrac", "clipfrac_higher", "clipfrac_lower", "ratio_mean", "ratio_std")


def ppo_clip_reference(logp, old, adv, clip, weights=None):
    log_ratio = logp - old
    ratio = torch.exp(log_ratio)
    unc = -adv * ratio
    clp = -adv * torch.clamp(ratio, 1.0 - clip, 1.0 + clip)
    per = torch.maximum(unc, clp)
    if weights is not None:
        per = per * weights.detach()
    loss = per.mean()
    with torch.no_grad():
        stats = torch.stack([
            torch.mean(-log_ratio),
            torch.mean((torch.abs(ratio - 1.0) > clip).float()),
            torch.mean((ratio - 1.0 > clip).float()),
            torch.mean((1.0 - ratio > clip).float()),
            ratio.mean(),
            ratio.std() if ratio.numel() > 1 else torch.zeros((), device=ratio.device),
        ])
    return loss, stats


class _PPOClip(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logp, old, adv, weights, clip):
        loss, stats = ext().ppo_clip_fwd(logp.float().contiguous(), old.float().contiguous(),
                                         adv.float().contiguous(), weights, float(clip))
        ctx.save_for_backward(logp, old, adv, weights if weights is not None else torch.empty(0, device=logp.device))
        ctx.clip = clip
        ctx.has_w = weights is not None
        ctx.mark_non_differentiable(stats)
        return loss, stats

    @staticmethod
    def backward(ctx, g_loss, g_stats):
        logp, old, adv, w = ctx.saved_tensors
        grad = ext().ppo_clip_bwd(logp.float().contiguous(), old.float().contiguous(), adv.float().contiguous(),
                                  w if ctx.has_w else None, float(ctx.clip), g_loss.float().contiguous())
        return grad.to(logp.dtype), None, None, None, None


def ppo_clip_loss(logp: torch.Tensor, old: torch.Tensor, adv: torch.Tensor, clip: float,
                  weights: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, dict]:
    """Returns ``(loss, {stat_name: 0-d tensor})``."""
    if logp.is_cuda:
        w = weights.detach().float().contiguous() if weights is not None else None
        loss, stats = _PPOClip.apply(logp, old.detach(), adv.detach(), w, float(clip))
    else:
        loss, stats = ppo_clip_reference(logp, old, adv, clip, weights)
    return loss, {k: stats[i] for i, k in enumerate(STAT_NAMES)}


def sq_dist_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    d = (a.float() - b.float()).pow(2)
    return d.flatten(1).mean(1) if d.ndim > 1 else d


class _SqDist(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return ext().sq_dist_fwd(a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        need_b = ctx.needs_input_grad[1]
        grads = ext().sq_dist_bwd(a, b, g.float().contiguous(), need_b)
        return grads[0], (grads[1] if need_b else None)


def sq_dist(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Per-sample ``mean((a - b)^2)`` over every non-batch dim -> ``[B]`` fp32.

    The squared distance between two reverse-SDE means behind the Flow-DPPO KL mask
    (``verl_omni/trainer/diffusion/diffusion_algos.py:361-463``), the GRPO-Guard bias term (``:466-587``)
    and the reference / distillation KLs (``:1013-1094``).  On CUDA (fp32, contiguous, per-sample size a
    multiple of 4) one read of both operands in a chunked block reduction replaces the
    sub / pow / mean chain and its two full-size temporaries; backward writes ``2 (a - b) g / n`` once.
    """
    if (a.is_cuda and a.dtype == torch.float32 and b.dtype == torch.float32 and a.shape == b.shape
            and a.ndim > 1 and a.is_contiguous() and b.is_contiguous() and (a.numel() // a.shape[0]) % 4 == 0
            and a.shape[0] <= 65535):
        return _SqDist.apply(a, b)
    return sq_dist_reference(a, b)
