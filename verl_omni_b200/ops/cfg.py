"""Classifier-free guidance combine, optionally with true-CFG norm renormalisation.

``comb = neg + g * (pos - neg)``; with ``renorm`` each (sample, position) vector over the channel
axis is rescaled to the norm of ``pos`` (Qwen-Image true CFG, reference
``verl_omni/pipelines/qwen_image_flow_grpo/common.py:32-40``; plain CFG as in
``verl_omni/pipelines/wan22_dance_grpo/common.py:41-57``).  Predictions are ``[B, C, ...]``; CUDA
tensors use one fused kernel (``csrc/cfg.cu``), CPU tensors the fp32 restatement below.
"""

from __future__ import annotations

import torch

from verl_omni_b200.ops._ext import ext


def cfg_combine_reference(pos: torch.Tensor, neg: torch.Tensor, g: float, renorm: bool = False) -> torch.Tensor:
    p, n = pos.float(), neg.float()
    comb = n + g * (p - n)
    if renorm:
        pn = torch.linalg.vector_norm(p, dim=1, keepdim=True)
        cn = torch.linalg.vector_norm(comb, dim=1, keepdim=True)
        comb = comb * torch.where(cn > 0, pn / cn, torch.ones_like(cn))
    return comb


def cfg_combine(pos: torch.Tensor, neg: torch.Tensor, g: float, renorm: bool = False) -> torch.Tensor:
    """fp32 combined prediction (no autograd: rollout-time guidance)."""
    if pos.is_cuda and not torch.is_grad_enabled():
        return ext().cfg_combine(pos.contiguous(), neg.contiguous(), float(g), bool(renorm))
    return cfg_combine_reference(pos, neg, g, renorm)
