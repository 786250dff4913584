"""Diffusion FLOPs / MFU counter (``verl_omni/utils/mfu/diffusion_flops_counter.py:79-370``).

Per-architecture FLOPs registry: dense ``2 * P_tok * tokens`` per forward (``P_tok`` = parameters
applied per token, i.e. excluding per-sample modulation / embedding MLPs), attention
``4 * L_attn * H * Dh * S_q * S_kv`` per forward, forward passes per step from CFG, and
``3x`` for forward+backward.  The device peak comes from ``VERL_OMNI_DEVICE_FLOPS_TFLOPS`` or the
measured B200 bf16 GEMM peak.
"""

from __future__ import annotations

import json
import os
from typing import Callable

import torch

FLOPS_REGISTRY: dict[str, Callable] = {}


def register_flops(family: str):
    def deco(fn):
        FLOPS_REGISTRY[family] = fn
        return fn

    return deco


def device_peak_tflops() -> float:
    env = os.environ.get("VERL_OMNI_DEVICE_FLOPS_TFLOPS")
    if env:
        return float(env)
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 2250.0  # dense bf16 nominal


def _linear_params(module: torch.nn.Module, per_token_filter) -> int:
    n = 0
    for name, p in module.named_parameters():
        if p.ndim == 2 and per_token_filter(name):
            n += p.numel()
    return n


@register_flops("sd3")
def mmdit_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    cfg = module.cfg
    D = cfg.hidden
    mlp = int(D * cfg.mlp_ratio)
    per_block_stream = 4 * D * D + 2 * D * mlp  # qkv + out + mlp
    flops = 0.0
    for i, blk in enumerate(module.transformer_blocks):
        flops += 2 * per_block_stream * image_tokens
        txt = (3 * D * D) if blk.cpo else per_block_stream
        flops += 2 * txt * text_tokens
        S = image_tokens + text_tokens
        flops += 4 * S * S * D
        if blk.dual:
            flops += 2 * 4 * D * D * image_tokens + 4 * image_tokens * image_tokens * D
    flops += 2 * (cfg.joint_attention_dim * D) * text_tokens
    flops += 2 * (cfg.in_channels * cfg.patch_size ** 2 * D * 2) * image_tokens
    return flops


@register_flops("wan")
def dit_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    cfg = module.cfg
    D = cfg.hidden
    per_tok = 4 * D * D + 2 * D * cfg.ffn + 2 * D * D  # self qkv+o, ffn, cross q+o
    flops = cfg.depth * (2 * per_tok * image_tokens + 2 * 2 * D * D * text_tokens
                         + 4 * image_tokens * image_tokens * D + 4 * image_tokens * text_tokens * D)
    return flops


class DiffusionFlopsCounter:
    def __init__(self, module, family: str):
        if family not in FLOPS_REGISTRY:
            raise KeyError(f"no FLOPs formula for {family!r}")
        self.module, self.family = module, family

    def forward_flops(self, image_tokens: int, text_tokens: int) -> float:
        return FLOPS_REGISTRY[self.family](self.module, image_tokens, text_tokens)

    def estimate_flops(self, num_samples: int, steps: int, image_tokens: int, text_tokens: int, *,
                       cfg_passes: int = 1, train: bool = True) -> float:
        passes = 3.0 if train else 1.0
        return self.forward_flops(image_tokens, text_tokens) * num_samples * steps * cfg_passes * passes

    def mfu(self, flops: float, seconds: float, n_gpus: int = 1) -> float:
        return flops / (seconds * n_gpus * device_peak_tflops() * 1e12)
