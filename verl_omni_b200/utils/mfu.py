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


@register_flops("flux")
def flux_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    cfg = module.cfg
    D = cfg.hidden
    mlp = int(D * cfg.mlp_ratio)
    S = image_tokens + text_tokens
    double = 2 * (4 * D * D + 2 * D * mlp) * S + 4 * S * S * D      # per-stream weights, joint attention
    single = 2 * (3 * D * D + D * mlp + (D + mlp) * D) * S + 4 * S * S * D  # fused qkv+mlp-in, out over [attn|mlp]
    return cfg.depth_double * double + cfg.depth_single * single + 2 * cfg.joint_attention_dim * D * text_tokens


@register_flops("qwen_image")
def qwen_image_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    cfg = module.cfg
    D = cfg.hidden
    mlp = int(D * getattr(cfg, "mlp_ratio", 4.0))
    S = image_tokens + text_tokens
    return cfg.depth * (2 * (4 * D * D + 2 * D * mlp) * S + 4 * S * S * D)


@register_flops("minimax_h3")
def h3_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    """Single stream over packed [text | audio | video] rows; the modulation linear runs once per sample."""
    cfg = module.cfg
    D = cfg.hidden
    hid = int(D * cfg.mlp_ratio)
    S = cfg.video_rows + cfg.audio_rows + text_tokens  # the packed rows are fixed by the model's layout
    return cfg.depth * (2 * (4 * D * D + 2 * D * hid) * S + 4 * S * S * D) + 2 * cfg.text_dim * D * text_tokens


@register_flops("ltx2")
def ltx2_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    """Video and audio streams per layer: self-attention, text cross-attention, cross-modal attention
    (queries of one stream, keys / values projected from the other), MLP.  The video and audio token counts
    are fixed by the model's latent layout."""
    cfg = module.cfg
    f, h, w = cfg.video_grid
    nv, na = f * h * w, cfg.audio_tokens
    T = text_tokens
    Dv, Da = cfg.video_hidden, cfg.audio_hidden

    def stream(D, N, Do, M):
        hid = int(D * cfg.mlp_ratio)
        lin = 2 * (4 * D * D + 2 * D * D + 2 * D * D + 2 * D * hid) * N  # qkv+o, text q+o, av q+o, mlp
        lin += 2 * (2 * D * D) * T + 2 * (2 * Do * D) * M  # text k/v, cross-modal k/v
        return lin + 4 * N * N * D + 4 * N * T * D + 4 * N * M * D

    per_layer = stream(Dv, nv, Da, na) + stream(Da, na, Dv, nv)
    return cfg.depth * per_layer + 2 * cfg.text_dim * (Dv + Da) * T


@register_flops("bagel")
def bagel_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    """Mixture-of-Transformers: prompt tokens through the understanding weights (causal attention), latent
    tokens through the generation weights attending to every token."""
    cfg = module.cfg
    D, hd = cfg.hidden, cfg.head_dim
    per_tok = (D * (cfg.q_heads + 2 * cfg.kv_heads) * hd + cfg.q_heads * hd * D + 3 * D * cfg.ffn)
    P, L = text_tokens, image_tokens
    attn = 2 * P * P * cfg.q_heads * hd + 4 * L * (P + L) * cfg.q_heads * hd
    return cfg.layers * (2 * per_tok * (P + L) + attn)


def generic_forward_flops(module, image_tokens: int, text_tokens: int) -> float:
    """Fallback: every 2-D weight applied to every token, full attention over all tokens (upper bound for
    families without a formula of their own)."""
    S = image_tokens + text_tokens
    dense = 2.0 * _linear_params(module, lambda n: "embed" not in n) * S
    cfg = getattr(module, "cfg", None)
    depth = getattr(cfg, "depth", 0) or getattr(cfg, "layers", 0) or 0
    hidden = getattr(cfg, "hidden", 0) or 0
    return dense + 4.0 * depth * S * S * hidden


def moe_llm_forward_flops(cfg, batch: int, seq: int) -> float:
    """Forward FLOPs of the MoE thinker's language model over ``batch`` sequences of ``seq`` tokens: the active
    parameters per token (q / k / v / o projections, router, ``top_k`` SwiGLU experts, vocabulary head) twice
    each, plus causal attention (half of 4 S^2 d per layer).  The audio / vision towers are not counted."""
    D, hd = cfg.hidden, cfg.head_dim
    attn_proj = D * (cfg.q_heads + 2 * cfg.kv_heads) * hd + cfg.q_heads * hd * D
    per_token = cfg.layers * (attn_proj + D * cfg.experts + cfg.top_k * 3 * D * cfg.expert_ffn) + D * cfg.vocab
    return 2.0 * per_token * batch * seq + cfg.layers * 2.0 * batch * seq * seq * cfg.q_heads * hd


def omni_step_mfu_metrics(cfg, *, batch: int, seq: int, timing: dict, n_gpus: int) -> dict:
    """``perf/mfu/{rollout,actor_infer,actor}`` of one omni GRPO step from its phase times: generation as one
    forward over the full sequences (prefill + cached decode), the old-log-prob forward, and the update
    (forward + backward = 3 forwards); ``batch`` counts the sequences of all ranks."""
    f = moe_llm_forward_flops(cfg, batch, seq)
    peak = device_peak_tflops() * 1e12 * max(1, n_gpus)
    out = {}
    for key, phase, mult in (("rollout", "gen", 1.0), ("actor_infer", "old_log_prob", 1.0),
                             ("actor", "update_actor", 3.0)):
        t = timing.get(phase)
        if t:
            out[f"perf/mfu/{key}"] = mult * f / (t * peak)
    return out


def token_counts(spec) -> tuple[int, int]:
    """(image-side, text-side) tokens of one sample of an architecture: the scheduler's sequence length or the
    2 x 2-patched latent, plus the reference-image latents of edit models; prompt embeddings, prompt ids or
    the text encoder's prompt length."""
    import numpy as np

    image = spec.sched_seq_len or int(np.prod(spec.latent_shape[1:])) // 4
    ref = spec.cond_shapes.get("image_latents")
    if ref is not None:
        image += int(np.prod(ref[1:])) // 4
    pe = spec.cond_shapes.get("prompt_embeds") or spec.cond_shapes.get("prompt_ids")
    text = int(pe[0]) if pe else int(spec.prompt_len if spec.text_encoder else 0)
    return image, text


class DiffusionFlopsCounter:
    def __init__(self, module, family: str):
        self.module, self.family = module, family
        self._fn = FLOPS_REGISTRY.get(family, generic_forward_flops)

    def forward_flops(self, image_tokens: int, text_tokens: int) -> float:
        return float(self._fn(self.module, image_tokens, text_tokens))

    def estimate_flops(self, num_samples: int, steps: int, image_tokens: int, text_tokens: int, *,
                       cfg_passes: int = 1, train: bool = True) -> float:
        passes = 3.0 if train else 1.0
        return self.forward_flops(image_tokens, text_tokens) * num_samples * steps * cfg_passes * passes

    def mfu(self, flops: float, seconds: float, n_gpus: int = 1) -> float:
        return flops / (max(seconds, 1e-9) * n_gpus * device_peak_tflops() * 1e12)


def step_mfu_metrics(counter: "DiffusionFlopsCounter", *, samples: int, rollout_steps: int, train_steps: int,
                     image_tokens: int, text_tokens: int, cfg_passes: int, timing: dict, step_time: float,
                     recompute_old: bool, ref_passes: int = 0, sp: int = 1) -> dict:
    """Per-rank model-FLOPs utilisation of one FlowGRPO step, by phase, against the measured bf16 GEMM
    peak (the reference reports ``perf/mfu/actor`` for the update and ``perf/mfu/actor_infer`` for the
    old-log-prob recompute).  ``samples`` are this rank's trajectories; under sequence parallelism each of
    the ``sp`` ranks of a group runs 1/sp of every sequence."""
    f = counter.forward_flops(image_tokens, text_tokens) / max(1, sp)
    gen = f * samples * rollout_steps * cfg_passes
    old = f * samples * train_steps if recompute_old else 0.0
    ref = f * samples * train_steps * ref_passes
    upd = 3.0 * f * samples * train_steps
    out = {"perf/flops_per_step_tflop": (gen + old + ref + upd) / 1e12,
           "perf/mfu/step": counter.mfu(gen + old + ref + upd, step_time)}
    if timing.get("update_actor"):
        out["perf/mfu/actor"] = counter.mfu(upd, timing["update_actor"])
    if recompute_old and timing.get("old_log_prob"):
        out["perf/mfu/actor_infer"] = counter.mfu(old, timing["old_log_prob"])
    if timing.get("gen"):
        out["perf/mfu/rollout"] = counter.mfu(gen, timing["gen"])
    return out
