"""Attention backend policy (``verl_omni/utils/diffusion_attention.py:33-135``).

The reference picks FA3 only for compute capability 8.0 <= cc < 10.0 and falls back to SDPA on
Blackwell, then forces actor and rollout to the same backend so log-probs recomputed by the trainer
match the rollout's.  Here the tcgen05 kernels are the native backend on sm_100 and the policy is:
``b200_fmha`` whenever a CUDA device with cc 10.x and the extension are present, else ``sdpa``; the
actor and rollout backends must agree (``validate_attention_consistency``).
"""

from __future__ import annotations

import os

import torch

NATIVE, SDPA = "b200_fmha", "sdpa"
ALIASES = {"native": SDPA, "torch_sdpa": SDPA, "TORCH_SDPA": SDPA, "_flash_3_varlen_hub": NATIVE,
           "FLASH_ATTN_3_HUB": NATIVE, "B200_FMHA": NATIVE, "b200_fmha": NATIVE, "sdpa": SDPA}


def native_available() -> bool:
    if not torch.cuda.is_available():
        return False
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        return False
    from verl_omni_b200.ops._ext import available

    return available()


def resolve_backend(requested: str) -> str:
    b = ALIASES.get(requested, requested)
    if b == NATIVE and not native_available():
        return SDPA
    return b


def apply_backend(backend: str) -> None:
    os.environ["VO_ATTN"] = "native" if backend == NATIVE else "torch"


def validate_attention_consistency(actor_backend: str, rollout_backend: str) -> str:
    a, r = resolve_backend(actor_backend), resolve_backend(rollout_backend)
    if a != r:
        raise ValueError(f"actor attention backend {a!r} differs from rollout backend {r!r}; recomputed "
                         "log-probs would not match the rollout's")
    return a
