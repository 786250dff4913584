"""Full / joint attention.

Inputs ``q, k, v`` are ``[B, H, S, Dh]`` bf16 (the layout the fused q/k-norm split writes); the
output is token-major ``[B, S, H*Dh]`` so it feeds the output projection GEMM directly.  CUDA
tensors run the tcgen05 flash-attention kernels (``csrc/fmha_sm100.cu``) when built; CPU tensors
use ``scaled_dot_product_attention`` (the fp32 oracle).
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

from verl_omni_b200.ops._ext import ext


# forward kernel generation: 2 = two query tiles per CTA with P/O in tensor memory, 1 = one tile per CTA
_FWD_VERSION = int(os.environ.get("VO_FMHA_FWD", "1"))
# backward kernel generation: 2 = pipelined (P^T/dS^T in tensor memory, concurrent dQ drain), 1 = serial
_BWD_VERSION = int(os.environ.get("VO_FMHA_BWD", "1"))


def _native() -> bool:
    return os.environ.get("VO_ATTN", "native") != "torch" and hasattr(ext(), "fmha_fwd")


class _FMHA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        o, lse = ext().fmha_fwd(q, k, v, causal, scale, _FWD_VERSION)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.meta = (causal, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        causal, scale = ctx.meta
        if os.environ.get("VO_ATTN_BWD", "native") != "torch" and hasattr(ext(), "fmha_bwd"):
            B, S, H, D = o.shape
            dq, dk, dv = ext().fmha_bwd(q, k, v, o, lse, do.contiguous().view(B, S, H, D), causal, scale,
                                        _BWD_VERSION)
            return dq, dk, dv, None, None
        # backward kernel not built: recompute through SDPA autograd
        B, S, H, D = o.shape
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            oo = F.scaled_dot_product_attention(qq, kk, vv, is_causal=causal, scale=scale)
            dq, dk, dv = torch.autograd.grad(oo, (qq, kk, vv), do.view(B, S, H, D).transpose(1, 2))
        return dq, dk, dv, None, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              scale: Optional[float] = None) -> torch.Tensor:
    """softmax(q k^T * scale) v over [B, H, S, Dh]; returns [B, S, H*Dh]."""
    B, H, S, Dh = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(Dh)
    # the tcgen05 kernels cover head_dim 64 / 128 (every DiT, ViT and LLM head here); other widths
    # (the VAE's single 512-wide mid-block head, miniature test models) use SDPA
    if q.is_cuda and _native() and Dh in (64, 128) and q.dtype == torch.bfloat16:
        o = _FMHA.apply(q, k, v, causal, scale)  # [B, S, H, Dh]
        return o.view(B, S, H * Dh)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)
    return o.transpose(1, 2).reshape(B, S, H * Dh)
