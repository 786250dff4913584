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


# forward kernel generation: 5 = as 4 with two independent softmax halves per tile at head_dim 64 (other
# widths run 4); 4 = one query tile per CTA, two CTAs per SM, double-buffered 64-key score
# blocks; 3 = two query tiles per CTA, P/O in tensor memory, two softmax warpgroups per tile; 2 = one
# softmax warpgroup per tile; 1 = one query tile per CTA
_FWD_VERSION = int(os.environ.get("VO_FMHA_FWD", "4"))


def _kv_version() -> int:
    """Forward generation for per-sequence key counts (versions 3 and 4 support them)."""
    return min(_FWD_VERSION, 5) if _FWD_VERSION >= 4 else 3
# backward kernel generation: 2 = pipelined (P^T/dS^T in tensor memory, concurrent dQ drain), 1 = serial
_BWD_VERSION = int(os.environ.get("VO_FMHA_BWD", "3"))


def _native() -> bool:
    return os.environ.get("VO_ATTN", "native") != "torch" and hasattr(ext(), "fmha_fwd")


class _FMHA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale, kv_len=None):
        if kv_len is not None:  # keys at positions >= kv_len[b] masked (forward v3 / v4)
            o, lse = ext().fmha_fwd(q, k, v, False, scale, _kv_version(), 0, kv_len=kv_len)
        else:
            o, lse = ext().fmha_fwd(q, k, v, causal, scale, _FWD_VERSION)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.kv_len = kv_len
        ctx.meta = (causal, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        causal, scale = ctx.meta
        if ctx.kv_len is not None or (os.environ.get("VO_ATTN_BWD", "native") != "torch"
                                      and hasattr(ext(), "fmha_bwd")):
            B, S, H, D = o.shape
            dq, dk, dv = ext().fmha_bwd(q, k, v, o, lse, do.contiguous().view(B, S, H, D), causal, scale,
                                        _BWD_VERSION, kv_len=ctx.kv_len)
            return dq, dk, dv, None, None, None
        # backward kernel not built: recompute through SDPA autograd
        B, S, H, D = o.shape
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            oo = F.scaled_dot_product_attention(qq, kk, vv, is_causal=causal, scale=scale)
            dq, dk, dv = torch.autograd.grad(oo, (qq, kk, vv), do.view(B, S, H, D).transpose(1, 2))
        return dq, dk, dv, None, None, None


class _FMHASplit(torch.autograd.Function):
    """Joint attention whose query rows [0, split) and [split, S) land in two separate outputs."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale, split, kv_len=None):
        if kv_len is not None:  # right-padded keys: per-sequence key counts (forward v3 / v4)
            o_a, lse, o_b = ext().fmha_fwd(q, k, v, causal, scale, _kv_version(), split, kv_len=kv_len)
        else:
            o_a, lse, o_b = ext().fmha_fwd(q, k, v, causal, scale, _FWD_VERSION, split)
        ctx.save_for_backward(q, k, v, o_a, o_b, lse)
        ctx.kv_len = kv_len
        ctx.meta = (causal, scale, split)
        B, _, H, D = o_a.shape
        return o_a.view(B, split, H * D), o_b.view(B, -1, H * D)

    @staticmethod
    def backward(ctx, do_a, do_b):
        q, k, v, o_a, o_b, lse = ctx.saved_tensors
        causal, scale, split = ctx.meta
        do_a = torch.zeros_like(o_a) if do_a is None else do_a.contiguous().view_as(o_a)
        do_b = torch.zeros_like(o_b) if do_b is None else do_b.contiguous().view_as(o_b)
        dq, dk, dv = ext().fmha_bwd(q, k, v, o_a, lse, do_a, causal, scale, _BWD_VERSION, o2=o_b, dO2=do_b,
                                    split=split, kv_len=ctx.kv_len)
        return dq, dk, dv, None, None, None, None


def attention_split(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, split: int, causal: bool = False,
                    scale: Optional[float] = None, kv_len: Optional[torch.Tensor] = None
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """Joint attention returning ``(o[:, :split], o[:, split:])`` as two ``[B, *, H*Dh]`` tensors.

    The tcgen05 forward writes each query row straight into its half (the image / text streams of an
    MMDiT block feed separate output projections), so no slice copies are made; the backward reads
    the two output gradients in place.  Needs ``split`` a multiple of 128 on the native path.
    """
    B, H, S, Dh = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(Dh)
    if (kv_len is None and q.is_cuda and _native() and Dh in (64, 128) and q.dtype == torch.bfloat16
            and _FWD_VERSION >= 2 and 0 < split < S and split % 128 == 0):
        return _FMHASplit.apply(q, k, v, causal, scale, int(split))
    if (kv_len is not None and not causal and q.is_cuda and _native() and Dh in (64, 128)
            and q.dtype == torch.bfloat16 and _FWD_VERSION >= 2 and 0 < split < S and split % 128 == 0):
        # right-padded prompts: native forward / backward with per-sequence key counts
        return _FMHASplit.apply(q, k, v, False, scale, int(split), kv_len.to(torch.int32).contiguous())
    o = attention(q, k, v, causal, scale, kv_len=kv_len)
    return o[:, :split].contiguous(), o[:, split:].contiguous()


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              scale: Optional[float] = None, kv_len: Optional[torch.Tensor] = None,
              key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(q k^T * scale) v over [B, H, S, Dh]; returns [B, S, H*Dh].

    ``kv_len`` [B] (optional): keys at positions >= kv_len[b] are masked (padded prompt tokens at the tail
    of a joint sequence); ``key_mask`` [B, Skv] bool (optional): keys where it is False are masked (the
    same padding after a sequence-parallel gather interleaved it).  Masked cases run on SDPA."""
    B, H, S, Dh = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(Dh)
    if (kv_len is not None and key_mask is None and not causal and q.is_cuda and _native() and Dh in (64, 128)
            and q.dtype == torch.bfloat16 and _FWD_VERSION >= 2):
        o = _FMHA.apply(q, k, v, False, scale, kv_len.to(torch.int32).contiguous())  # [B, S, H, Dh]
        return o.view(B, S, H * Dh)
    if kv_len is not None or key_mask is not None:
        keep = key_mask.to(q.device, torch.bool) if key_mask is not None else (
            torch.arange(k.shape[2], device=q.device)[None, :] < kv_len.to(q.device)[:, None])
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=keep[:, None, None, :], is_causal=False, scale=scale)
        return o.transpose(1, 2).reshape(B, S, H * Dh)
    # the tcgen05 kernels cover head_dim 64 / 128 (every DiT, ViT and LLM head here); other widths
    # (the VAE's single 512-wide mid-block head, miniature test models) use SDPA
    if q.is_cuda and _native() and Dh in (64, 128) and q.dtype == torch.bfloat16:
        o = _FMHA.apply(q, k, v, causal, scale)  # [B, S, H, Dh]
        return o.view(B, S, H * Dh)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)
    return o.transpose(1, 2).reshape(B, S, H * Dh)
