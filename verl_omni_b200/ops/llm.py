"""Row ops of the MoE language model on their sm_100a kernels (``csrc/llm_ops.cu``), with fp32 torch
oracles for CPU tensors: RMSNorm, SwiGLU, the softmax router with top-k, and the per-head q/k RMSNorm
fused with rotate-half RoPE (Qwen3 attention: ``verl_omni/models/transformers/qwen3_omni_thinker.py``
runs these as separate torch ops through the HF modules)."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from verl_omni_b200.ops._ext import ext


def _native(*ts: torch.Tensor) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts)


def _accum_w(w: torch.Tensor, g32: torch.Tensor):
    mg = getattr(w, "main_grad", None)
    if mg is not None:
        mg.add_(g32.view_as(mg))
        return None
    return g32.to(w.dtype)


# ---------------------------------------------------------------------------------------------- RMSNorm
def rms_norm_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        y, rstd = ext().rms_norm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        mg = getattr(w, "main_grad", None)
        dw = mg if mg is not None else torch.empty(w.shape, device=w.device, dtype=torch.float32)
        dx = ext().rms_norm_bwd(dy.contiguous(), x, w, rstd, dw.view(-1), mg is not None)
        return dx, (None if mg is not None else dw.to(w.dtype)), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if _native(x, w) and x.shape[-1] % 8 == 0 and x.is_contiguous():
        return _RMSNorm.apply(x, w, float(eps))
    return rms_norm_reference(x, w, eps)


# ---------------------------------------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, da):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(da.contiguous(), gu)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``gu = [gate | up]`` along the last dim."""
    if _native(gu) and gu.shape[-1] % 16 == 0 and gu.is_contiguous():
        return _SwiGLU.apply(gu)
    g, u = gu.float().chunk(2, -1)
    return (F.silu(g) * u).to(gu.dtype)


# ---------------------------------------------------------------------------------------------- router
class _RouterGates(torch.autograd.Function):
    """Renormalised top-k gates from router logits; the backward runs through the saved softmax."""

    @staticmethod
    def forward(ctx, logits, k):
        probs, gates, idx = ext().router_topk(logits.float().contiguous(), int(k))
        ctx.save_for_backward(probs, gates, idx)
        ctx.mark_non_differentiable(idx, probs)
        return gates, idx, probs

    @staticmethod
    def backward(ctx, dgates, _didx, _dprobs):
        probs, gates, idx = ctx.saved_tensors
        # gates_k = p_{i_k} / S, S = sum_j p_{i_j}:  d p_{i_k} = (dg_k - sum_j dg_j gates_j) / S
        sel = probs.gather(1, idx)
        S = sel.sum(-1, keepdim=True)
        dsel = (dgates - (dgates * gates).sum(-1, keepdim=True)) / S
        dp = torch.zeros_like(probs).scatter_(1, idx, dsel)
        # softmax backward
        dlogits = probs * (dp - (dp * probs).sum(-1, keepdim=True))
        return dlogits, None


def router_topk(logits: torch.Tensor, k: int):
    """Softmax router: returns (gates [T, k] renormalised, idx [T, k] int64, probs [T, E] fp32)."""
    if logits.is_cuda and logits.shape[-1] <= 256 and k <= 32:
        return _RouterGates.apply(logits, k)
    probs = torch.softmax(logits.float(), -1)
    g, idx = torch.topk(probs, k, dim=-1)
    return g / g.sum(-1, keepdim=True), idx, probs


# ---------------------------------------------------------------------------------------------- q/k norm + RoPE
def head_norm_rope_reference(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                             eps: float) -> torch.Tensor:
    """x [B, S, H, Dh] -> [B, H, S, Dh]: per-head RMSNorm * w, rotate-half RoPE (cos/sin [S, Dh/2])."""
    y = rms_norm_reference(x, w, eps).float().transpose(1, 2)
    d2 = y.shape[-1] // 2
    y1, y2 = y[..., :d2], y[..., d2:]
    c, s = cos.float()[None, None], sin.float()[None, None]
    return torch.cat([y1 * c - y2 * s, y1 * s + y2 * c], -1).to(x.dtype)


class _HeadNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, col0, H, w, cos, sin, eps):
        y = ext().head_rmsnorm_rope(x, col0, H, w, cos, sin, eps)
        ctx.save_for_backward(x, w, cos, sin)
        ctx.meta = (col0, H, eps)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, cos, sin = ctx.saved_tensors
        col0, H, eps = ctx.meta
        dw = torch.zeros(w.numel(), device=w.device, dtype=torch.float32)
        dxh = ext().head_rmsnorm_rope_bwd(dy.contiguous(), x, col0, H, w, cos, sin, eps, dw)  # [B, S, H, Dh]
        dx = torch.zeros_like(x)
        B, S = x.shape[:2]
        dx[:, :, col0:col0 + H * w.numel()] = dxh.view(B, S, -1)
        return dx, None, None, _accum_w(w, dw), None, None, None


def head_norm_rope(x: torch.Tensor, col0: int, H: int, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   eps: float = 1e-6) -> torch.Tensor:
    """Heads ``[col0, col0 + H Dh)`` of a projection output ``x [B, S, *]`` -> ``[B, H, S, Dh]`` normalised
    (per head, weight ``w`` [Dh]) and rotated (rotate-half RoPE, fp32 tables [S, Dh/2])."""
    Dh = w.numel()
    if _native(x, w) and x.stride(-1) == 1 and Dh <= 256 and Dh % 2 == 0:
        return _HeadNormRope.apply(x, int(col0), int(H), w, cos.float().contiguous(), sin.float().contiguous(),
                                   float(eps))
    B, S = x.shape[:2]
    xh = x[..., col0:col0 + H * Dh].reshape(B, S, H, Dh)
    return head_norm_rope_reference(xh, w, cos, sin, eps)
