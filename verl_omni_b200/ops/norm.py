"""AdaLN-modulated LayerNorm and fused q/k RMSNorm + QKV split (sm_100a kernels; torch oracle on CPU)."""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from verl_omni_b200.ops._ext import ext


# ----------------------------------------------------------------------------- AdaLN LayerNorm
def adaln_ln_reference(x, shift, scale, eps=1e-6):
    """x [B, S, D]; shift/scale [B, D] -> LN(x)*(1+scale)+shift (LN without affine)."""
    y = F.layer_norm(x.float(), (x.shape[-1],), eps=eps)
    return (y * (1 + scale.float()[:, None]) + shift.float()[:, None]).to(x.dtype)


class _AdaLN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mod, shift_idx, scale_idx, nchunks, eps):
        B, S, D = x.shape
        y, mean, rstd = ext().adaln_ln_fwd(x, mod, shift_idx * D, scale_idx * D, None, None, S, eps)
        ctx.save_for_backward(x, mean, rstd, mod)
        ctx.meta = (shift_idx, scale_idx, nchunks)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, mean, rstd, mod = ctx.saved_tensors
        shift_idx, scale_idx, nchunks = ctx.meta
        B, S, D = x.shape
        dx, dshift, dscale = ext().adaln_ln_bwd(dy.contiguous(), x, mean, rstd, mod, shift_idx * D, scale_idx * D, S)
        dmod = torch.zeros(B, nchunks, D, device=x.device, dtype=torch.float32)
        dmod[:, shift_idx] = dshift
        dmod[:, scale_idx] = dscale
        return dx, dmod.reshape(B, nchunks * D).to(mod.dtype), None, None, None, None


def adaln_layernorm(x: torch.Tensor, mod: torch.Tensor, shift_idx: int, scale_idx: int, nchunks: int,
                    eps: float = 1e-6) -> torch.Tensor:
    """``mod`` is the modulation GEMM output [B, nchunks*D]; chunk ``shift_idx``/``scale_idx`` are used in place."""
    D = x.shape[-1]
    if not x.is_cuda:
        m = mod.view(mod.shape[0], nchunks, D)
        return adaln_ln_reference(x, m[:, shift_idx], m[:, scale_idx], eps)
    return _AdaLN.apply(x.contiguous(), mod.contiguous(), shift_idx, scale_idx, nchunks, eps)


class _AffineLN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        D = x.shape[-1]
        y, mean, rstd = ext().adaln_ln_fwd(x.reshape(-1, D), None, 0, 0, w, b, 1, eps)
        ctx.save_for_backward(x, w, b, mean, rstd)
        return y.view_as(x)

    @staticmethod
    def backward(ctx, dy):
        # y = xhat * w + b is the modulated form xhat * (1 + scale) + shift of one sample whose sequence is
        # every row: the AdaLN backward kernel gives dx and the column sums db = sum dy, dw = sum dy * xhat
        x, w, b, mean, rstd = ctx.saved_tensors
        D = x.shape[-1]
        N = x.numel() // D
        mod = torch.cat([b.float(), w.float() - 1.0]).to(torch.bfloat16).reshape(1, 2 * D)
        dx, db, dw = ext().adaln_ln_bwd(dy.contiguous().reshape(1, N, D), x.reshape(1, N, D), mean, rstd, mod, 0, D, N)
        return dx.view_as(x), dw.reshape(D).to(w.dtype), db.reshape(D).to(b.dtype), None


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
            and x.shape[-1] % 8 == 0):
        return _AffineLN.apply(x.contiguous(), w.contiguous(), b.contiguous(), eps)
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


# ----------------------------------------------------------------------------- q/k RMSNorm + split
def apply_rope_reference(x, cos, sin):
    """Interleaved-pair rotary embedding on the last dim; x [B, S, H, Dh], cos/sin [S, Dh/2]."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[None, :, None, :].to(x.dtype), sin[None, :, None, :].to(x.dtype)
    out = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    return out.flatten(-2)


def _split_reference(x2d, wq, wk, heads, S_seg, parts, eps, rope):
    rows = x2d.shape[0]
    B = rows // S_seg
    outs = []
    for which, off in enumerate(parts):
        if off < 0:
            outs.append(None)
            continue
        width = heads * (wq.shape[0] if wq is not None else wk.shape[0])
        t = x2d[:, off:off + width].float().view(B, S_seg, heads, -1)
        if which < 2:
            w = wq if which == 0 else wk
            t = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w.float()
            if rope is not None:
                t = apply_rope_reference(t, rope[0][:S_seg] if rope[0].shape[0] >= S_seg else rope[0], rope[1][:S_seg] if rope[1].shape[0] >= S_seg else rope[1])
        outs.append(t.permute(0, 2, 1, 3).to(x2d.dtype))
    return outs


class _QKSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q_buf, k_buf, v_buf, x2d, wq, wk, S_seg, seg_off, parts, rope_cos, rope_sin, eps):
        rq, rk = ext().qk_rmsnorm_fwd(x2d, wq, wk, q_buf, k_buf, v_buf, S_seg, seg_off, rope_cos, rope_sin, eps,
                                      list(parts))
        ctx.save_for_backward(x2d, wq, wk, rq, rk,
                              rope_cos if rope_cos is not None else torch.empty(0),
                              rope_sin if rope_sin is not None else torch.empty(0))
        ctx.meta = (S_seg, seg_off, parts, rope_cos is not None)
        dirty = [t for t in (q_buf, k_buf, v_buf) if t is not None]
        ctx.mark_dirty(*dirty)
        return q_buf, k_buf, v_buf

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x2d, wq, wk, rq, rk, rc, rs = ctx.saved_tensors
        S_seg, seg_off, parts, has_rope = ctx.meta
        c = lambda t: t.contiguous() if t is not None else None  # noqa: E731
        dx, dwq, dwk = ext().qk_rmsnorm_bwd(x2d, wq, wk, c(dq), c(dk), c(dv), rq, rk, S_seg, seg_off,
                                            rc if has_rope else None, rs if has_rope else None, list(parts))
        gq = dwq.to(wq.dtype) if parts[0] >= 0 else None
        gk = dwk.to(wk.dtype) if parts[1] >= 0 else None
        return dq, dk, dv, dx, gq, gk, None, None, None, None, None, None


def qk_norm_split_into(q_buf, k_buf, v_buf, x2d, wq, wk, S_seg: int, seg_off: int, parts=None, rope=None,
                       eps: float = 1e-6):
    """Scatter one stream's projections into joint attention buffers ``[B, H, S_total, Dh]``.

    ``x2d`` [B*S_seg, W] holds q at column ``parts[0]``, k at ``parts[1]``, v at ``parts[2]``
    (-1: absent; default: a fused [q|k|v] projection).  q and k get per-head RMSNorm with weights
    ``wq``/``wk`` (and rotary embedding when ``rope=(cos, sin)`` [S_total, Dh/2] is given); v is copied.
    The buffers are written at sequence rows ``[seg_off, seg_off+S_seg)`` and returned (autograd-tracked).
    """
    ref = next(t for t in (q_buf, k_buf, v_buf) if t is not None)
    H, dh = ref.shape[1], ref.shape[3]
    D = H * dh
    if parts is None:
        parts = (0, D, 2 * D)
    if not x2d.is_cuda:
        rr = None
        if rope is not None:
            rr = (rope[0][seg_off:seg_off + S_seg], rope[1][seg_off:seg_off + S_seg])
        outs = _split_reference(x2d, wq, wk, H, S_seg, parts, eps, rr)
        res = []
        for buf, o in zip((q_buf, k_buf, v_buf), outs):
            if buf is None:
                res.append(None)
                continue
            buf = buf.clone()
            buf[:, :, seg_off:seg_off + S_seg] = o
            res.append(buf)
        return tuple(res)
    rc, rs = (rope if rope is not None else (None, None))
    return _QKSplit.apply(q_buf, k_buf, v_buf, x2d.contiguous(), wq, wk, S_seg, seg_off, tuple(parts), rc, rs, eps)


# ----------------------------------------------------------------------------- GroupNorm (+SiLU)
def group_norm_act(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, groups: int, eps: float = 1e-6,
                   silu: bool = False) -> torch.Tensor:
    """GroupNorm with an optional fused SiLU.  bf16 channels-last CUDA tensors without autograd use the
    NHWC kernel (``csrc/groupnorm.cu``); everything else the eager op."""
    if (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 4 and not torch.is_grad_enabled()
            and x.is_contiguous(memory_format=torch.channels_last) and x.shape[1] % 8 == 0):
        return ext().group_norm_nhwc(x, weight.to(x.dtype), bias.to(x.dtype), groups, eps, silu)
    y = F.group_norm(x, groups, weight, bias, eps)
    return F.silu(y) if silu else y
