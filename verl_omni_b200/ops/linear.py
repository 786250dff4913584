"""Linear layers on the tcgen05 GEMM with fused epilogues and fp32 main-grad accumulation.

Forward ``y = x W^T + b`` with optional fused epilogues:

* ``gelu``     : ``y = gelu_tanh(x W^T + b)`` (pre-activation kept for backward);
* ``gate_res`` : ``y = res + gate[b] * (x W^T + b)`` -- the AdaLN-Zero gated residual of DiT blocks.

Backward computes ``dX = dY W`` and accumulates ``dW = dY^T X`` straight into the fp32
``weight.main_grad`` buffer that the sharded engine owns (no bf16 weight-grad tensor, no
separate accumulation pass), and ``db`` into ``bias.main_grad``.  Parameters without a
``main_grad`` get ordinary ``.grad`` tensors.  CPU tensors use ``torch.nn.functional``.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.nn.functional as F

from verl_omni_b200.ops import gemm as G
from verl_omni_b200.ops._ext import ext


def _accum(param: torch.Tensor, grad: torch.Tensor):
    """Returns the grad to hand back to autograd (None when accumulated into main_grad)."""
    mg = getattr(param, "main_grad", None)
    if mg is None:
        return grad.to(param.dtype)
    mg.add_(grad.view_as(mg))
    return None


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, epilogue, gate, res, S):
        x2 = x.reshape(-1, x.shape[-1])
        out, pre = G.linear_fwd(x2, w, b, epilogue=epilogue, gate=gate, res=res.reshape(-1, w.shape[0]) if res is not None else None, S=S)
        ctx.save_for_backward(x2, w, pre if pre is not None else torch.empty(0, device=x.device), gate if gate is not None else torch.empty(0, device=x.device))
        ctx.meta = (epilogue, S, x.shape, b is not None, b)
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w, pre, gate = ctx.saved_tensors
        epilogue, S, xshape, has_b, b = ctx.meta
        dy2, d_gate, gb = _bwd_prep(dy, w, b if has_b else None, pre, gate, epilogue, S)
        d_res = dy if epilogue == "gate_res" else None  # the residual passes through
        dx = G.matmul_nn(dy2, w)  # [M, N] x [N, K] -> [M, K]
        dw = G.wgrad(dy2, x2, getattr(w, "main_grad", None))
        gw = None if dw is None else dw.to(w.dtype)
        return dx.view(xshape), gw, gb, None, d_gate, d_res, None


def _bwd_prep(dy, w, b, pre, gate, epilogue: str, S: int):
    """dY of the GEMM (after gelu' / gate scaling), the gate gradient and the bias gradient to return
    (None when it went into ``bias.main_grad``)."""
    N = w.shape[0]
    dy2 = dy.reshape(-1, N)
    if not dy2.is_contiguous():
        dy2 = dy2.contiguous()
    d_gate = gb = None
    if _fused_prep_ok(dy2, gate if epilogue == "gate_res" else None):
        # one pass over dY: gelu'/gate scaling, gate grad and bias grad (into bias.main_grad)
        mode = _MODE[epilogue]
        mg = getattr(b, "main_grad", None) if b is not None else None
        db = None
        if b is not None:
            db = mg if mg is not None else torch.empty(N, device=dy.device, dtype=torch.float32)
        dy2, dg = ext().linear_bwd_prep(dy2, pre if mode else None, gate if mode == 2 else None, S, mode, db,
                                        mg is not None)
        if mode == 2:
            d_gate = dg
        if b is not None and mg is None:
            gb = db.to(b.dtype)
        return dy2, d_gate, gb
    if epilogue == "gate_res":
        # y_lin = pre (saved linear output); dgate[b, n] = sum_s dy * y_lin
        B = dy2.shape[0] // S
        d_gate = (dy2.float().view(B, S, -1) * pre.float().view(B, S, -1)).sum(1).to(gate.dtype)
        dy2 = (dy2.view(B, S, -1) * gate.view(B, 1, -1)).reshape(dy2.shape).contiguous()
    elif epilogue == "gelu":
        dy2 = G.gelu_bwd(dy2, pre)
    if b is not None:
        gb = _accum(b, dy2.float().sum(0))
    return dy2, d_gate, gb


class _LinearPairFn(torch.autograd.Function):
    """Two independent linears (same epilogue kind) whose forward, dgrad and wgrad GEMMs each run as one
    grouped persistent launch: the image and text streams of a joint transformer block."""

    @staticmethod
    def forward(ctx, x0, w0, b0, x1, w1, b1, epilogue, gate0, res0, S0, gate1, res1, S1):
        e = ext()
        a0 = x0.reshape(-1, x0.shape[-1])
        a1 = x1.reshape(-1, x1.shape[-1])
        r0 = res0.reshape(-1, w0.shape[0]) if res0 is not None else None
        r1 = res1.reshape(-1, w1.shape[0]) if res1 is not None else None
        code = EPI_CODES[epilogue] if epilogue != "none" else None
        if code is None:
            if (b0 is None) != (b1 is None):
                raise ValueError("paired linears must both have a bias or both not")
            code = EPI_CODES["bias"] if b0 is not None else EPI_CODES["none"]
        o0, s0, o1, s1 = e.gemm_fwd_pair(a0, w0, b0, gate0, r0, S0, a1, w1, b1, gate1, r1, S1, code)
        empty = torch.empty(0, device=x0.device)
        ctx.save_for_backward(a0, w0, s0 if s0 is not None and s0.numel() else empty,
                              gate0 if gate0 is not None else empty, a1, w1,
                              s1 if s1 is not None and s1.numel() else empty, gate1 if gate1 is not None else empty)
        ctx.meta = (epilogue, S0, S1, x0.shape, x1.shape, b0, b1)
        return o0.view(*x0.shape[:-1], w0.shape[0]), o1.view(*x1.shape[:-1], w1.shape[0])

    @staticmethod
    def backward(ctx, dy0, dy1):
        a0, w0, pre0, gate0, a1, w1, pre1, gate1 = ctx.saved_tensors
        epilogue, S0, S1, xs0, xs1, b0, b1 = ctx.meta
        e = ext()
        d0, dg0, gb0 = _bwd_prep(dy0, w0, b0, pre0, gate0, epilogue, S0)
        d1, dg1, gb1 = _bwd_prep(dy1, w1, b1, pre1, gate1, epilogue, S1)
        dx0, dx1 = e.gemm_dgrad_pair(d0, w0, d1, w1)
        mg0, mg1 = getattr(w0, "main_grad", None), getattr(w1, "main_grad", None)
        gw0 = gw1 = None
        if mg0 is not None and mg1 is not None:
            e.gemm_wgrad_pair(d0, a0, mg0, d1, a1, mg1, True)
        else:
            g0, g1 = G.wgrad(d0, a0, mg0), G.wgrad(d1, a1, mg1)
            gw0 = None if g0 is None else g0.to(w0.dtype)
            gw1 = None if g1 is None else g1.to(w1.dtype)
        gr = epilogue == "gate_res"
        return (dx0.view(xs0), gw0, gb0, dx1.view(xs1), gw1, gb1, None, dg0, dy0 if gr else None, None, dg1,
                dy1 if gr else None, None)


def linear_pair_native_ok(x0, w0, x1, w1) -> bool:
    """Both linears can share one grouped tcgen05 launch (bf16 CUDA, 16-byte rows, >= 128 rows each)."""
    if os.environ.get("VO_GEMM_PAIR", "1") == "0":
        return False
    if not (x0.is_cuda and x1.is_cuda and x0.dtype == x1.dtype == w0.dtype == w1.dtype == torch.bfloat16):
        return False
    r0, r1 = x0.numel() // x0.shape[-1], x1.numel() // x1.shape[-1]
    return (G._use_native(x0.shape[-1], w0.shape[0], rows=r0) and G._use_native(x1.shape[-1], w1.shape[0], rows=r1)
            and hasattr(ext(), "gemm_fwd_pair"))


def linear_pair(x0, w0, b0, x1, w1, b1, *, epilogue: str = "none", gate0=None, res0=None, S0: int = 1, gate1=None,
                res1=None, S1: int = 1):
    """``(linear(x0, w0, b0, ...), linear(x1, w1, b1, ...))`` as grouped GEMM launches when possible."""
    if linear_pair_native_ok(x0, w0, x1, w1):
        return _LinearPairFn.apply(x0, w0, b0, x1, w1, b1, epilogue, gate0, res0, S0, gate1, res1, S1)
    return (linear(x0, w0, b0, epilogue=epilogue, gate=gate0, res=res0, S=S0),
            linear(x1, w1, b1, epilogue=epilogue, gate=gate1, res=res1, S=S1))


_MODE = {"none": 0, "gelu": 1, "gate_res": 2}


def _fused_prep_ok(dy2: torch.Tensor, gate: Optional[torch.Tensor]) -> bool:
    if dy2.dtype != torch.bfloat16 or dy2.shape[1] % 8 or dy2.data_ptr() % 16:
        return False
    if gate is not None and (gate.dtype != torch.bfloat16 or gate.dim() != 2 or gate.stride(1) != 1
                             or gate.stride(0) % 8 or gate.data_ptr() % 16):
        return False
    return hasattr(ext(), "linear_bwd_prep")


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None, *, epilogue: str = "none",
           gate: Optional[torch.Tensor] = None, res: Optional[torch.Tensor] = None, S: int = 1) -> torch.Tensor:
    """``gate`` is [B, N] (per-sample), ``res`` has the output's shape; ``S`` = rows per sample."""
    if not x.is_cuda:
        y = F.linear(x, w, b)
        if epilogue == "gelu":
            return F.gelu(y, approximate="tanh")
        if epilogue == "gate_res":
            B = gate.shape[0]
            return res + (y.view(B, -1, y.shape[-1]) * gate[:, None]).view_as(res)
        return y
    return _LinearFn.apply(x, w, b, epilogue, gate, res, S)


class _LoRALinearFn(torch.autograd.Function):
    """``y = epilogue(x W^T + b + s * (x A^T) B^T)`` with the low-rank term folded into the main GEMM.

    Forward: ``u = x A^T`` (skinny GEMM), then one tcgen05 GEMM reducing over ``[x | u]`` against
    ``[W | s B]`` with the fused epilogue.  Backward (W and b frozen): ``v = dY (s B)``, one dgrad GEMM
    over ``[dY | v]`` against ``[W ; A]`` gives dX, and the two adapter gradients are skinny weight
    GEMMs ``dB = dY^T (s u)``, ``dA = v^T x`` accumulated into the adapters' fp32 ``main_grad``.
    """

    @staticmethod
    def forward(ctx, x, w, b, A, B, scaling, epilogue, gate, res, S):
        e = ext()
        x2 = x.reshape(-1, x.shape[-1])
        u = e.gemm_fwd(x2, A, None, EPI_CODES["none"], None, None, 1)[0]  # [M, r]
        sB = (B.float() * scaling).to(x.dtype).contiguous()
        res2 = res.reshape(-1, w.shape[0]) if res is not None else None
        out, saved = e.gemm_fwd(x2, w, b, _epi_code(epilogue, b), gate, res2, S, ext_a=u, ext_b=sB)
        empty = torch.empty(0, device=x.device)
        ctx.save_for_backward(x2, w, A, B, u, sB, saved if saved is not None and saved.numel() else empty,
                              gate if gate is not None else empty)
        ctx.meta = (epilogue, S, x.shape, float(scaling))
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w, A, B, u, sB, pre, gate = ctx.saved_tensors
        epilogue, S, xshape, scaling = ctx.meta
        e = ext()
        N = w.shape[0]
        dy2 = dy.reshape(-1, N).contiguous()
        d_gate = d_res = None
        if epilogue == "gate_res":
            d_res = dy
        mode = _MODE[epilogue]
        if mode:
            dy2, dg = e.linear_bwd_prep(dy2, pre, gate if mode == 2 else None, S, mode, None, False)
            if mode == 2:
                d_gate = dg
        v = e.gemm_dgrad(dy2, sB)  # [M, r] = dY (s B)
        dx = e.gemm_dgrad(dy2, w, ext_a=v, ext_b=A)
        gA = gB = None
        su = (u.float() * scaling).to(u.dtype)
        for p, lhs, rhs in ((B, dy2, su), (A, v, x2)):
            mg = getattr(p, "main_grad", None)
            if mg is not None:
                G.wgrad(lhs, rhs, mg)
            else:
                g = G.wgrad(lhs, rhs, None).to(p.dtype)
                if p is A:
                    gA = g
                else:
                    gB = g
        return dx.view(xshape), None, None, gA, gB, None, None, d_gate, d_res, None


EPI_CODES = {"none": 0, "bias": 1, "gelu": 2, "gate_res": 3}


def _epi_code(epilogue: str, b) -> int:
    if epilogue == "none":
        return EPI_CODES["bias"] if b is not None else EPI_CODES["none"]
    return EPI_CODES[epilogue]


def lora_linear_native_ok(x: torch.Tensor, w: torch.Tensor, A: torch.Tensor) -> bool:
    rows = x.numel() // x.shape[-1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and A.dtype == torch.bfloat16
            and G._use_native(x.shape[-1], w.shape[0], A.shape[0], rows=rows) and hasattr(ext(), "gemm_fwd"))


def lora_linear(x, w, b, A, B, scaling: float, *, epilogue: str = "none", gate=None, res=None, S: int = 1):
    """Fused LoRA linear on the tcgen05 GEMM (bf16, CUDA); see :class:`_LoRALinearFn`."""
    return _LoRALinearFn.apply(x, w, b, A, B, float(scaling), epilogue, gate, res, S)
