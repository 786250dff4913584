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
        N = w.shape[0]
        dy2 = dy.reshape(-1, N)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        d_gate = d_res = None
        if epilogue == "gate_res":
            d_res = dy  # residual passes through
        gb = None
        if _fused_prep_ok(dy2, gate if epilogue == "gate_res" else None):
            # one pass over dY: gelu'/gate scaling, gate grad and bias grad (into bias.main_grad)
            mode = _MODE[epilogue]
            mg = getattr(b, "main_grad", None) if has_b else None
            db = None
            if has_b:
                db = mg if mg is not None else torch.empty(N, device=dy.device, dtype=torch.float32)
            dy2, dg = ext().linear_bwd_prep(dy2, pre if mode else None, gate if mode == 2 else None, S, mode, db,
                                            mg is not None)
            if mode == 2:
                d_gate = dg
            if has_b and mg is None:
                gb = db.to(b.dtype)
        else:
            if epilogue == "gate_res":
                # y_lin = pre (saved linear output); dgate[b, n] = sum_s dy * y_lin
                B = dy2.shape[0] // S
                d_gate = (dy2.float().view(B, S, -1) * pre.float().view(B, S, -1)).sum(1).to(gate.dtype)
                dy2 = (dy2.view(B, S, -1) * gate.view(B, 1, -1)).reshape(dy2.shape).contiguous()
            elif epilogue == "gelu":
                dy2 = G.gelu_bwd(dy2, pre)
            if has_b:
                gb = _accum(b, dy2.float().sum(0))
        dx = G.matmul_nn(dy2, w)  # [M, N] x [N, K] -> [M, K]
        dw = G.wgrad(dy2, x2, getattr(w, "main_grad", None))
        gw = None if dw is None else dw.to(w.dtype)
        return dx.view(xshape), gw, gb, None, d_gate, d_res, None


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
