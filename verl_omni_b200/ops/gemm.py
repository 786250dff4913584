"""GEMM entry points used by the layers.

All three GEMMs of a linear layer run on the hand-written tcgen05/TMEM/TMA kernel
(``csrc/gemm_sm100.cu``) when the extension provides it:

* forward  ``Y[M,N] = X[M,K] W[N,K]^T``           (A K-major, B K-major) + fused epilogue
* dgrad    ``dX[M,K] = dY[M,N] W[N,K]``           (B MN-major)
* wgrad    ``dW[N,K] += dY[M,N]^T X[M,K]``        (A and B MN-major, fp32 accumulate into main_grad)

``VO_GEMM=torch`` selects the cuBLAS path (used only as the comparison baseline in tests and
benchmarks).
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.nn.functional as F

from verl_omni_b200.ops._ext import ext

_GELU_C = 0.7978845608028654  # sqrt(2/pi)


# Below this many output rows a 128/256-row tensor-core tile is mostly padding (e.g. the AdaLN
# modulation linear over one embedding per sample): such skinny GEMMs go to cuBLAS.
_MIN_ROWS = 128


def _use_native(*dims: int, rows: int = _MIN_ROWS) -> bool:
    """The tcgen05 GEMM needs 16-byte rows (every dim a multiple of 8 bf16); odd-width heads such as a
    scalar reward head (N = 1) go to cuBLAS, as do GEMMs with fewer than ``_MIN_ROWS`` output rows."""
    if any(d % 8 for d in dims) or rows < _MIN_ROWS:
        return False
    return os.environ.get("VO_GEMM", "native") != "torch" and hasattr(ext(), "gemm_fwd")


# epilogue codes shared with csrc/gemm_sm100.cu
EPI_NONE, EPI_BIAS, EPI_GELU, EPI_GATE_RES = 0, 1, 2, 3


def linear_fwd(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], *, epilogue: str = "none",
               gate: Optional[torch.Tensor] = None, res: Optional[torch.Tensor] = None, S: int = 1):
    """Returns ``(out, saved)``: ``saved`` is the pre-activation (gelu) or the linear output (gate_res)."""
    if x.dtype == w.dtype == torch.bfloat16 and _use_native(x.shape[1], w.shape[0], rows=x.shape[0]):
        e = ext()
        if epilogue == "gelu":
            out, pre = e.gemm_fwd(x, w, b, EPI_GELU, None, None, S)
            return out, pre
        if epilogue == "gate_res":
            out, lin = e.gemm_fwd(x, w, b, EPI_GATE_RES, gate, res, S)
            return out, lin
        out, _ = e.gemm_fwd(x, w, b, EPI_BIAS if b is not None else EPI_NONE, None, None, S)
        return out, None
    y = F.linear(x, w, b)
    if epilogue == "gelu":
        return F.gelu(y, approximate="tanh"), y
    if epilogue == "gate_res":
        B = gate.shape[0]
        out = res + (y.view(B, S, -1) * gate[:, None]).view_as(res)
        return out, y
    return y, None


def matmul_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a[M,N] @ b[N,K]`` (b row-major: the MN-major B operand)."""
    if a.dtype == b.dtype == torch.bfloat16 and _use_native(a.shape[1], b.shape[1], rows=a.shape[0]):
        return ext().gemm_dgrad(a, b)
    return a @ b


def wgrad(dy: torch.Tensor, x: torch.Tensor, main_grad: Optional[torch.Tensor]):
    """``dy[M,N]^T @ x[M,K]``; accumulated (fp32) into ``main_grad`` when given (returns None).

    The output is ``[N, K]``: the tile count depends on N and K only, so a short reduction (the AdaLN
    modulation linear, M = one row per sample) still fills the tensor-core tiles, and the fused fp32
    accumulation into ``main_grad`` replaces a bf16 GEMM plus a separate add."""
    if dy.dtype == x.dtype == torch.bfloat16 and _use_native(dy.shape[1], x.shape[1],
                                                             rows=min(dy.shape[1], x.shape[1])):
        if main_grad is not None:
            ext().gemm_wgrad(dy, x, main_grad, True)
            return None
        out = torch.empty(dy.shape[1], x.shape[1], device=dy.device, dtype=torch.float32)
        ext().gemm_wgrad(dy, x, out, False)
        return out
    g = dy.t() @ x
    if main_grad is not None:
        main_grad.add_(g.view_as(main_grad))
        return None
    return g


def gelu_bwd(dy: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    if _use_native(dy.shape[-1]):
        return ext().gelu_tanh_bwd(dy.contiguous(), pre.contiguous())
    x = pre.float()
    inner = _GELU_C * (x + 0.044715 * x ** 3)
    t = torch.tanh(inner)
    d = 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * _GELU_C * (1 + 3 * 0.044715 * x * x)
    return (dy.float() * d).to(dy.dtype)
