"""Mixture-of-experts SwiGLU on expert-grouped tcgen05 GEMMs.

Routing produces ``T x top_k`` (token, expert) pairs.  The dispatch sorts them by expert and lays them out
in one buffer where every expert's rows start on a 128-row boundary and the gap rows are zero; then each
128-row tile belongs to exactly one expert and a single persistent GEMM launch covers all experts:

* forward / dgrad: ``csrc/gemm_sm100.cu`` grouped mode 1 -- the B tile rows are offset by the tile's expert
  (weights stacked ``[E, N, K]``), unused tiles of the upper-bound buffer are skipped on the device;
* weight gradient: grouped mode 2 -- work units are (expert, output tile), each reducing over its expert's
  row range only, straight into the fp32 ``main_grad`` of the stacked weight.

Everything is computed on the device (counts, offsets, tile table): no host synchronisation per layer.
Counterpart of the expert loop of the reference's MoE thinker (vLLM / Megatron fused MoE, and the unfused
per-expert loop of ``verl_omni/models/transformers/qwen3_omni_thinker.py:246-276``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

TILE = 128


def _ext():
    from verl_omni_b200.ops._ext import ext

    return ext()


@dataclass
class DispatchPlan:
    tok: torch.Tensor          # [P] source token of each sorted pair
    dst: torch.Tensor          # [P] padded row of each sorted pair
    order: torch.Tensor        # [P] sorted pair -> flat (token, slot) index
    seg: torch.Tensor          # [E + 1] int32 padded row offsets of the experts
    tile_expert: torch.Tensor  # [Mp / 128] int32 expert of each row tile (-1: unused)
    rows: int                  # Mp (upper bound of the padded rows)


def plan_dispatch(idx: torch.Tensor, n_experts: int) -> DispatchPlan:
    """Device-side sort-by-expert with 128-row padding per expert (``idx`` [T, K] expert ids)."""
    T, K = idx.shape
    P = T * K
    dev = idx.device
    flat_e = idx.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    sorted_e = flat_e[order]
    # scatter-add count (bincount reads the maximum id back to the host to size its output)
    counts = torch.zeros(n_experts, dtype=torch.int64, device=dev).scatter_add_(0, flat_e, torch.ones_like(flat_e))
    padded = (counts + TILE - 1) // TILE * TILE
    seg = torch.zeros(n_experts + 1, dtype=torch.int64, device=dev)
    seg[1:] = torch.cumsum(padded, 0)
    first = torch.cumsum(counts, 0) - counts  # first sorted position of each expert
    rank_in = torch.arange(P, device=dev) - first[sorted_e]
    dst = seg[sorted_e] + rank_in
    rows = (P + n_experts * (TILE - 1) + TILE - 1) // TILE * TILE
    tile_start = torch.arange(0, rows, TILE, device=dev)
    te = torch.searchsorted(seg[1:], tile_start, right=True)
    tile_expert = torch.where(tile_start < seg[-1], te, torch.full_like(te, -1)).to(torch.int32)
    tok = torch.arange(T, device=dev).repeat_interleave(K)[order]
    return DispatchPlan(tok, dst, order, seg.to(torch.int32), tile_expert, rows)


def _accum(param: torch.Tensor, grad32: torch.Tensor):
    mg = getattr(param, "main_grad", None)
    if mg is None:
        return grad32.to(param.dtype)
    mg.add_(grad32.view_as(mg))
    return None


class _ExpertFFN(torch.autograd.Function):
    """SwiGLU experts on expert-sorted padded rows: y = (silu(x Wg^T) * (x Wu^T)) Wd^T per row's expert."""

    @staticmethod
    def forward(ctx, xs, w_gate_up, w_down, tile_expert, seg):
        e = _ext()
        gu = e.moe_gemm_fwd(xs, w_gate_up, tile_expert)  # [Mp, 2F]
        a = e.swiglu_fwd(gu)  # silu(gate) * up, bf16 (one pass)
        y = e.moe_gemm_fwd(a, w_down, tile_expert)  # [Mp, D]
        ctx.save_for_backward(xs, gu, a, w_gate_up, w_down, tile_expert, seg)
        return y

    @staticmethod
    def backward(ctx, dy):
        xs, gu, a, w_gate_up, w_down, tile_expert, seg = ctx.saved_tensors
        e = _ext()
        dy = dy.contiguous()
        da = e.moe_gemm_dgrad(dy, w_down, tile_expert)  # [Mp, F]
        gd = None
        mg = getattr(w_down, "main_grad", None)
        if mg is not None:
            e.moe_gemm_wgrad(dy, a, seg, mg.view(w_down.shape), True)
        else:
            buf = torch.zeros(w_down.shape, device=dy.device, dtype=torch.float32)
            e.moe_gemm_wgrad(dy, a, seg, buf, True)
            gd = buf.to(w_down.dtype)
        dgu = e.swiglu_bwd(da, gu)  # d(gate | up) in one pass
        dxs = e.moe_gemm_dgrad(dgu, w_gate_up, tile_expert)
        ggu = None
        mg = getattr(w_gate_up, "main_grad", None)
        if mg is not None:
            e.moe_gemm_wgrad(dgu, xs, seg, mg.view(w_gate_up.shape), True)
        else:
            buf = torch.zeros(w_gate_up.shape, device=dy.device, dtype=torch.float32)
            e.moe_gemm_wgrad(dgu, xs, seg, buf, True)
            ggu = buf.to(w_gate_up.dtype)
        return dxs, ggu, gd, None, None


def native_ok(h: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> bool:
    """The grouped kernels need bf16 CUDA tensors and 128-multiple expert widths (weight-gradient tiles)."""
    if not (h.is_cuda and h.dtype == torch.bfloat16 and w_gate_up.dtype == torch.bfloat16):
        return False
    D, F2 = h.shape[-1], w_gate_up.shape[1]
    return D % 128 == 0 and F2 % 256 == 0 and hasattr(_ext(), "moe_gemm_fwd")


def moe_ffn(h: torch.Tensor, idx: torch.Tensor, gates: torch.Tensor, w_gate_up: torch.Tensor,
            w_down: torch.Tensor) -> torch.Tensor:
    """Top-k routed SwiGLU experts: ``h`` [T, D], ``idx`` / ``gates`` [T, K], ``w_gate_up`` [E, 2F, D],
    ``w_down`` [E, D, F]; returns [T, D] = sum_k gates[:, k] * expert_{idx[:, k]}(h)."""
    E = w_gate_up.shape[0]
    plan = plan_dispatch(idx, E)
    xs = h.new_zeros(plan.rows, h.shape[1])
    xs = xs.index_copy(0, plan.dst, h.index_select(0, plan.tok))
    y = _ExpertFFN.apply(xs, w_gate_up, w_down, plan.tile_expert, plan.seg)
    w = gates.reshape(-1)[plan.order].unsqueeze(-1)
    out = torch.zeros_like(h)
    return out.index_add(0, plan.tok, (y.index_select(0, plan.dst) * w).to(h.dtype))


def moe_ffn_local(h: torch.Tensor, idx: torch.Tensor, gates: torch.Tensor, w_gate_up: torch.Tensor,
                  w_down: torch.Tensor, e0: int) -> torch.Tensor:
    """The contribution of this rank's experts [e0, e0 + El) to ``sum_k gates[:, k] expert_{idx[:, k]}(h)``,
    with every other slot dropped on the device (no host synchronisation).

    Slots of other ranks' experts are sorted into a sink segment whose tiles are marked -1, which the
    grouped GEMM skips; their rows are excluded with ``where`` (the skipped rows hold no values)."""
    El = w_gate_up.shape[0]
    loc = (idx >= e0) & (idx < e0 + El)
    lidx = torch.where(loc, idx - e0, torch.full_like(idx, El))
    plan = plan_dispatch(lidx, El + 1)
    tile_expert = torch.where(plan.tile_expert >= El, torch.full_like(plan.tile_expert, -1), plan.tile_expert)
    xs = h.new_zeros(plan.rows, h.shape[1])
    xs = xs.index_copy(0, plan.dst, h.index_select(0, plan.tok))
    y = _ExpertFFN.apply(xs, w_gate_up, w_down, tile_expert, plan.seg)
    keep = loc.reshape(-1)[plan.order].unsqueeze(-1)
    w = gates.reshape(-1)[plan.order].unsqueeze(-1).float()
    contrib = torch.where(keep, y.index_select(0, plan.dst).float() * w, torch.zeros((), device=h.device))
    return torch.zeros(h.shape, dtype=torch.float32, device=h.device).index_add(0, plan.tok, contrib)


def moe_ffn_local_reference(h, idx, gates, w_gate_up, w_down, e0: int) -> torch.Tensor:
    El = w_gate_up.shape[0]
    loc = (idx >= e0) & (idx < e0 + El)
    return moe_ffn_reference(h, torch.where(loc, idx - e0, 0), torch.where(loc, gates, torch.zeros_like(gates)),
                             w_gate_up, w_down)


def moe_ffn_reference(h, idx, gates, w_gate_up, w_down) -> torch.Tensor:
    """fp32 per-expert loop (oracle)."""
    out = torch.zeros(h.shape, dtype=torch.float32, device=h.device)
    for e in range(w_gate_up.shape[0]):
        tk, sl = (idx == e).nonzero(as_tuple=True)
        if tk.numel() == 0:
            continue
        x = h[tk].float()
        g, u = (x @ w_gate_up[e].float().t()).chunk(2, -1)
        y = (F.silu(g) * u) @ w_down[e].float().t()
        out.index_add_(0, tk, y * gates[tk, sl].float().unsqueeze(-1))
    return out
