"""Ulysses attention with both all-to-all exchanges fused into the kernels around it (inference path).

The NCCL form of a sequence-parallel attention (``parallel/ulysses.py``) runs QKV GEMM -> 3 all-to-alls
(q, k, v: tokens -> heads) -> attention -> 1 all-to-all (heads -> tokens) -> output projection.  Here:

1. the QKV projection GEMM's epilogue stores every output row/column chunk straight into the symmetric
   buffer of the rank that owns those heads (``csrc/gemm_sm100.cu`` ``EPI_SCATTER``) -- image and text
   token segments of a joint block run as one grouped launch;
2. after a one-element all-reduce orders the ranks, each rank normalises q/k (RMSNorm + RoPE) for its
   heads over the whole sequence from its own buffer;
3. the attention kernel writes every output row into the buffer of the rank that owns the token
   (``csrc/fmha_fwd2_sm100.cu`` peer output), and a second one-element all-reduce orders the ranks;
4. the output projection reads the rank's own buffer.

The destination layout on every rank is block-major by source: ``[W][image rows B x Si | text rows B x St]
x 3*D/W`` (one contiguous ``[B*S, 3D/W]`` matrix per source rank and segment), and the gathered sequence
order is ``[img_0 txt_0 img_1 txt_1 ...]`` as on the NCCL path.

Buffer reuse across layers is safe with one buffer set: a rank's next write into a peer's buffer comes
after an all-reduce that the peer only reaches once it has finished reading that buffer.

Used when gradients are off (rollout / old-log-prob recompute): the returned outputs are views of the
symmetric buffers, valid until the next call.  Counterpart of diffusers' Ulysses context parallelism in
the reference (``verl_omni/workers/engine/fsdp/diffusers_impl.py:175-194,458-462``).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from verl_omni_b200.ops import attention as A
from verl_omni_b200.parallel import dist as D

_WS: dict = {}


def _ext():
    from verl_omni_b200.ops._ext import ext

    return ext()


def enabled(group, x: torch.Tensor, heads: int, hidden: int) -> bool:
    """The fused path applies: CUDA bf16, no autograd, NCCL group on one node, 32-column head slices."""
    if group is None or os.environ.get("VO_ULYSSES_FUSED", "1") == "0":
        return False
    if not (x.is_cuda and x.dtype == torch.bfloat16) or torch.is_grad_enabled():
        return False
    W = D.world_size(group)
    if W < 2 or W > 8 or heads % W or (hidden // W) % 32 or (hidden // heads) not in (64, 128):
        return False
    key = ("ok", id(group))
    if key not in _WS:
        from verl_omni_b200.parallel.symm_mem import available

        _WS[key] = available(group) and hasattr(_ext(), "gemm_scatter") and hasattr(_ext(), "fmha_fwd_peer")
    return _WS[key]


class _Workspace:
    def __init__(self, group, B: int, Si: int, St: int, hidden: int, device):
        from verl_omni_b200.parallel.symm_mem import SymmetricBuffer

        W = D.world_size(group)
        self.W, self.B, self.Si, self.St = W, B, Si, St
        self.Sl = Si + St
        Dg = hidden // W
        self.qkv = SymmetricBuffer(W * B * self.Sl * 3 * Dg, torch.bfloat16, device, group)
        self.o_img = SymmetricBuffer(B * Si * hidden, torch.bfloat16, device, group)
        self.o_txt = SymmetricBuffer(B * St * hidden, torch.bfloat16, device, group) if St else None


def _workspace(group, B, Si, St, hidden, device) -> _Workspace:
    key = (id(group), B, Si, St, hidden, str(device))
    ws = _WS.get(key)
    if ws is None:
        ws = _WS[key] = _Workspace(group, B, Si, St, hidden, device)
    return ws


def gathered_rope(rope: tuple, Si: int, St: int, group) -> tuple:
    """Full-sequence RoPE rows (image rows then text rows) reordered to the gathered order
    [img_0 txt_0 img_1 txt_1 ...]."""
    key = ("rope", id(group), id(rope[0]), Si, St)
    if key not in _WS:
        W = D.world_size(group)
        si, st = Si // W, St // W

        def perm(t):
            parts = []
            for r in range(W):
                parts.append(t[r * si:(r + 1) * si])
                if St:
                    parts.append(t[Si + r * st:Si + (r + 1) * st])
            return torch.cat(parts, 0).contiguous()

        _WS[key] = (perm(rope[0]), perm(rope[1]), rope)  # keep the source alive: the key uses its id
    c, s, _ = _WS[key]
    return c, s


def joint_attention_fused(h_img: torch.Tensor, h_txt: Optional[torch.Tensor], qkv_img, qkv_txt, norms_img: tuple,
                          norms_txt: Optional[tuple], heads: int, group, rope: Optional[tuple] = None,
                          eps: float = 1e-6, scale: Optional[float] = None):
    """Sequence-parallel joint attention of one block with the exchanges in the kernels.

    ``h_img`` [B, Si_l, D] / ``h_txt`` [B, St_l, D] (or None): this rank's normalised tokens; ``qkv_img`` /
    ``qkv_txt``: the fused QKV :class:`~verl_omni_b200.models.layers.Linear` modules; ``norms_*``: (q, k)
    RMSNorm weights; ``rope``: (cos, sin) rows of the full sequence (image rows, then text rows).
    Returns (o_img [B, Si_l, D], o_txt [B, St_l, D] or None) -- views valid until the next call."""
    from verl_omni_b200.ops.norm import qk_norm_split_into
    from verl_omni_b200.parallel.symm_mem import stream_barrier

    e = _ext()
    B, Si, Dm = h_img.shape
    St = h_txt.shape[1] if h_txt is not None else 0
    W, r = D.world_size(group), D.rank(group)
    Dg, Hg, dh = Dm // W, heads // W, Dm // heads
    Sl, S = Si + St, (Si + St) * W
    ws = _workspace(group, B, Si, St, Dm, h_img.device)
    blk = B * Sl * 3 * Dg  # elements of one source rank's block
    rows = W * B * Sl
    # 1. QKV GEMM, epilogue stores into the head owners' buffers
    e.gemm_scatter(h_img.reshape(B * Si, Dm), qkv_img.weight, qkv_img.bias, Si, Si, r * B * Sl,
                   h_txt.reshape(B * St, Dm) if St else None, qkv_txt.weight if St else None,
                   qkv_txt.bias if St else None, max(St, 1), max(St, 1), r * B * Sl + B * Si,
                   ws.qkv.peer_ptrs, Dm, Dg, 3 * Dg, rows)
    stream_barrier(group, h_img.device)
    # 2. q/k RMSNorm + RoPE for this rank's heads over the gathered sequence
    buf = ws.qkv.tensor
    mk = lambda: torch.empty(B, Hg, S, dh, device=h_img.device, dtype=h_img.dtype)  # noqa: E731
    q, k, v = mk(), mk(), mk()
    rope_g = gathered_rope(rope, Si * W, St * W, group) if rope is not None else None
    for src in range(W):
        base = src * blk
        q, k, v = qk_norm_split_into(q, k, v, buf[base:base + B * Si * 3 * Dg].view(B * Si, 3 * Dg), norms_img[0],
                                     norms_img[1], Si, src * Sl, rope=rope_g, eps=eps)
        if St:
            t0 = base + B * Si * 3 * Dg
            q, k, v = qk_norm_split_into(q, k, v, buf[t0:t0 + B * St * 3 * Dg].view(B * St, 3 * Dg), norms_txt[0],
                                         norms_txt[1], St, src * Sl + Si, rope=rope_g, eps=eps)
    # 3. attention; every output row goes to its token's owner
    sc = scale if scale is not None else dh ** -0.5
    e.fmha_fwd_peer(q, k, v, ws.o_img.peer_ptrs, ws.o_txt.peer_ptrs if St else [], Sl, Si, heads, r * Hg, sc,
                    A._kv_version())
    stream_barrier(group, h_img.device)
    o_img = ws.o_img.tensor.view(B, Si, Dm)
    o_txt = ws.o_txt.tensor.view(B, St, Dm) if St else None
    return o_img, o_txt


def release_all() -> None:
    """Frees every workspace (collective over each workspace's group; call on all ranks)."""
    for key in list(_WS):
        ws = _WS.pop(key)
        if isinstance(ws, _Workspace):
            for b in (ws.qkv, ws.o_img, ws.o_txt):
                if b is not None:
                    b.close()
