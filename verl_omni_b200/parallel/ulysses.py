"""Ulysses sequence parallelism: all-to-all between sequence-sharded and head-sharded attention layouts.

Same scheme as diffusers' ``ContextParallelConfig(ulysses_degree=sp)`` used by the reference
(``verl_omni/workers/engine/fsdp/diffusers_impl.py:175-194,458-462``): every rank holds ``S/sp`` tokens
of each sample; before attention q/k/v go from ``[B, H, S/sp, D]`` to ``[B, H/sp, S, D]`` (all heads
of the local sequence -> local heads of the whole sequence), attention runs on full sequences, and the
token-major output goes back from ``[B, S, H/sp*D]`` to ``[B, S/sp, H*D]``.  The gathered sequence is
ordered by source rank; full (non-causal) attention is invariant to key order and the inverse exchange
restores each rank's queries.

The exchanges are autograd functions (backward = the inverse exchange).  On one node with symmetric
memory each is a single peer-memory kernel that writes the destination layout directly
(``parallel/peer_a2a.py``); otherwise NCCL ``all_to_all_single`` with permute copies around it; gloo has no
all-to-all, so CPU ranks emulate it with an all-gather.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from verl_omni_b200.parallel import dist as D


def _all_to_all(x: torch.Tensor, group) -> torch.Tensor:
    """x [sp, ...] (chunk r goes to rank r) -> [sp, ...] (chunk r came from rank r)."""
    sp = D.world_size(group)
    if sp == 1:
        return x
    x = x.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty_like(x)
        dist.all_to_all_single(out, x, group=group)
        return out
    parts = [torch.empty_like(x) for _ in range(sp)]
    dist.all_gather(parts, x, group=group)
    me = D.rank(group)
    return torch.stack([parts[src][me] for src in range(sp)], 0)


class _SeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        B, H, S, Dh = x.shape
        sp = D.world_size(group)
        if H % sp:
            raise ValueError(f"heads ({H}) must be divisible by the Ulysses degree ({sp})")
        send = x.reshape(B, sp, H // sp, S, Dh).permute(1, 0, 2, 3, 4)  # [sp, B, H/sp, S, D]
        recv = _all_to_all(send, group)  # [sp(src), B, H/sp, S, D]
        return recv.permute(1, 2, 0, 3, 4).reshape(B, H // sp, sp * S, Dh)

    @staticmethod
    def backward(ctx, g):
        B, Hl, St, Dh = g.shape
        sp = D.world_size(ctx.group)
        send = g.reshape(B, Hl, sp, St // sp, Dh).permute(2, 0, 1, 3, 4)  # [sp(dst), B, H/sp, S/sp, D]
        recv = _all_to_all(send, ctx.group)  # [sp(src head slice), B, H/sp, S/sp, D]
        return recv.permute(1, 0, 2, 3, 4).reshape(B, sp * Hl, St // sp, Dh), None


class _HeadToSeq(torch.autograd.Function):
    """token-major [B, S, Hl*D] (sequence ordered by source rank) -> [B, S/sp, H*D]."""

    @staticmethod
    def forward(ctx, o, group, Dh):
        ctx.group, ctx.Dh = group, Dh
        B, St, W = o.shape
        sp = D.world_size(group)
        send = o.reshape(B, sp, St // sp, W).permute(1, 0, 2, 3)  # [sp(dst), B, S/sp, Hl*D]
        recv = _all_to_all(send, group)  # [sp(src head slice), B, S/sp, Hl*D]
        return recv.permute(1, 2, 0, 3).reshape(B, St // sp, sp * W)

    @staticmethod
    def backward(ctx, g):
        B, Sl, Wf = g.shape
        sp = D.world_size(ctx.group)
        W = Wf // sp
        send = g.reshape(B, Sl, sp, W).permute(2, 0, 1, 3)  # [sp(dst head slice), B, S/sp, W]
        recv = _all_to_all(send, ctx.group)  # [sp(src seq chunk), B, S/sp, W]
        return recv.permute(1, 0, 2, 3).reshape(B, sp * Sl, W), None, None


def seq_to_head(x: torch.Tensor, group) -> torch.Tensor:
    from verl_omni_b200.parallel import peer_a2a as PA

    if PA.applies(group, [x]):  # one peer-memory kernel: layout change + NVLink transfer
        return PA.seq_to_head(group, x)[0]
    return _SeqToHead.apply(x, group)


def seq_to_head_many(xs: list, group) -> list:
    """Several [B, H, S/sp, D] tensors through one exchange (q, k and v of one attention)."""
    from verl_omni_b200.parallel import peer_a2a as PA

    if PA.applies(group, xs):
        return list(PA.seq_to_head(group, *xs))
    return [_SeqToHead.apply(x, group) for x in xs]


def head_to_seq(o: torch.Tensor, group, head_dim: int) -> torch.Tensor:
    from verl_omni_b200.parallel import peer_a2a as PA

    if PA.applies(group, [o]):
        return PA.head_to_seq(o, group)
    return _HeadToSeq.apply(o, group, head_dim)


_ORDERS: dict = {}


def segment_major_order(segments: list[int], world: int, device) -> torch.Tensor:
    """Key permutation of a gathered sequence ``[seg0_r0 seg1_r0 .. seg0_r1 seg1_r1 ..]`` (each rank holds
    ``segments[i]`` rows of segment i) into segment-major order ``[seg0_r0 seg0_r1 .. seg1_r0 seg1_r1 ..]``:
    the original token order of every segment, segments one after the other."""
    key = (tuple(segments), world, str(device))
    if key not in _ORDERS:
        sl, idx, off = sum(segments), [], 0
        for n in segments:
            for r in range(world):
                idx.append(torch.arange(r * sl + off, r * sl + off + n))
            off += n
        _ORDERS[key] = torch.cat(idx).to(device)
    return _ORDERS[key]


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group, causal: bool = False,
                      scale: Optional[float] = None, key_mask: Optional[torch.Tensor] = None,
                      kv_len: Optional[torch.Tensor] = None, key_segments: Optional[list] = None) -> torch.Tensor:
    """q/k/v [B, H, S/sp, D] (local tokens, all heads) -> token-major output [B, S/sp, H*D].

    ``key_mask`` [B, S] (optional) marks valid keys in the gathered order (rank-major concatenation of the
    local sequences, see :func:`gather_key_mask`).  ``kv_len`` [B] with ``key_segments`` (rows per rank of
    each segment, e.g. [image, text]) instead counts the valid keys in segment-major order: the gathered
    keys and values are permuted into that order (attention is invariant to a joint key / value
    permutation), which turns right-padded text into a key-count mask the tcgen05 kernels take natively."""
    from verl_omni_b200.ops.attention import attention

    if group is None or D.world_size(group) == 1:
        return attention(q, k, v, causal=causal, scale=scale, key_mask=key_mask, kv_len=kv_len)
    Dh = q.shape[-1]
    qg, kg, vg = seq_to_head_many([q, k, v], group)
    if kv_len is not None:
        order = segment_major_order(list(key_segments), D.world_size(group), k.device)
        kg, vg = kg.index_select(2, order), vg.index_select(2, order)
    o = attention(qg, kg, vg, causal=causal, scale=scale, key_mask=key_mask, kv_len=kv_len)
    return head_to_seq(o, group, Dh)


def joint_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, split: int, *, sp_group=None,
                    kv_len: Optional[torch.Tensor] = None, key_mask: Optional[torch.Tensor] = None):
    """Joint image+text attention of a double-stream block: returns the image rows ``[:split]`` and text rows
    ``[split:]`` of the (local) sequence.  Without sequence parallelism this is the split-output FMHA; with
    it, q/k/v hold this rank's image and text tokens and the exchange runs around a full-sequence attention
    (the gathered sequence is ordered [img_0 txt_0 img_1 txt_1 ...], which full attention does not see)."""
    from verl_omni_b200.ops.attention import attention_split

    if sp_group is None or D.world_size(sp_group) == 1:
        if key_mask is not None:
            from verl_omni_b200.ops.attention import attention

            o = attention(q, k, v, key_mask=key_mask)
            return o[:, :split].contiguous(), o[:, split:].contiguous()
        return attention_split(q, k, v, split, kv_len=kv_len)
    if kv_len is not None and key_mask is None:  # valid keys: every image token, then a prefix of the text
        o = ulysses_attention(q, k, v, sp_group, kv_len=kv_len, key_segments=[split, q.shape[2] - split])
    else:
        o = ulysses_attention(q, k, v, sp_group, key_mask=key_mask)
    return o[:, :split].contiguous(), o[:, split:].contiguous()


def gather_key_mask(local_valid: torch.Tensor, group) -> torch.Tensor:
    """[B, S_local] bool validity of this rank's keys -> [B, S] in the gathered (rank-major) order."""
    if group is None or D.world_size(group) == 1:
        return local_valid
    lv = local_valid.to(torch.uint8).contiguous()
    parts = [torch.empty_like(lv) for _ in range(D.world_size(group))]
    dist.all_gather(parts, lv, group=group)
    return torch.cat(parts, 1).bool()


def sp_info(group) -> tuple[int, int]:
    """(rank, world) inside the sequence-parallel group (0, 1 without one)."""
    if group is None:
        return 0, 1
    return D.rank(group), D.world_size(group)


class _GatherSeq(torch.autograd.Function):
    """All-gather along dim 1 (tokens); backward keeps this rank's slice (every rank's loss is identical)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        sp = D.world_size(group)
        if sp == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(sp)]
        dist.all_gather(parts, x.contiguous(), group=group)
        ctx.n = x.shape[1]
        return torch.cat(parts, 1)

    @staticmethod
    def backward(ctx, g):
        if D.world_size(ctx.group) == 1:
            return g, None
        r = D.rank(ctx.group)
        return g[:, r * ctx.n:(r + 1) * ctx.n].contiguous(), None


def gather_sequence(x: torch.Tensor, group) -> torch.Tensor:
    return _GatherSeq.apply(x, group)


def shard_sequence(x: torch.Tensor, group, dim: int = 1) -> torch.Tensor:
    sp, r = D.world_size(group), D.rank(group)
    if sp == 1:
        return x
    n = x.shape[dim]
    if n % sp:
        raise ValueError(f"sequence length {n} is not divisible by the Ulysses degree {sp}; pad first")
    return x.narrow(dim, r * (n // sp), n // sp)


def pad_to_multiple(x: torch.Tensor, m: int, dim: int = 1) -> torch.Tensor:
    """Zero-pad ``dim`` to a multiple of ``m`` (the reference pads prompt embeds for SP, ``diffusers_impl.py:574-583``)."""
    n = x.shape[dim]
    pad = (-n) % m
    if pad == 0:
        return x
    shape = list(x.shape)
    shape[dim] = pad
    return torch.cat([x, x.new_zeros(shape)], dim)


def make_sp_groups(sp: int):
    """Consecutive ranks form Ulysses groups of size ``sp``; returns (sp_group, dp_group) of this rank."""
    ws, r = D.world_size(), D.rank()
    if sp == 1 or ws == 1:
        return None, None
    if ws % sp:
        raise ValueError(f"world size {ws} not divisible by sp {sp}")
    sp_groups = [dist.new_group(list(range(i, i + sp))) for i in range(0, ws, sp)]
    dp_groups = [dist.new_group(list(range(j, ws, sp))) for j in range(sp)]
    return sp_groups[r // sp], dp_groups[r % sp]


def local_rows(table: torch.Tensor, segments: list[int], group) -> torch.Tensor:
    """Rows of a per-position table (RoPE cos/sin) for this rank's slice of every segment: the table is laid
    out segment after segment (e.g. image tokens then text tokens); each segment is split into ``world``
    equal chunks and the local sequence is the concatenation of this rank's chunk of each segment."""
    r, W = sp_info(group)
    if W == 1:
        return table
    out, off = [], 0
    for n in segments:
        if n % W:
            raise ValueError(f"segment length {n} is not divisible by the Ulysses degree {W}; pad first")
        out.append(table[off + r * (n // W): off + (r + 1) * (n // W)])
        off += n
    return torch.cat(out, 0).contiguous()
