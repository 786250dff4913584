"""Ulysses exchanges as one peer-memory kernel each: the layout change and the NVLink transfer in one pass.

The NCCL form of a Ulysses exchange (``parallel/ulysses.py``) is permute-copy -> ``all_to_all_single`` ->
permute-copy.  Here every rank stores its chunks straight into the final layout of the destination
rank's receive buffer (``csrc/symm.cu`` ``peer_a2a``), one one-element all-reduce orders the ranks, and the
receiver copies its slot out into an ordinary tensor (autograd keeps it).  The four exchanges of a
sequence-parallel attention -- sequence -> heads for q/k/v (one launch for all three) and heads ->
sequence for the output, plus their inverses in backward -- each become one launch.

Job descriptor (all sizes in elements): ``n_i x n_j x n_k`` contiguous chunks of ``len`` elements;
chunk ``(i, j, k)`` is read at ``i*si + j*sj + k*sk`` of the source and written on rank
``(j if rank_dim == 1 else k) // rdiv`` at ``dbase + i*di + j'*dj + k'*dk``, where ``j'``/``k'`` is what
is left of that index after the rank is divided out.

Receive buffers are double-buffered: a rank writes exchange ``n`` into slot ``n % 2`` of its peers; the
peer finished copying slot ``n % 2`` out (exchange ``n - 2``) before the all-reduce that closed exchange
``n - 1``, which the writer has passed, so one all-reduce per exchange suffices.  Ranks must run their
exchanges in the same order (they do: the model is the same on every rank of the group).

Counterpart of the all-to-alls of diffusers' Ulysses context parallelism used by the reference
(``verl_omni/workers/engine/fsdp/diffusers_impl.py:175-194,458-462``).
"""

from __future__ import annotations

import os
from typing import Optional, Sequence

import torch

from verl_omni_b200.parallel import dist as D

_STATE: dict = {}

# job row: src, ni, nj, nk, si, sj, sk, di, dj, dk, dbase, len, rank_dim, rdiv
Job = tuple


def _ext():
    from verl_omni_b200.ops._ext import ext

    return ext()


# ------------------------------------------------------------------------------------------ job builders
def s2h_job(x: torch.Tensor, r: int, W: int, out_off: int) -> Job:
    """x [B, H, S_l, Dh] (this rank's tokens, every head) -> on rank q: [B, H/W, W*S_l, Dh], heads
    [q*H/W, (q+1)*H/W), this rank's tokens at rows [r*S_l, (r+1)*S_l)."""
    B, H, Sl, Dh = x.shape
    Hl = H // W
    L = Sl * Dh
    return (x, B, H, 1, H * L, L, 0, Hl * W * L, W * L, 0, out_off + r * L, L, 1, Hl)


def s2h_bwd_job(g: torch.Tensor, r: int, W: int, out_off: int) -> Job:
    """g [B, H/W, W*S_l, Dh] (this rank's heads, every token) -> on rank q: [B, H, S_l, Dh], rank q's
    tokens, heads [r*H/W, (r+1)*H/W)."""
    B, Hl, S, Dh = g.shape
    Sl = S // W
    L = Sl * Dh
    return (g, B, Hl, W, Hl * S * Dh, S * Dh, L, Hl * W * L, L, 0, out_off + r * Hl * L, L, 2, 1)


def h2s_job(o: torch.Tensor, r: int, W: int, out_off: int) -> Job:
    """o [B, W*S_l, F] (this rank's heads, token-major, F = H/W*Dh) -> on rank q: [B, S_l, W*F], rank q's
    tokens, columns [r*F, (r+1)*F)."""
    B, S, F = o.shape
    Sl = S // W
    return (o, B, S, 1, S * F, F, 0, Sl * W * F, W * F, 0, out_off + r * F, F, 1, Sl)


def h2s_bwd_job(g: torch.Tensor, r: int, W: int, out_off: int) -> Job:
    """g [B, S_l, W*F] (this rank's tokens, every head) -> on rank q: [B, W*S_l, F], columns of rank q's
    heads, this rank's tokens at rows [r*S_l, (r+1)*S_l)."""
    B, Sl, WF = g.shape
    F = WF // W
    return (g, B, Sl, W, Sl * WF, WF, F, W * Sl * F, F, 0, out_off + r * Sl * F, F, 2, 1)


def emulate(jobs_per_rank: Sequence[Sequence[Job]], cap: int) -> list[torch.Tensor]:
    """Host restatement of ``peer_a2a`` on W emulated ranks: returns every rank's receive buffer."""
    W = len(jobs_per_rank)
    recv = [None] * W
    for jobs in jobs_per_rank:
        for (src, ni, nj, nk, si, sj, sk, di, dj, dk, dbase, L, rank_dim, rdiv) in jobs:
            flat = src.reshape(-1)
            if recv[0] is None:
                recv = [torch.zeros(cap, dtype=flat.dtype) for _ in range(W)]
            for i in range(ni):
                for j in range(nj):
                    for k in range(nk):
                        jj, kk = j, k
                        if rank_dim == 1:
                            q, jj = j // rdiv, j % rdiv
                        else:
                            q, kk = k // rdiv, k % rdiv
                        s0 = i * si + j * sj + k * sk
                        d0 = dbase + i * di + jj * dj + kk * dk
                        recv[q][d0:d0 + L] = flat[s0:s0 + L]
    return recv


# ------------------------------------------------------------------------------------------ exchange
class _Slots:
    def __init__(self, group, device):
        self.group, self.device = group, device
        self.bufs: list = [None, None]
        self.turn = 0

    def slot(self, numel: int):
        from verl_omni_b200.parallel.symm_mem import SymmetricBuffer

        b = self.bufs[self.turn]
        if b is None or b.numel < numel:
            # every rank asks for the same size in the same exchange: the (collective) growth stays in step
            if b is not None:
                b.close()
            b = self.bufs[self.turn] = SymmetricBuffer(max(numel, 1 << 20), torch.bfloat16, self.device, self.group)
        self.turn ^= 1
        return b


def enabled(group, *ts: torch.Tensor) -> bool:
    if group is None or os.environ.get("VO_ULYSSES_PEER", "1") == "0":
        return False
    if not all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts):
        return False
    W = D.world_size(group)
    if W < 2 or W > 16:
        return False
    key = ("ok", id(group))
    if key not in _STATE:
        from verl_omni_b200.parallel.symm_mem import available

        _STATE[key] = available(group) and hasattr(_ext(), "peer_a2a")
    return _STATE[key]


def exchange(jobs: Sequence[Job], out_shapes: Sequence[tuple], group) -> list[torch.Tensor]:
    """Runs one exchange (all ``jobs`` in one launch) and returns this rank's received tensors.

    ``out_shapes[t]`` is job t's receive shape; its data sits at element offset ``sum(numel of earlier
    shapes)`` of the slot -- the ``out_off`` the job was built with."""
    from verl_omni_b200.parallel.symm_mem import stream_barrier

    dev = jobs[0][0].device
    key = ("slots", id(group), str(dev))
    if key not in _STATE:
        _STATE[key] = _Slots(group, dev)
    numels = [int(torch.Size(s).numel()) for s in out_shapes]
    total = sum(numels)
    buf = _STATE[key].slot(total)
    rows = torch.tensor([[j[0].data_ptr(), *j[1:]] for j in jobs], dtype=torch.int64)
    _ext().peer_a2a(rows, [j[0].numel() for j in jobs], buf.peer_ptrs, buf.numel)
    stream_barrier(group, dev)  # every rank's chunks have landed
    outs, off = [], 0
    for n, s in zip(numels, out_shapes):
        outs.append(buf.tensor[off:off + n].view(s).clone())
        off += n
    return outs


# ------------------------------------------------------------------------------------------ autograd
class _SeqToHeadPeer(torch.autograd.Function):
    """q/k/v [B, H, S_l, Dh] -> [B, H/W, W*S_l, Dh] each, in one exchange."""

    @staticmethod
    def forward(ctx, group, *xs):
        ctx.group = group
        W, r = D.world_size(group), D.rank(group)
        xs = [x.contiguous() for x in xs]
        jobs, shapes, off = [], [], 0
        for x in xs:
            B, H, Sl, Dh = x.shape
            jobs.append(s2h_job(x, r, W, off))
            shapes.append((B, H // W, W * Sl, Dh))
            off += x.numel()
        return tuple(exchange(jobs, shapes, group))

    @staticmethod
    def backward(ctx, *gs):
        group = ctx.group
        W, r = D.world_size(group), D.rank(group)
        gs = [g.contiguous() for g in gs]
        jobs, shapes, off = [], [], 0
        for g in gs:
            B, Hl, S, Dh = g.shape
            jobs.append(s2h_bwd_job(g, r, W, off))
            shapes.append((B, Hl * W, S // W, Dh))
            off += g.numel()
        return (None, *exchange(jobs, shapes, group))


class _HeadToSeqPeer(torch.autograd.Function):
    """o [B, W*S_l, F] (local heads, token-major) -> [B, S_l, W*F]."""

    @staticmethod
    def forward(ctx, o, group):
        ctx.group = group
        W, r = D.world_size(group), D.rank(group)
        o = o.contiguous()
        B, S, F = o.shape
        return exchange([h2s_job(o, r, W, 0)], [(B, S // W, W * F)], group)[0]

    @staticmethod
    def backward(ctx, g):
        group = ctx.group
        W, r = D.world_size(group), D.rank(group)
        g = g.contiguous()
        B, Sl, WF = g.shape
        return exchange([h2s_bwd_job(g, r, W, 0)], [(B, W * Sl, WF // W)], group)[0], None


def seq_to_head(group, *xs: torch.Tensor) -> tuple:
    return _SeqToHeadPeer.apply(group, *xs)


def head_to_seq(o: torch.Tensor, group) -> torch.Tensor:
    return _HeadToSeqPeer.apply(o, group)


def applies(group, xs: Sequence[torch.Tensor], W: Optional[int] = None) -> bool:
    """Peer path for these tensors: enabled group, 8-element-aligned chunks on both sides."""
    if not enabled(group, *xs):
        return False
    W = W or D.world_size(group)
    for x in xs:
        if x.dim() == 4 and (x.shape[1] % W or (x.shape[2] * x.shape[3]) % 8):
            return False
        if x.dim() == 3 and (x.shape[1] % W or x.shape[2] % 8):
            return False
    return True


def release_all() -> None:
    """Frees the receive buffers (collective over each group; call on all ranks)."""
    for key in list(_STATE):
        v = _STATE.pop(key)
        if isinstance(v, _Slots):
            for b in v.bufs:
                if b is not None:
                    b.close()
