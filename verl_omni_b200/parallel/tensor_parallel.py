"""Megatron-style tensor parallelism with sequence parallelism, collectives fused into the GEMMs.

Layout (Megatron TP + SP, the reference's ``strategy: megatron`` engine for the Qwen3-Omni thinker,
``trainer/config/_generated_omni_megatron_trainer.yaml:34-67``): between layers every rank holds ``S / tp``
tokens of the sequence; a column-parallel linear needs the whole sequence (all-gather, then GEMM with this
rank's output columns) and a row-parallel linear produces partial sums of the whole sequence that are
reduce-scattered back to the token owners.

Fused path (CUDA, NCCL group on one node, symmetric memory; ``VO_TP_FUSED``, default ``1``):

* all-gather -> GEMM: each rank publishes its token shard in a symmetric buffer.  The GEMM on the rank's
  own rows starts at once while the copy engine pulls the peers' shards over NVLink on a side stream, one
  event per peer, so each shard crosses NVLink once and its GEMM starts as soon as it has landed (the
  pull of the next shard overlaps the GEMM on the previous one).  ``VO_TP_FUSED=kernel`` instead lets the
  GEMM's TMA producer read every A tile straight from the owning peer (``GemmDesc::gather`` 1; the weight
  gradients ``gather`` 2 / 3): no staging copy, but every output column tile re-reads its A tiles across
  NVLink, which costs more than the copy at the layer sizes measured;
* GEMM -> reduce-scatter: the epilogue stores each output row, in bf16 with plain 16-byte stores over
  NVLink, into this rank's slot of the owner's buffer (``EPI_PEER_RED`` slot mode); after a one-element
  all-reduce orders the ranks the owner sums its slots (``slot_sum``, bias fused).  The dgrad of a
  column-parallel layer uses the same epilogue; the dgrad / wgrad of a row-parallel layer consume the
  gathered output gradient chunk by chunk like the forward of a column-parallel layer.

Reference path (CPU / gloo, or when the fused path does not apply): all-gather and reduce-scatter as
collectives around plain GEMMs -- numerically the oracle of the fused path.

Symmetric buffers come in pairs used alternately: a rank rewrites a buffer only after an all-reduce that
every peer reaches once it has finished reading that buffer's previous contents.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from verl_omni_b200.parallel import dist as D


def _ext():
    from verl_omni_b200.ops._ext import ext

    return ext()


# ---------------------------------------------------------------- reference collectives
def all_gather_seq(x: torch.Tensor, group) -> torch.Tensor:
    """[S_l, C] shards -> [S, C] (rank-major)."""
    W = D.world_size(group)
    if W == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(W)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, 0)


def reduce_scatter_seq(y: torch.Tensor, group) -> torch.Tensor:
    """[S, C] partial sums -> this rank's [S / W, C] rows of the sum."""
    W = D.world_size(group)
    if W == 1:
        return y
    t = y.float().contiguous()
    dist.all_reduce(t, group=group)  # gloo has no reduce-scatter; the reference path sums everywhere
    r = D.rank(group)
    n = y.shape[0] // W
    return t[r * n:(r + 1) * n].to(y.dtype)


# ---------------------------------------------------------------- fused workspace
class _Pair:
    """Two symmetric buffers of one size, handed out alternately."""

    def __init__(self, numel: int, dtype, device, group):
        from verl_omni_b200.parallel.symm_mem import SymmetricBuffer

        self.bufs = [SymmetricBuffer(numel, dtype, device, group) for _ in range(2)]
        for b in self.bufs:  # defined contents before first use (cudaMalloc does not clear)
            b.tensor.zero_()
        torch.cuda.synchronize(device)
        D.barrier(group)
        self.i = 0

    def next(self):
        b = self.bufs[self.i]
        self.i ^= 1
        return b


class TPContext:
    """Tensor-parallel group + the symmetric buffers of its fused collectives."""

    def __init__(self, group):
        self.group = group
        self.world, self.rank = D.world_size(group), D.rank(group)
        self._pairs: dict = {}
        self._fused: Optional[bool] = None
        self._side: Optional[torch.cuda.Stream] = None

    def fused(self, t: torch.Tensor) -> bool:
        if os.environ.get("VO_TP_FUSED", "1") == "0" or self.world < 2 or self.world > 8:
            return False
        if not (t.is_cuda and t.dtype == torch.bfloat16):
            return False
        if self._fused is None:
            from verl_omni_b200.parallel.symm_mem import available

            self._fused = available(self.group) and hasattr(_ext(), "gemm_tp")
        return self._fused

    def buf(self, key: str, numel: int, dtype, device):
        k = (key, numel, dtype, str(device))
        if k not in self._pairs:
            self._pairs[k] = _Pair(numel, dtype, device, self.group)
        return self._pairs[k].next()

    @staticmethod
    def in_kernel_gather() -> bool:
        return os.environ.get("VO_TP_FUSED", "1") == "kernel"

    def side_stream(self, device) -> torch.cuda.Stream:
        if self._side is None:
            self._side = torch.cuda.Stream(device)
        return self._side

    def barrier(self, device) -> None:
        from verl_omni_b200.parallel.symm_mem import stream_barrier

        stream_barrier(self.group, device)

    def publish(self, key: str, x: torch.Tensor):
        """Copies this rank's shard into a symmetric buffer and orders the ranks: peers may read it."""
        b = self.buf(key, x.numel(), x.dtype, x.device)
        b.tensor.view_as(x).copy_(x)
        self.barrier(x.device)
        return b

    def release(self) -> None:
        for p in self._pairs.values():
            for b in p.bufs:
                b.close()
        self._pairs.clear()


def _fused_ok(ctx: TPContext, x: torch.Tensor, *dims: int) -> bool:
    return ctx.fused(x) and all(d % 128 == 0 for d in dims)


def _gathered_chunks(tp: TPContext, key: str, x: torch.Tensor, consume) -> None:
    """All-gather overlapped with its consumer: publishes ``x`` [S_l, C], then calls ``consume(p, chunk)``
    for every rank p, own shard first, then each peer's shard once the copy engine has pulled it into this
    GPU's memory (side stream, one event per peer)."""
    xb = tp.publish(key, x)
    W, r = tp.world, tp.rank
    main = torch.cuda.current_stream(x.device)
    side = tp.side_stream(x.device)
    side.wait_stream(main)  # after the barrier: every peer's shard is published
    peers = [(r + j) % W for j in range(1, W)]
    staged = torch.empty((W - 1,) + tuple(x.shape), device=x.device, dtype=x.dtype)
    nbytes = x.numel() * x.element_size()
    events = []
    with torch.cuda.stream(side):
        for j, p in enumerate(peers):
            _ext().peer_copy(staged[j], xb.peer_ptrs[p], nbytes)
            ev = torch.cuda.Event()
            ev.record(side)
            events.append(ev)
    consume(r, x)
    for j, p in enumerate(peers):
        main.wait_event(events[j])
        consume(p, staged[j])


def _gemm_ag(ctx: TPContext, xb, S_l: int, K: int, w: torch.Tensor, bias) -> torch.Tensor:
    """y[S, N] = gather(x)[S, K] W^T with the A tiles read from the peers' published shards."""
    S, N = S_l * ctx.world, w.shape[0]
    y = torch.empty(S, N, device=w.device, dtype=w.dtype)
    _ext().gemm_tp(None, w, S, N, K, K, K, 0, 0, y, None, bias, 1, xb.peer_ptrs, S_l, [], 0)
    return y


def _reduce_to_owner(ctx: TPContext, key: str, S: int, N: int, launch, bias=None) -> torch.Tensor:
    """Runs ``launch(red_ptrs, rows, slot)`` (a GEMM whose epilogue stores every output row, in bf16, into
    this rank's slot of the owning rank's buffer ``[world, S / world, N]``), orders the ranks and returns
    the sum of this rank's slots (+ ``bias``).  Every slot is rewritten in full by each use, so the buffers
    need no clearing; the partial sums are rounded to bf16 before the fp32 sum, as a bf16 reduce-scatter
    rounds them."""
    S_l = S // ctx.world
    slots = ctx.buf(key, ctx.world * S_l * N, torch.bfloat16, torch.device("cuda", torch.cuda.current_device()))
    launch(slots.peer_ptrs, S_l, ctx.rank)
    ctx.barrier(slots.tensor.device)
    return _ext().slot_sum(slots.tensor.view(ctx.world * S_l, N), ctx.world, bias)


# ---------------------------------------------------------------- autograd functions
class _ColumnParallel(torch.autograd.Function):
    """x shard [S_l, K] -> y [S, N_l] = all_gather(x) W_l^T (+ b_l)."""

    @staticmethod
    def forward(ctx, x, w, b, tp: TPContext):
        ctx.tp = tp
        S_l, K = x.shape
        if _fused_ok(tp, x, S_l, K, w.shape[0]):
            N_l = w.shape[0]
            if tp.in_kernel_gather():
                y = _gemm_ag(tp, tp.publish("col_x", x), S_l, K, w, b)
            else:
                y = torch.empty(S_l * tp.world, N_l, device=x.device, dtype=x.dtype)
                _gathered_chunks(tp, "col_x", x.contiguous(), lambda p, xc: _ext().gemm_tp(
                    xc, w, S_l, N_l, K, K, K, 0, 0, y[p * S_l:(p + 1) * S_l], None, b, 0, [], 0, [], 0))
            ctx.fused = True
        else:
            y = torch.nn.functional.linear(all_gather_seq(x, tp.group), w, b)
            ctx.fused = False
        ctx.save_for_backward(x, w)
        ctx.has_b = b is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        tp = ctx.tp
        dy = dy.contiguous()
        S, N_l = dy.shape
        S_l, K = x.shape
        gb = dy.float().sum(0).to(w.dtype) if ctx.has_b else None
        if ctx.fused:
            # dX: partial over this rank's output columns, reduce-scattered by the dgrad epilogue
            dx = _reduce_to_owner(tp, "col_dx", S, K, lambda red, rows, slot: _ext().gemm_tp(
                dy, w, S, K, N_l, N_l, K, 0, 1, None, None, None, 0, [], 0, red, rows, slot))
            # dW = dY^T gather(x): the reduction over tokens reads every peer's x shard again
            gw = torch.zeros(N_l, K, device=w.device, dtype=torch.float32)
            if tp.in_kernel_gather():
                xb = tp.publish("col_x", x)
                _ext().gemm_tp(dy, None, N_l, K, S, N_l, K, 1, 1, None, gw, None, 3, xb.peer_ptrs, S_l, [], 0)
            else:
                _gathered_chunks(tp, "col_x", x.contiguous(), lambda p, xc: _ext().gemm_tp(
                    dy[p * S_l:(p + 1) * S_l], xc, N_l, K, S_l, N_l, K, 1, 1, None, gw, None, 0, [], 0, [], 0))
            return dx, gw.to(w.dtype), gb, None
        xg = all_gather_seq(x, tp.group)
        dx = reduce_scatter_seq(dy @ w, tp.group)
        return dx, (dy.t().float() @ xg.float()).to(w.dtype), gb, None


class _RowParallel(torch.autograd.Function):
    """x [S, K_l] -> y shard [S_l, N] = reduce_scatter(x W_l^T) (+ b)."""

    @staticmethod
    def forward(ctx, x, w, b, tp: TPContext):
        ctx.tp = tp
        S, K_l = x.shape
        N = w.shape[0]
        if _fused_ok(tp, x, S // max(tp.world, 1), K_l, N) and S % tp.world == 0:
            y = _reduce_to_owner(tp, "row_y", S, N, lambda red, rows, slot: _ext().gemm_tp(
                x, w, S, N, K_l, K_l, K_l, 0, 0, None, None, None, 0, [], 0, red, rows, slot), bias=b)
            ctx.fused = True
        else:
            y = reduce_scatter_seq(torch.nn.functional.linear(x, w), tp.group)
            if b is not None:
                y = y + b
            ctx.fused = False
        ctx.save_for_backward(x, w)
        ctx.has_b = b is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        tp = ctx.tp
        dy = dy.contiguous()
        S_l, N = dy.shape
        S, K_l = x.shape
        gb = dy.float().sum(0) if ctx.has_b else None
        if gb is not None:  # every rank's bias gradient covers only its tokens: sum them
            dist.all_reduce(gb, group=tp.group)
            gb = gb.to(w.dtype)
        if ctx.fused:
            x = x.contiguous()
            dx = torch.empty(S, K_l, device=x.device, dtype=x.dtype)
            gw = torch.zeros(N, K_l, device=w.device, dtype=torch.float32)
            if tp.in_kernel_gather():
                yb = tp.publish("row_dy", dy)
                # dX = gather(dY) W_l: A tiles from the peers' dY shards
                _ext().gemm_tp(None, w, S, K_l, N, N, K_l, 0, 1, dx, None, None, 1, yb.peer_ptrs, S_l, [], 0)
                # dW = gather(dY)^T x: the reduction over tokens reads the peers' dY shards
                _ext().gemm_tp(None, x, N, K_l, S, N, K_l, 1, 1, None, gw, None, 2, yb.peer_ptrs, S_l, [], 0)
            else:
                def consume(p, dyc):  # rows of rank p: dX rows = dY_p W_l, dW += dY_p^T x_p
                    _ext().gemm_tp(dyc, w, S_l, K_l, N, N, K_l, 0, 1, dx[p * S_l:(p + 1) * S_l], None, None, 0,
                                   [], 0, [], 0)
                    _ext().gemm_tp(dyc, x[p * S_l:(p + 1) * S_l], N, K_l, S_l, N, K_l, 1, 1, None, gw, None, 0,
                                   [], 0, [], 0)

                _gathered_chunks(tp, "row_dy", dy, consume)
            return dx, gw.to(w.dtype), gb, None
        dyg = all_gather_seq(dy, tp.group)
        return (dyg @ w).to(x.dtype), (dyg.t().float() @ x.float()).to(w.dtype), gb, None


def column_parallel_linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], tp: TPContext):
    """Sequence-sharded x [S_l, K] -> full-sequence output columns of this rank [S, N_l]."""
    return _ColumnParallel.apply(x, w, b, tp)


def row_parallel_linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], tp: TPContext):
    """Full-sequence input columns of this rank [S, K_l] -> sequence-sharded output [S_l, N]."""
    return _RowParallel.apply(x, w, b, tp)
