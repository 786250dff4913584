"""Pipeline parallelism: layer stages on consecutive ranks, 1F1B micro-batch schedule over NCCL p2p.

Counterpart of Megatron's pipeline schedule used by the reference's omni Megatron trainer
(``trainer/config/_generated_omni_megatron_trainer.yaml:34-67``: ``pipeline_model_parallel_size``).
Stage ``s`` of ``S`` owns a contiguous slice of the model; micro-batch activations travel forward and
their gradients backward as point-to-point sends between neighbouring stages.  The schedule is 1F1B:
stage ``s`` runs ``S - s - 1`` warm-up forwards, then alternates one forward with one backward, then drains
the remaining backwards, so at most ``S - s`` micro-batches' activations are alive per stage.  Every send
is non-blocking (``isend``) and is waited on only before its buffer could be reused, and every receive is
posted by the stage that needs it next, so neighbouring stages never wait on each other's sends; the
transfers overlap the compute of the following micro-batch.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist


class PipelineStage:
    """``fn(x, i)``: this stage's computation of micro-batch ``i`` (``x`` is None on the first stage; the
    last stage returns a scalar loss).  ``act_shape``: shape of the activation entering this stage (and
    leaving the previous one); ``out_shape``: the activation this stage sends on."""

    def __init__(self, fn: Callable, stage: int, n_stages: int, ranks: Sequence[int], act_shape, out_shape,
                 dtype: torch.dtype, device: torch.device):
        """``act_shape`` / ``out_shape``: a shape, or a callable of the micro-batch index returning one
        (micro-batches of different sizes)."""
        self.fn, self.s, self.S = fn, int(stage), int(n_stages)
        self.ranks = list(ranks)  # global rank of every stage
        self.act_shape = act_shape if callable(act_shape) else tuple(act_shape or ())
        self.out_shape = out_shape if callable(out_shape) else tuple(out_shape or ())
        self.dtype, self.device = dtype, device
        self.p2p_dev = device if dist.get_backend() == "nccl" else torch.device("cpu")
        self._pending: list = []

    def _shape(self, shape, i: int) -> tuple:
        return tuple(shape(i)) if callable(shape) else shape

    @property
    def first(self) -> bool:
        return self.s == 0

    @property
    def last(self) -> bool:
        return self.s == self.S - 1

    def _send(self, t: torch.Tensor, dst_stage: int) -> None:
        buf = t.detach().to(self.p2p_dev, self.dtype).contiguous()
        self._pending.append((dist.isend(buf, self.ranks[dst_stage]), buf))

    def _recv(self, shape, src_stage: int) -> torch.Tensor:
        buf = torch.empty(shape, dtype=self.dtype, device=self.p2p_dev)
        dist.recv(buf, self.ranks[src_stage])
        return buf.to(self.device)

    def forward_only(self, n_micro: int, fn: Optional[Callable] = None) -> list[torch.Tensor]:
        """Forwards of ``n_micro`` micro-batches without autograd (log-prob recomputation); returns the last
        stage's outputs (empty on the other stages)."""
        fn = fn or self.fn
        outs = []
        with torch.no_grad():
            for i in range(int(n_micro)):
                x = None if self.first else self._recv(self._shape(self.act_shape, i), self.s - 1)
                out = fn(x, i)
                if self.last:
                    outs.append(out)
                else:
                    self._send(out, self.s + 1)
        self._drain()
        return outs

    def _drain(self) -> None:
        for w, _ in self._pending:
            w.wait()
        self._pending.clear()

    def run(self, n_micro: int) -> list[torch.Tensor]:
        """One forward + backward over ``n_micro`` micro-batches; returns the last stage's losses (detached)."""
        M = int(n_micro)
        warm = min(self.S - self.s - 1, M)
        saved: dict = {}
        losses = []

        def fwd(i):
            x = None
            if not self.first:
                x = self._recv(self._shape(self.act_shape, i), self.s - 1).requires_grad_(True)
            out = self.fn(x, i)
            if not self.last:
                self._send(out, self.s + 1)
            else:
                losses.append(out.detach())
            saved[i] = (x, out)

        def bwd(i):
            x, out = saved.pop(i)
            if self.last:
                out.backward()
            else:
                g = self._recv(self._shape(self.out_shape, i), self.s + 1)
                out.backward(g)
            if not self.first:
                self._send(x.grad, self.s - 1)

        for i in range(warm):
            fwd(i)
        for i in range(M - warm):
            fwd(warm + i)
            bwd(i)
        for i in range(M - warm, M):
            bwd(i)
        self._drain()
        return losses


class PipeLink:
    """One pipeline stage's point-to-point links and its stage group, for the passes that are not 1F1B:
    the autoregressive decode sends each step's hidden states down the stages and broadcasts the last
    stage's sampled tokens back to all of them."""

    def __init__(self, stage: int, n_stages: int, ranks: Sequence[int], group, device: torch.device):
        self.s, self.S, self.ranks, self.group, self.device = int(stage), int(n_stages), list(ranks), group, device
        self.p2p_dev = device if dist.get_backend(group) == "nccl" else torch.device("cpu")

    @property
    def first(self) -> bool:
        return self.s == 0

    @property
    def last(self) -> bool:
        return self.s == self.S - 1

    def send_next(self, t: torch.Tensor) -> None:
        dist.send(t.detach().to(self.p2p_dev).contiguous(), self.ranks[self.s + 1])

    def recv_prev(self, shape, dtype: torch.dtype) -> torch.Tensor:
        buf = torch.empty(tuple(shape), dtype=dtype, device=self.p2p_dev)
        dist.recv(buf, self.ranks[self.s - 1])
        return buf.to(self.device)

    def bcast_last(self, t: torch.Tensor) -> torch.Tensor:
        """The last stage's ``t`` on every stage (same shape and dtype given everywhere)."""
        buf = t.to(self.p2p_dev).contiguous()
        dist.broadcast(buf, src=self.ranks[-1], group=self.group)
        return buf.to(self.device)


def stage_layers(n_layers: int, n_stages: int, stage: int) -> tuple[int, int]:
    """Layers [lo, hi) of ``stage``: contiguous, sizes differing by at most one (earlier stages larger)."""
    base, extra = divmod(int(n_layers), int(n_stages))
    lo = stage * base + min(stage, extra)
    return lo, lo + base + (1 if stage < extra else 0)
