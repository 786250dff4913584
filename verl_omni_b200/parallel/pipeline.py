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

from typing import Callable, Sequence

import torch
import torch.distributed as dist


class PipelineStage:
    """``fn(x, i)``: this stage's computation of micro-batch ``i`` (``x`` is None on the first stage; the
    last stage returns a scalar loss).  ``act_shape``: shape of the activation entering this stage (and
    leaving the previous one); ``out_shape``: the activation this stage sends on."""

    def __init__(self, fn: Callable, stage: int, n_stages: int, ranks: Sequence[int], act_shape, out_shape,
                 dtype: torch.dtype, device: torch.device):
        self.fn, self.s, self.S = fn, int(stage), int(n_stages)
        self.ranks = list(ranks)  # global rank of every stage
        self.act_shape, self.out_shape = tuple(act_shape or ()), tuple(out_shape or ())
        self.dtype, self.device = dtype, device
        self.p2p_dev = device if dist.get_backend() == "nccl" else torch.device("cpu")
        self._pending: list = []

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

    def run(self, n_micro: int) -> list[torch.Tensor]:
        """One forward + backward over ``n_micro`` micro-batches; returns the last stage's losses (detached)."""
        M = int(n_micro)
        warm = min(self.S - self.s - 1, M)
        saved: dict = {}
        losses = []

        def fwd(i):
            x = None
            if not self.first:
                x = self._recv(self.act_shape, self.s - 1).requires_grad_(True)
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
                g = self._recv(self.out_shape, self.s + 1)
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
        for w, _ in self._pending:
            w.wait()
        self._pending.clear()
        return losses
