"""Symmetric device memory across the ranks of one node, and the fused optimizer collective.

A :class:`SymmetricBuffer` is one ``cudaMalloc`` allocation per rank of identical size; each rank
exports a CUDA IPC handle, the handles are exchanged over the process group, and every rank maps
every peer's allocation.  Kernels then read and write peer memory with plain loads and stores that
travel over NVLink/NVSwitch (no copy engine, no NCCL channel).

:func:`fused_optimizer_step` is the sharded engine's step on symmetric buffers: it replaces
``reduce-scatter(main_grad) -> clip -> AdamW -> all-gather(bf16 weights)`` (the FSDP2 step of the
reference's engine, ``verl_omni/workers/engine/diffusers/diffusers_impl.py:412-520``) by two kernels:

1. ``peer_grad_reduce`` - every rank sums its parameter shard of all peers' fp32 ``main_grad``
   buffers with P2P loads and produces the partial squared norm of the reduced shard;
2. ``peer_adamw_bcast`` - after the norm all-reduce, AdamW on the shard (clip / non-finite skip on
   the device) and the bf16 result is stored straight into every peer's flat weight buffer.

Cross-GPU ordering uses one-element all-reduces on the compute stream (no host sync): a rank
reaches the kernel after it only once every rank has enqueued and finished the work before it.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from verl_omni_b200.parallel import dist as D

_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1}


def _ext():
    from verl_omni_b200.ops._ext import ext

    return ext()


def available(group=None) -> bool:
    """Symmetric memory needs CUDA, NCCL and all ranks of the group on this node (IPC reachable)."""
    if not (torch.cuda.is_available() and dist.is_initialized()):
        return False
    if dist.get_backend(group) != "nccl":
        return False
    W = dist.get_world_size(group)
    if W < 2 or W > 16:
        return False
    import socket

    hosts = D.all_gather_object(socket.gethostname(), group)
    return len(set(hosts)) == 1


class SymmetricBuffer:
    """One allocation of ``numel`` elements per rank, mapped on every rank of ``group``."""

    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device, group=None):
        self.numel, self.dtype, self.device, self.group = int(numel), dtype, device, group
        self.world, self.rank = D.world_size(group), D.rank(group)
        nbytes = self.numel * torch.empty((), dtype=dtype).element_size()
        self.ptr, handle, err = None, None, None
        self.peer_ptrs = []
        self._closed = True
        with torch.cuda.device(device):
            try:  # local steps first: a failure here must not leave peers waiting in the exchange
                self.ptr = _ext().symm_malloc(nbytes)
                handle = bytes(_ext().ipc_get_handle(self.ptr).numpy().tobytes())
            except Exception as e:  # noqa: BLE001 - re-raised after the collective
                err = e
            handles = D.all_gather_object(handle, group)
            if err is not None or any(h is None for h in handles):
                if self.ptr is not None:
                    _ext().symm_free(self.ptr)
                raise err or RuntimeError("a peer could not export its symmetric buffer")
            self._closed = False
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.peer_ptrs.append(self.ptr)
                else:
                    self.peer_ptrs.append(_ext().ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
        self.tensor = _ext().tensor_from_ptr(self.ptr, self.numel, _DTYPE_CODE[dtype], device.index or 0)

    def close(self, collective: bool = True) -> None:
        """Unmap peers and free the local allocation.  ``collective``: every rank calls it, and barriers
        keep a peer's memory mapped until no rank can still touch it; ``False`` only before any kernel
        has used the buffer (set-up failure paths)."""
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        if collective:
            D.barrier(self.group)
        for r, p in enumerate(self.peer_ptrs):
            if r != self.rank:
                _ext().ipc_close(p)
        if collective:
            D.barrier(self.group)
        _ext().symm_free(self.ptr)


def stream_barrier(group=None, device: Optional[torch.device] = None) -> None:
    """Orders this rank's stream after every rank's preceding stream work (1-element all-reduce)."""
    t = torch.zeros(1, dtype=torch.float32, device=device or torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t, group=group)


def fused_optimizer_step(flat16: SymmetricBuffer, grad: SymmetricBuffer, lo: int, n: int, master: torch.Tensor,
                         grad_shard: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, *, lr: float,
                         betas: tuple[float, float], eps: float, weight_decay: float, step: int, max_norm: float,
                         group=None) -> torch.Tensor:
    """Reduce-scatter + clip + AdamW + all-gather over peer memory; returns the global grad norm."""
    W = grad.world
    stream_barrier(group, master.device)  # every rank's main_grad is final
    # peer lists start at this rank: at any moment the W ranks read (and write) W different peers
    r = grad.rank
    gptrs = grad.peer_ptrs[r:] + grad.peer_ptrs[:r]
    fptrs = flat16.peer_ptrs[r:] + flat16.peer_ptrs[:r]
    sq = _ext().peer_grad_reduce(gptrs, lo, n, 1.0 / W, grad_shard)
    dist.all_reduce(sq, group=group)  # also orders: every rank finished reading main_grad
    _ext().peer_adamw_bcast(fptrs, lo, n, master, grad_shard, exp_avg, exp_avg_sq, lr,
                            float(betas[0]), float(betas[1]), eps, weight_decay, step, max_norm, sq)
    stream_barrier(group, master.device)  # every peer's weights written before anyone reads them
    return sq.sqrt()


def fused_optimizer_step_reference(flats: list, grads: list, lo: int, n: int, master, exp_avg, exp_avg_sq, *,
                                   lr, betas, eps, weight_decay, step, max_norm, sq_total=None):
    """Host restatement of the two kernels on W emulated ranks' tensors (one rank's shard ``[lo, lo+n)``).

    ``sq_total`` is the all-reduced squared norm (defaults to this shard's own).  Returns the squared
    norm of this shard; updates ``master``/moments in place and writes bf16 results into every
    ``flats[r][lo:lo+n]``.
    """
    W = len(grads)
    g = sum(gr[lo:lo + n].float() for gr in grads) * (1.0 / W)
    sq = float((g.double() ** 2).sum())
    total = sq if sq_total is None else sq_total
    norm = math.sqrt(total)
    if math.isfinite(norm):
        coef = min(1.0, max_norm / (norm + 1e-6)) if max_norm > 0 else 1.0
        g = g * coef
        b1, b2 = betas
        master.mul_(1 - lr * weight_decay)
        exp_avg.mul_(b1).add_(g, alpha=1 - b1)
        exp_avg_sq.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
        master.sub_(lr / bc1 * exp_avg / (exp_avg_sq.sqrt() / math.sqrt(bc2) + eps))
    for f in flats:
        f[lo:lo + n].copy_(master.to(f.dtype))
    return sq
