"""Trainer -> rollout weight resharding as one peer-memory copy kernel.

The trainer holds every parameter replicated in its flat bf16 buffer.  A rollout replica on other
GPUs of the node holds its own flat buffer in symmetric memory, possibly tensor-parallel sharded
(``tp`` ranks, each parameter split along dim 0 or dim 1, or replicated).  A *plan* lists the byte
ranges to move: ``(src_off, dst_off, nbytes, dst_slot)`` rows; :func:`push` executes the whole plan
with a single kernel that stores into the peers' mapped buffers over NVLink (``csrc/symm.cu``
``peer_push``), then orders the receivers after it with a one-element all-reduce.

Counterpart of the reference's bucketed ZMQ / NCCL weight transfer
(``verl_omni/workers/engine_workers.py:973-1162``, ``verl_omni/workers/rollout/vllm_rollout/utils.py:81-197``):
there the actor gathers full tensors, casts them and streams 2 GB buckets through IPC; here the
copy plan is computed once and every update is one kernel.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Optional

import torch

_ALIGN = 16  # bytes: the kernel moves 16-byte vectors; every shard starts on this boundary


@dataclass
class ParamSpec:
    name: str
    shape: tuple
    offset: int  # element offset in the trainer's flat buffer
    shard_dim: Optional[int] = None  # None: replicated on every rollout rank; 0 / 1: split across tp ranks


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def rollout_layout(specs: list[ParamSpec], tp: int, elem: int = 2) -> tuple[dict, int]:
    """Byte offset of every parameter's shard in a rollout rank's flat buffer, and the buffer size."""
    off, layout = 0, {}
    for s in specs:
        numel = int(torch.Size(s.shape).numel())
        local = numel if s.shard_dim is None else numel // tp
        layout[s.name] = off
        off += _align(local * elem)
    return layout, off


def plan_tp(specs: list[ParamSpec], tp: int, dst_slots: list[int], elem: int = 2) -> torch.Tensor:
    """Copy plan from the trainer's flat buffer to ``tp`` rollout ranks (``dst_slots[d]`` = peer slot
    of rollout TP rank d).  Dim-0 shards are one contiguous range; dim-1 shards are one range per row."""
    if len(dst_slots) != tp:
        raise ValueError("one destination slot per tensor-parallel rank")
    layout, _ = rollout_layout(specs, tp, elem)
    rows = []
    for s in specs:
        numel = int(torch.Size(s.shape).numel())
        src0 = s.offset * elem
        if (src0 % _ALIGN) != 0:
            raise ValueError(f"{s.name}: trainer offset not 16-byte aligned")
        for d in range(tp):
            dst0 = layout[s.name]
            if s.shard_dim is None:
                rows.append((src0, dst0, numel * elem, dst_slots[d], 0))
            elif s.shard_dim == 0:
                R = s.shape[0]
                if R % tp:
                    raise ValueError(f"{s.name}: dim 0 ({R}) not divisible by tp={tp}")
                per = numel // tp
                rows.append((src0 + d * per * elem, dst0, per * elem, dst_slots[d], 0))
            elif s.shard_dim == 1:
                R, C = s.shape[0], int(torch.Size(s.shape[1:]).numel())
                if s.shape[1] % tp:
                    raise ValueError(f"{s.name}: dim 1 ({s.shape[1]}) not divisible by tp={tp}")
                cs = C // tp
                if (cs * elem) % _ALIGN or (C * elem) % _ALIGN:
                    raise ValueError(f"{s.name}: column shards must be 16-byte multiples")
                for r in range(R):
                    rows.append((src0 + (r * C + d * cs) * elem, dst0 + r * cs * elem, cs * elem, dst_slots[d], 0))
            else:
                raise ValueError(f"{s.name}: unsupported shard_dim {s.shard_dim}")
    return torch.tensor(rows, dtype=torch.int64).reshape(-1, 5)


def plan_replicate(nbytes: int, dst_slots: Iterable[int]) -> torch.Tensor:
    """Whole buffer to every destination (data-parallel rollout replicas)."""
    return torch.tensor([(0, 0, int(nbytes), int(d), 0) for d in dst_slots], dtype=torch.int64).reshape(-1, 5)


def execute_plan_reference(src: torch.Tensor, dsts: list[torch.Tensor], plan: torch.Tensor) -> None:
    """Host restatement of the kernel on byte views (CPU tests)."""
    s8 = src.view(torch.uint8)
    d8 = [d.view(torch.uint8) for d in dsts]
    for so, do, nb, slot, _ in plan.tolist():
        d8[slot][do:do + nb].copy_(s8[so:so + nb])


def push(src: torch.Tensor, dst_ptrs: list[int], plan: torch.Tensor, group=None) -> None:
    """Runs the plan with one kernel, then orders every rank of ``group`` after it."""
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.parallel.symm_mem import stream_barrier

    if src.data_ptr() % _ALIGN:
        raise ValueError("source buffer must be 16-byte aligned")
    ext().peer_push(src.data_ptr(), plan, list(dst_ptrs))
    stream_barrier(group, src.device)
