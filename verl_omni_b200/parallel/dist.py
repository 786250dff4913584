"""Process-group plumbing: one process per GPU (torchrun env) over NCCL, or gloo ranks on CPU.

Collective helpers fall back to gloo-supported primitives (``all_gather`` / ``all_reduce``)
when the tensor-form collectives are not available on the backend.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    backend: Optional[str] = None

    @property
    def is_main(self) -> bool:
        return self.rank == 0


_INFO: Optional[DistInfo] = None


def init_distributed(backend: Optional[str] = None, timeout_s: int = 600, device: Optional[str] = None) -> DistInfo:
    """Initialise from torchrun env vars (RANK/WORLD_SIZE/LOCAL_RANK/MASTER_ADDR/PORT).

    Single-process runs without those vars get a world of one and no process group.
    """
    global _INFO
    if _INFO is not None:
        return _INFO
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = (device or ("cuda" if torch.cuda.is_available() else "cpu")) == "cuda"
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    be = backend or ("nccl" if use_cuda else "gloo")
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = dict(backend=be, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
        if use_cuda:
            kw["device_id"] = dev
        dist.init_process_group(**kw)
    _INFO = DistInfo(rank, world, local, dev, be if world > 1 else None)
    return _INFO


def info() -> DistInfo:
    return _INFO if _INFO is not None else DistInfo()


def set_info(i: DistInfo) -> None:
    global _INFO
    _INFO = i


# group that ``group=None`` resolves to (None: the world).  A process subset that runs a trainer of its own --
# the trainer ranks of a standalone-rollout topology -- sets its group here so the trainer, its engine and
# every collective helper operate on that subset without threading the group through each call.
_DEFAULT_GROUP = None


def set_default_group(group) -> None:
    global _DEFAULT_GROUP
    _DEFAULT_GROUP = group


def default_group():
    return _DEFAULT_GROUP


def _g(group):
    return group if group is not None else _DEFAULT_GROUP


def world_size(group=None) -> int:
    return dist.get_world_size(_g(group)) if dist.is_initialized() else 1


def rank(group=None) -> int:
    return dist.get_rank(_g(group)) if dist.is_initialized() else 0


_HSDP_CACHE: dict = {}


def make_hsdp_groups(fsdp_size: int):
    """(shard_group, replica_group) of this rank: shards are ``fsdp_size`` consecutive ranks, replicas
    the ranks with the same position in their shard group.  Every rank creates every group (the
    collective contract of ``new_group``); results are cached per size."""
    if fsdp_size in _HSDP_CACHE:
        return _HSDP_CACHE[fsdp_size]
    if _DEFAULT_GROUP is not None:
        # new_group is collective over the world: a process subset cannot create sub-groups on its own
        raise NotImplementedError("HSDP / EP / TP sub-groups inside a trainer that runs on a subset of the ranks")
    ws, r = world_size(), rank()
    if ws % fsdp_size:
        raise ValueError(f"world size {ws} not divisible by fsdp_size {fsdp_size}")
    shard = [dist.new_group(list(range(i, i + fsdp_size))) for i in range(0, ws, fsdp_size)]
    rep = [dist.new_group(list(range(j, ws, fsdp_size))) for j in range(fsdp_size)]
    _HSDP_CACHE[fsdp_size] = (shard[r // fsdp_size], rep[r % fsdp_size])
    return _HSDP_CACHE[fsdp_size]


def make_partition_groups(rank_lists) -> object:
    """The group of this rank among a partition of the world into ``rank_lists`` (every rank creates every
    group in the same order, the collective contract of ``new_group``; cached per partition)."""
    key = ("partition", tuple(tuple(int(x) for x in l) for l in rank_lists))
    if key in _HSDP_CACHE:
        return _HSDP_CACHE[key]
    if _DEFAULT_GROUP is not None:
        raise NotImplementedError("sub-groups inside a trainer that runs on a subset of the ranks")
    r, mine = rank(), None
    for l in key[1]:
        g = dist.new_group(list(l))
        if r in l:
            mine = g
    if mine is None:
        raise ValueError(f"rank {r} is in no group of {key[1]}")
    _HSDP_CACHE[key] = mine
    return mine


def barrier(group=None) -> None:
    group = _g(group)
    if dist.is_initialized():
        if dist.get_backend(group) == "nccl":
            dist.barrier(group, device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier(group)


def all_reduce(t: torch.Tensor, op=dist.ReduceOp.SUM, group=None) -> torch.Tensor:
    group = _g(group)
    if dist.is_initialized() and world_size(group) > 1:
        dist.all_reduce(t, op=op, group=group)
    return t


def all_reduce_max(x: float, group=None, device=None) -> float:
    group = _g(group)
    if not dist.is_initialized() or world_size(group) == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def all_gather_into(out: torch.Tensor, shard: torch.Tensor, group=None) -> None:
    """``out`` (flat, world*shard elements) <- concat of every rank's ``shard``."""
    group = _g(group)
    ws = world_size(group)
    if ws == 1:
        if out.data_ptr() != shard.data_ptr():
            out.copy_(shard)
        return
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, shard, group=group)
    else:
        parts = list(out.chunk(ws))
        dist.all_gather(parts, shard.clone(), group=group)


def reduce_scatter_into(shard: torch.Tensor, full: torch.Tensor, group=None, op=dist.ReduceOp.SUM) -> None:
    """``shard`` <- this rank's slice of the element-wise reduction of every rank's ``full``."""
    group = _g(group)
    ws = world_size(group)
    if ws == 1:
        if shard.data_ptr() != full.data_ptr():
            shard.copy_(full)
        return
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(shard, full, op=op, group=group)
    else:
        tmp = full.clone()
        dist.all_reduce(tmp, op=op, group=group)
        shard.copy_(tmp.chunk(ws)[rank(group)])


def all_gather_object(obj, group=None) -> list:
    group = _g(group)
    if not dist.is_initialized() or world_size(group) == 1:
        return [obj]
    out = [None] * world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def broadcast_object(obj, src: int = 0, group=None):
    group = _g(group)
    if not dist.is_initialized() or world_size(group) == 1:
        return obj
    lst = [obj]
    dist.broadcast_object_list(lst, src=src, group=group)
    return lst[0]


def destroy() -> None:
    global _INFO
    if dist.is_initialized():
        dist.destroy_process_group()
    _INFO = None
