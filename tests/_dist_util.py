"""Spawn gloo CPU ranks for multi-process tests (127.0.0.1 rendezvous)."""

import os
import socket

import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, args, device="cpu"):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import torch

    torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))
    from verl_omni_b200.parallel import dist as D

    D.init_distributed(device=device, timeout_s=120)
    try:
        fn(rank, world, *args)
    finally:
        D.destroy()


def run_ranks(fn, world: int = 2, args=(), device: str = "cpu"):
    """``device="cuda"``: one NCCL rank per GPU (rank r on ``cuda:r``)."""
    mp.spawn(_entry, args=(world, free_port(), fn, args, device), nprocs=world, join=True)
