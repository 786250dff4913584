"""Step metrics: data / timing / throughput / MFU (``verl_omni/trainer/diffusion/diffusion_metric_utils.py:25-183``).

Keys follow the reference: ``critic/rewards/*``, ``critic/advantages/*``, ``timing_s/*``,
``timing_per_image_ms/*``, ``perf/throughput`` (= samples / (step time * n_gpus)),
``perf/time_per_step``, ``perf/mfu/actor``.
"""

from __future__ import annotations

import time
from contextlib import contextmanager
from typing import Optional

import numpy as np
import torch


def _stats(prefix: str, x: torch.Tensor) -> dict:
    x = x.detach().float().reshape(-1).cpu()
    return {f"{prefix}/mean": float(x.mean()), f"{prefix}/max": float(x.max()), f"{prefix}/min": float(x.min()),
            f"{prefix}/std": float(x.std()) if x.numel() > 1 else 0.0}


def compute_data_metrics_diffusion(scores: torch.Tensor, advantages: torch.Tensor, uid) -> dict:
    m = {}
    m.update(_stats("critic/rewards", scores))
    m.update(_stats("critic/advantages", advantages))
    # fraction of prompt groups whose rewards are all equal (zero-std groups carry no signal)
    groups: dict = {}
    for s, u in zip(scores.detach().float().cpu().tolist(), list(uid)):
        groups.setdefault(u, []).append(s)
    zero = [float(np.std(v) < 1e-8) for v in groups.values()]
    m["critic/zero_std_group_ratio"] = float(np.mean(zero)) if zero else 0.0
    m["critic/group_size"] = float(np.mean([len(v) for v in groups.values()])) if groups else 0.0
    return m


def compute_timing_metrics_diffusion(timing: dict, n_samples: int) -> dict:
    out = {f"timing_s/{k}": v for k, v in timing.items()}
    for k, v in timing.items():
        out[f"timing_per_image_ms/{k}"] = 1000.0 * v / max(1, n_samples)
    return out


def compute_throughput_metrics_diffusion(step_time: float, n_samples_global: int, n_gpus: int) -> dict:
    return {"perf/time_per_step": step_time, "perf/total_num_samples": n_samples_global,
            "perf/throughput": n_samples_global / max(1e-9, step_time * n_gpus)}


class PhaseTimer:
    """Wall-clock phase timer that synchronises the device at phase boundaries (``marked_timer``)."""

    def __init__(self, device: Optional[torch.device] = None):
        self.device = device
        self.timing: dict = {}

    @contextmanager
    def __call__(self, name: str):
        cuda = self.device is not None and self.device.type == "cuda"
        if cuda:
            torch.cuda.synchronize(self.device)
            torch.cuda.nvtx.range_push(name)  # phase ranges for nsys / ncu range filters
        t0 = time.perf_counter()
        try:
            yield
        finally:
            if cuda:
                torch.cuda.synchronize(self.device)
                torch.cuda.nvtx.range_pop()
            self.timing[name] = self.timing.get(name, 0.0) + time.perf_counter() - t0


def dit_train_flops(n_params: int, tokens: int, attn_layers: int, heads: int, head_dim: int, seq: int,
                    passes: float) -> float:
    """Dense 2*P*tokens per forward + attention 4*L*H*Dh*S^2 per forward, times ``passes``
    (forward = 1, forward+backward = 3): the per-architecture formula of
    ``verl_omni/utils/mfu/diffusion_flops_counter.py:166-179``."""
    dense = 2.0 * n_params * tokens
    attn = 4.0 * attn_layers * heads * head_dim * seq * seq
    return (dense + attn) * passes
