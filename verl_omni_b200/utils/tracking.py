"""Experiment tracking and media dumps (``verl_omni/utils/tracking.py:31-186``, verl ``Tracking``).

Backends: ``console`` (one JSON line per step), ``jsonl`` (file), ``tensorboard`` (when importable),
``wandb`` (when importable; skipped otherwise).  ``dump_generations`` writes rollout images as PNG
(via PIL when available, else raw ``.npy``) next to a JSONL of prompts / scores, like the
reference's rollout/validation dumps.
"""

from __future__ import annotations

import json
import logging
import os
from typing import Iterable, Optional

import numpy as np
import torch

_log = logging.getLogger(__name__)


class Tracking:
    def __init__(self, project_name: str, experiment_name: str, default_backend: Iterable[str] = ("console",),
                 log_dir: str = "logs", config: Optional[dict] = None):
        self.backends = list(default_backend)
        self.dir = os.path.join(log_dir, project_name, experiment_name)
        self._jsonl = None
        self._tb = None
        self._wandb = None
        if "jsonl" in self.backends:
            os.makedirs(self.dir, exist_ok=True)
            self._jsonl = open(os.path.join(self.dir, "metrics.jsonl"), "a")
        if "tensorboard" in self.backends:
            try:
                from torch.utils.tensorboard import SummaryWriter

                self._tb = SummaryWriter(self.dir)
            except Exception as e:  # noqa: BLE001
                _log.warning("tensorboard unavailable: %s", e)
        if "wandb" in self.backends:
            try:
                import wandb

                self._wandb = wandb.init(project=project_name, name=experiment_name, config=config or {})
            except Exception as e:  # noqa: BLE001
                _log.warning("wandb unavailable: %s", e)

    def log(self, data: dict, step: int) -> None:
        clean = {k: (float(v) if isinstance(v, (int, float, np.floating)) else v) for k, v in data.items()
                 if isinstance(v, (int, float, np.floating, str))}
        if "console" in self.backends:
            print(json.dumps({"step": step, **{k: (round(v, 6) if isinstance(v, float) else v)
                                                for k, v in clean.items()}}), flush=True)
        if self._jsonl is not None:
            self._jsonl.write(json.dumps({"step": step, **clean}) + "\n")
            self._jsonl.flush()
        if self._tb is not None:
            for k, v in clean.items():
                if isinstance(v, float):
                    self._tb.add_scalar(k, v, step)
        if self._wandb is not None:
            self._wandb.log(clean, step=step)

    def finish(self) -> None:
        if self._jsonl is not None:
            self._jsonl.close()
        if self._tb is not None:
            self._tb.close()


def to_uint8_images(images: torch.Tensor) -> np.ndarray:
    """[B, 3, H, W] in [-1, 1] -> [B, H, W, 3] uint8."""
    return ((images.detach().float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(0, 2, 3, 1).cpu().numpy()


def dump_generations(path: str, step: int, images: Optional[torch.Tensor], prompts: list, scores: list) -> str:
    os.makedirs(path, exist_ok=True)
    rows = []
    u8 = to_uint8_images(images) if images is not None else None
    for i, (p, s) in enumerate(zip(prompts, scores)):
        rec = {"step": step, "index": i, "prompt": str(p), "score": float(s)}
        if u8 is not None:
            stem = os.path.join(path, f"step{step}_{i}")
            try:
                from PIL import Image

                Image.fromarray(u8[i]).save(stem + ".png")
                rec["image"] = stem + ".png"
            except Exception:  # noqa: BLE001
                np.save(stem + ".npy", u8[i])
                rec["image"] = stem + ".npy"
        rows.append(rec)
    fn = os.path.join(path, f"{step}.jsonl")
    with open(fn, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
    return fn
