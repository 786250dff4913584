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


def to_uint8_video(video: torch.Tensor) -> np.ndarray:
    """[3, F, H, W] (or [F, 3, H, W]) in [-1, 1] -> [F, H, W, 3] uint8."""
    v = video.detach().float()
    if v.shape[0] == 3 and v.shape[1] != 3:
        v = v.permute(1, 0, 2, 3)
    return ((v.clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(0, 2, 3, 1).cpu().numpy()


def write_video(stem: str, frames: np.ndarray, fps: int = 24) -> str:
    """``frames`` [F, H, W, 3] uint8 -> ``stem.mp4`` through imageio-ffmpeg when installed (the reference's
    writer), else an animated ``stem.gif`` through PIL, else ``stem.npy``.  Returns the written path."""
    try:
        import imageio.v3 as iio  # optional

        iio.imwrite(stem + ".mp4", frames, fps=fps, codec="libx264")
        return stem + ".mp4"
    except Exception:  # noqa: BLE001 - no ffmpeg writer here: fall back
        pass
    try:
        from PIL import Image

        ims = [Image.fromarray(f) for f in frames]
        ims[0].save(stem + ".gif", save_all=True, append_images=ims[1:], duration=max(1, int(1000 / fps)), loop=0)
        return stem + ".gif"
    except Exception:  # noqa: BLE001
        np.save(stem + ".npy", frames)
        return stem + ".npy"


def write_wav(path: str, audio: torch.Tensor, sample_rate: int) -> str:
    """Mono or [channels, samples] float audio in [-1, 1] -> 16-bit PCM WAV (standard-library ``wave``)."""
    import wave

    a = audio.detach().float().cpu()
    if a.ndim == 1:
        a = a[None]
    pcm = (a.clamp(-1, 1) * 32767.0).round().to(torch.int16).t().contiguous().numpy()  # interleaved
    with wave.open(path, "wb") as w:
        w.setnchannels(a.shape[0])
        w.setsampwidth(2)
        w.setframerate(int(sample_rate))
        w.writeframes(pcm.tobytes())
    return path


def dump_media_generations(path: str, step: int, prompts: list, scores: list, *,
                           images: Optional[torch.Tensor] = None, videos: Optional[torch.Tensor] = None,
                           audios: Optional[list] = None, sample_rates: Optional[list] = None,
                           fps: int = 24) -> str:
    """Rollout / validation dump with video (mp4 / gif) and audio (wav) next to the JSONL record, the media
    side of the reference's ``_dump_generations`` (``utils/tracking.py:74-186``)."""
    fn = dump_generations(path, step, images, prompts, scores)
    rows = [json.loads(ln) for ln in open(fn)]
    for i, rec in enumerate(rows):
        stem = os.path.join(path, f"step{step}_{i}")
        if videos is not None:
            rec["video"] = write_video(stem, to_uint8_video(videos[i]), fps)
        if audios is not None and audios[i] is not None:
            sr = int(sample_rates[i]) if sample_rates is not None else 16000
            rec["audio"] = write_wav(stem + ".wav", torch.as_tensor(audios[i]), sr)
    with open(fn, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
    return fn
