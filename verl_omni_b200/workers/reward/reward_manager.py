"""Reward managers and scorers.

* ``VisualRewardManager`` (``verl_omni/reward_loop/reward_manager/visual.py:39-120``): validates the
  rollout payload (decoded images in [-1,1] / uint8, or latents) and calls a registered scorer.
* ``MultiVisualRewardManager`` (``multi.py:49-191``): weighted sum of sub-rewards; a failing
  ``required`` sub-reward raises, an optional one contributes 0 and is counted in the metrics.
* Scorers: ``mlp_latent`` (frozen MLP on mean-pooled latents), ``vit`` / ``vit_video`` (frozen
  ViT-B/16-shaped scorer on decoded images / per video frame), ``hash_tokens`` (seeded hash of
  response token ids, the rule-based reward of the omni GRPO config), ``jpeg_compressibility``
  (CPU rule: negative JPEG size in KB, needs PIL), ``http`` (remote scorer over HTTP).
"""

from __future__ import annotations

import hashlib
import io
import logging
import pickle
from typing import Any, Callable, Optional

import numpy as np
import torch

from verl_omni_b200.utils.dataproto import DataProto

_log = logging.getLogger(__name__)
SCORERS: dict[str, Callable] = {}
REWARD_MANAGERS: dict[str, type] = {}


def register_scorer(name: str):
    def deco(fn):
        SCORERS[name] = fn
        return fn

    return deco


def register_reward_manager(name: str):
    def deco(cls):
        REWARD_MANAGERS[name] = cls
        return cls

    return deco


class ModelScorer:
    """Wraps a frozen scoring module; ``input_key`` selects images or latents from the batch."""

    def __init__(self, module: torch.nn.Module, input_key: str, device, micro_batch: int = 16):
        self.module = module.eval()
        for p in self.module.parameters():
            p.requires_grad_(False)
        self.input_key = input_key
        self.device = device
        self.micro_batch = micro_batch

    @torch.no_grad()
    def __call__(self, batch: DataProto, **_) -> torch.Tensor:
        x = batch.batch[self.input_key]
        outs = [self.module(x[i:i + self.micro_batch].to(self.device)) for i in range(0, x.shape[0], self.micro_batch)]
        return torch.cat(outs, 0).float()


@register_scorer("hash_tokens")
def hash_token_reward(batch: DataProto, seed: int = 0, **_) -> torch.Tensor:
    """Deterministic rule reward in [0, 1) from a seeded hash of each response's token ids."""
    ids = batch.batch["responses"].detach().cpu().numpy()
    out = []
    for row in ids:
        h = hashlib.blake2b(row.astype(np.int64).tobytes(), digest_size=8, key=int(seed).to_bytes(8, "little"))
        out.append(int.from_bytes(h.digest(), "little") / 2.0 ** 64)
    return torch.tensor(out, dtype=torch.float32)


@register_scorer("jpeg_compressibility")
def jpeg_compressibility(batch: DataProto, **_) -> torch.Tensor:
    """Negative JPEG size (KB) of each decoded image (``utils/reward_score/jpeg_compressibility.py:27-61``)."""
    from PIL import Image  # optional dependency

    imgs = batch.batch["images"]
    u8 = ((imgs.float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(0, 2, 3, 1).cpu().numpy()
    out = []
    for im in u8:
        buf = io.BytesIO()
        Image.fromarray(im).save(buf, format="JPEG", quality=95)
        out.append(-buf.tell() / 1000.0)
    return torch.tensor(out, dtype=torch.float32)


@register_scorer("http")
def http_scorer(batch: DataProto, url: str = "", timeout: float = 60.0, **_) -> torch.Tensor:
    """POST pickled uint8 images to a scoring service; expects a pickled list of floats back."""
    import requests

    imgs = batch.batch["images"]
    u8 = ((imgs.float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).cpu().numpy()
    r = requests.post(url, data=pickle.dumps({"images": u8}), timeout=timeout)
    r.raise_for_status()
    return torch.tensor(pickle.loads(r.content), dtype=torch.float32)


# ------------------------------------------------------------------ model-based scorers of the reference family
class _ModuleScorer:
    """A frozen scorer module called on the batch's images / audio and prompts (``models/scorers.py``)."""

    def __init__(self, kind: str, module: torch.nn.Module, device, micro_batch: int = 8):
        self.kind, self.module, self.device, self.mb = kind, module.eval(), device, micro_batch
        for p in self.module.parameters():
            p.requires_grad_(False)

    @torch.no_grad()
    def __call__(self, batch: DataProto, **_) -> torch.Tensor:
        from verl_omni_b200.models.scorers import _texts

        n = len(batch)
        texts = _texts(batch, n)
        truths = list(batch.non_tensor_batch.get("ground_truth", [None] * n))
        out = []
        for i in range(0, n, self.mb):
            sl = slice(i, min(n, i + self.mb))
            imgs = batch.batch["images"][sl].to(self.device) if "images" in batch.batch else None
            mels = batch.batch["audio_mels"][sl].to(self.device) if "audio_mels" in batch.batch else None
            if imgs is not None and imgs.ndim == 5:  # video: score the middle frame
                imgs = imgs[:, :, imgs.shape[2] // 2]
            if self.kind in ("pickscore", "hpsv3"):
                s = self.module.score(imgs, texts[sl])
            elif self.kind in ("ocr", "unified_reward"):
                s = self.module.score(imgs, texts[sl], truths[sl])
            elif self.kind == "clap":
                s = self.module.score(mels, texts[sl])
            else:  # imagebind
                s = self.module.score(texts[sl], images=imgs, mels=mels)
            out.append(s.float().cpu())
        return torch.cat(out, 0)


def build_model_scorer(kind: str, device, dtype=torch.bfloat16, **sizes) -> _ModuleScorer:
    """``pickscore`` | ``hpsv3`` | ``ocr`` | ``unified_reward`` | ``clap`` | ``imagebind`` at their reference
    shapes (or ``sizes`` overrides for small runs), random-init and frozen."""
    from verl_omni_b200.models import scorers as S

    if kind == "pickscore":
        m = S.PickScoreScorer(**sizes)
    elif kind == "hpsv3":
        m = S.HPSv3Scorer(**sizes)
    elif kind == "ocr":
        m = S.VLMJudge("ocr", **sizes)
    elif kind == "unified_reward":
        m = S.VLMJudge("unified", **sizes)
    elif kind == "clap":
        m = S.CLAPScorer(**sizes)
    elif kind == "imagebind":
        m = S.ImageBindScorer(**sizes)
    else:
        raise KeyError(f"unknown model scorer {kind!r}")
    return _ModuleScorer(kind, m.to(device=device, dtype=dtype), device)


def _decoded_responses(batch: DataProto) -> list[str]:
    from verl_omni_b200.models.scorers import byte_text

    if "response_text" in batch.non_tensor_batch:
        return [str(x) for x in batch.non_tensor_batch["response_text"]]
    return byte_text(batch.batch["responses"].cpu())


@register_scorer("mmk12")
def mmk12_scorer(batch: DataProto, **_) -> torch.Tensor:
    from verl_omni_b200.models.scorers import mmk12_reward

    return mmk12_reward(_decoded_responses(batch), list(batch.non_tensor_batch.get("ground_truth",
                                                                                    [None] * len(batch))))


@register_scorer("choice")
def choice_scorer(batch: DataProto, **_) -> torch.Tensor:
    from verl_omni_b200.models.scorers import choice_reward

    return choice_reward(_decoded_responses(batch), list(batch.non_tensor_batch.get("ground_truth",
                                                                                     [None] * len(batch))))


@register_reward_manager("visual")
class VisualRewardManager:
    def __init__(self, scorer: Callable, name: str = "reward", **kwargs):
        self.scorer = scorer
        self.name = name
        self.kwargs = kwargs

    def validate(self, batch: DataProto) -> None:
        if "images" in batch.batch:
            im = batch.batch["images"]
            if im.dtype != torch.uint8 and not torch.is_floating_point(im):
                raise TypeError(f"images must be uint8 or float, got {im.dtype}")
        elif "final_latents" not in batch.batch and "responses" not in batch.batch:
            raise KeyError("reward payload needs `images`, `final_latents` or `responses`")

    def __call__(self, batch: DataProto) -> tuple[torch.Tensor, dict]:
        self.validate(batch)
        s = self.scorer(batch, **self.kwargs)
        return s, {f"reward/{self.name}_mean": float(s.float().mean())}


@register_reward_manager("multi")
class MultiVisualRewardManager:
    """``sub_rewards``: list of (name, manager, weight, required)."""

    def __init__(self, sub_rewards: list):
        self.subs = sub_rewards

    def __call__(self, batch: DataProto) -> tuple[torch.Tensor, dict]:
        total = None
        metrics = {}
        for name, mgr, weight, required in self.subs:
            try:
                s, _ = mgr(batch)
                metrics[f"reward/{name}_mean"] = float(s.float().mean())
            except Exception as e:  # noqa: BLE001
                if required:
                    raise RuntimeError(f"required sub-reward {name!r} failed: {e}") from e
                _log.warning("optional sub-reward %s failed (%s); contributing 0", name, e)
                metrics[f"reward/{name}_failed"] = 1.0
                s = torch.zeros(len(batch))
            s = s.float().cpu() * float(weight)
            total = s if total is None else total + s
        return total, metrics
