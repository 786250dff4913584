"""Random-init, shape-faithful reward scorers of the reference's ``utils/reward_score`` family.

No checkpoints are reachable offline, so each scorer keeps the architecture and the scoring rule of its
reference counterpart with random (frozen) weights; every tower runs on the native GEMM / FMHA / LayerNorm
kernels through :class:`Tower`.

* ``PickScoreScorer`` (``pickscore_reward.py:50-198``): CLIP-H/14-shaped image tower + text tower,
  reward = logit_scale * cos(image, prompt).
* ``HPSv3Scorer`` (``hpsv3_reward.py:178-438``): a Qwen2-VL-shaped VLM (vision patches projected into a
  causal LM) with an uncertainty head (mu, log sigma); reward = mu.
* ``VLMJudge`` (``genrm_ocr.py:96``, ``unified_reward.py:167``): the same VLM decoding text greedily;
  ``ocr``: 1 - normalised edit distance between the decoded text and the prompt's ground truth;
  ``unified``: the first digit 1-5 in the decoded text, mapped to [0, 1].
* ``CLAPScorer`` (``clap.py:61``): log-mel audio tower + text tower, reward = cos(audio, text).
* ``ImageBindScorer`` (``imagebind.py:224``): image / audio / text towers into one embedding space,
  reward = mean cosine of the present modalities with the text.
* Rule scorers ``mmk12`` / ``choice``: answer extraction from a decoded LLM response compared with the
  ground truth (exact match after normalisation; the last A-E letter for multiple choice).
Text is tokenised with a byte-level tokeniser (UTF-8 bytes mod vocab) in the absence of the real ones.
"""

from __future__ import annotations

import math
import re
from typing import Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import Linear
from verl_omni_b200.ops.attention import attention
from verl_omni_b200.ops.norm import layer_norm


def byte_ids(texts: Sequence[str], vocab: int, length: int) -> torch.Tensor:
    rows = []
    for t in texts:
        ids = [(b % (vocab - 1)) + 1 for b in str(t or "").encode("utf-8")][:length]
        rows.append(ids + [0] * (length - len(ids)))
    return torch.tensor(rows, dtype=torch.long)


def byte_text(ids: torch.Tensor) -> list[str]:
    out = []
    for row in ids.tolist():
        out.append(bytes([(int(i) - 1) % 256 for i in row if int(i) > 0]).decode("utf-8", errors="ignore"))
    return out


class Tower(nn.Module):
    """Pre-LN transformer over a token sequence (bidirectional or causal), optional pooled projection."""

    def __init__(self, dim: int, depth: int, heads: int, mlp_ratio: float = 4.0, out_dim: Optional[int] = None,
                 causal: bool = False):
        super().__init__()
        self.dim, self.heads, self.causal = dim, heads, causal
        self.blocks = nn.ModuleList()
        for _ in range(depth):
            b = nn.Module()
            b.ln1_w, b.ln1_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
            b.qkv, b.proj = Linear(dim, 3 * dim), Linear(dim, dim)
            b.ln2_w, b.ln2_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
            b.fc1, b.fc2 = Linear(dim, int(dim * mlp_ratio)), Linear(int(dim * mlp_ratio), dim)
            self.blocks.append(b)
        self.ln_w, self.ln_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
        self.out = Linear(dim, out_dim, bias=False) if out_dim else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, D = x.shape
        H = self.heads
        for b in self.blocks:
            h = layer_norm(x, b.ln1_w, b.ln1_b)
            qkv = b.qkv(h).view(B, S, 3, H, D // H).permute(2, 0, 3, 1, 4)
            x = x + b.proj(attention(qkv[0].contiguous(), qkv[1].contiguous(), qkv[2].contiguous(),
                                     causal=self.causal))
            x = x + b.fc2(b.fc1(layer_norm(x, b.ln2_w, b.ln2_b), epilogue="gelu"))
        return layer_norm(x, self.ln_w, self.ln_b)

    def pooled(self, x: torch.Tensor, idx: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = self.forward(x)
        p = h[:, 0] if idx is None else h[torch.arange(h.shape[0], device=h.device), idx]
        return self.out(p) if self.out is not None else p


class ImageEncoder(nn.Module):
    """ViT patch embedding + class token + positions -> Tower."""

    def __init__(self, image_size: int, patch: int, dim: int, depth: int, heads: int, out_dim: int):
        super().__init__()
        self.patch, self.image_size = patch, image_size
        n = (image_size // patch) ** 2
        self.embed = Linear(3 * patch * patch, dim)
        self.cls = nn.Parameter(torch.randn(1, 1, dim) * 0.02)
        self.pos = nn.Parameter(torch.randn(1, n + 1, dim) * 0.02)
        self.tower = Tower(dim, depth, heads, out_dim=out_dim)

    def tokens(self, images: torch.Tensor) -> torch.Tensor:
        dt = self.embed.weight.dtype
        s, p = self.image_size, self.patch
        if images.shape[-1] != s or images.shape[-2] != s:
            images = F.interpolate(images.float(), size=(s, s), mode="bilinear", align_corners=False)
        B, C = images.shape[:2]
        x = images.to(dt).view(B, C, s // p, p, s // p, p).permute(0, 2, 4, 1, 3, 5).reshape(B, -1, C * p * p)
        x = self.embed(x)
        return torch.cat([self.cls.to(dt).expand(B, -1, -1), x], 1) + self.pos.to(dt)

    def forward(self, images: torch.Tensor) -> torch.Tensor:
        return self.tower.pooled(self.tokens(images))


class TextTower(nn.Module):
    """Token embedding + positions -> Tower, pooled at the last non-pad token (CLIP's EOT pooling)."""

    def __init__(self, vocab: int, length: int, dim: int, depth: int, heads: int, out_dim: int):
        super().__init__()
        self.vocab, self.length = vocab, length
        self.embed = nn.Embedding(vocab, dim)
        self.pos = nn.Parameter(torch.randn(length, dim) * 0.02)
        self.tower = Tower(dim, depth, heads, out_dim=out_dim, causal=True)

    def forward(self, texts: Sequence[str], device) -> torch.Tensor:
        ids = byte_ids(texts, self.vocab, self.length).to(device)
        dt = self.pos.dtype
        x = self.embed(ids).to(dt) + self.pos[None]
        last = (ids > 0).sum(-1).clamp_min(1) - 1
        return self.tower.pooled(x, last)


def _texts(batch, n: int, key: str = "raw_prompt") -> list[str]:
    v = batch.non_tensor_batch.get(key)
    return [str(x) for x in v[:n]] if v is not None else [""] * n


class PickScoreScorer(nn.Module):
    def __init__(self, image_size: int = 224, patch: int = 14, vision_dim: int = 1280, vision_depth: int = 32,
                 vision_heads: int = 16, text_dim: int = 1024, text_depth: int = 24, text_heads: int = 16,
                 embed_dim: int = 1024, vocab: int = 49408, text_len: int = 77):
        super().__init__()
        self.visual = ImageEncoder(image_size, patch, vision_dim, vision_depth, vision_heads, embed_dim)
        self.text = TextTower(vocab, text_len, text_dim, text_depth, text_heads, embed_dim)
        self.logit_scale = nn.Parameter(torch.tensor(math.log(100.0)))

    @torch.no_grad()
    def score(self, images: torch.Tensor, texts: Sequence[str]) -> torch.Tensor:
        i = F.normalize(self.visual(images).float(), dim=-1)
        t = F.normalize(self.text(texts, images.device).float(), dim=-1)
        return self.logit_scale.exp() * (i * t).sum(-1)


class SmallVLM(nn.Module):
    """Qwen2-VL-shaped: a ViT over image patches, a projector, and a causal LM over [image tokens | prompt]."""

    def __init__(self, image_size: int = 448, patch: int = 14, vision_dim: int = 1280, vision_depth: int = 32,
                 vision_heads: int = 16, lm_dim: int = 1536, lm_depth: int = 28, lm_heads: int = 12,
                 vocab: int = 151936, text_len: int = 64):
        super().__init__()
        self.vocab, self.text_len = vocab, text_len
        self.visual = ImageEncoder(image_size, patch, vision_dim, vision_depth, vision_heads, None)
        self.proj = Linear(vision_dim, lm_dim)
        self.embed = nn.Embedding(vocab, lm_dim)
        self.lm = Tower(lm_dim, lm_depth, lm_heads, causal=True)
        self.lm_head = Linear(lm_dim, vocab, bias=False)

    def hidden(self, images: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        v = self.proj(self.visual.tower(self.visual.tokens(images)))
        t = self.embed(ids).to(v.dtype)
        return self.lm(torch.cat([v, t], 1))

    @torch.no_grad()
    def greedy(self, images: torch.Tensor, texts: Sequence[str], new_tokens: int) -> torch.Tensor:
        ids = byte_ids(texts, self.vocab, self.text_len).to(images.device)
        out = []
        for _ in range(new_tokens):  # recomputes the short sequence each step (judge outputs are a few tokens)
            h = self.hidden(images, ids)
            nxt = self.lm_head(h[:, -1:].contiguous()).float()[:, -1, :256].argmax(-1) + 1  # byte range
            out.append(nxt)
            ids = torch.cat([ids, nxt[:, None]], 1)
        return torch.stack(out, 1)


class HPSv3Scorer(nn.Module):
    def __init__(self, **vlm_kwargs):
        super().__init__()
        self.vlm = SmallVLM(**vlm_kwargs)
        self.head = Linear(self.vlm.lm.dim, 2, bias=False)  # (mu, log sigma)

    @torch.no_grad()
    def score(self, images: torch.Tensor, texts: Sequence[str]) -> torch.Tensor:
        ids = byte_ids(texts, self.vlm.vocab, self.vlm.text_len).to(images.device)
        h = self.vlm.hidden(images, ids)
        last = h.shape[1] - ids.shape[1] + (ids > 0).sum(-1).clamp_min(1) - 1
        pooled = h[torch.arange(h.shape[0], device=h.device), last]
        return F.linear(pooled, self.head.weight).float()[:, 0]


def edit_distance(a: str, b: str) -> int:
    prev = list(range(len(b) + 1))
    for i, ca in enumerate(a, 1):
        cur = [i]
        for j, cb in enumerate(b, 1):
            cur.append(min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (ca != cb)))
        prev = cur
    return prev[-1]


class VLMJudge(nn.Module):
    def __init__(self, mode: str = "ocr", new_tokens: int = 16, **vlm_kwargs):
        super().__init__()
        if mode not in ("ocr", "unified"):
            raise ValueError(f"judge mode {mode!r}")
        self.mode, self.new_tokens = mode, new_tokens
        self.vlm = SmallVLM(**vlm_kwargs)

    @torch.no_grad()
    def score(self, images: torch.Tensor, texts: Sequence[str], truths: Sequence[Optional[str]]) -> torch.Tensor:
        prompt = "Read the text in the image." if self.mode == "ocr" else "Rate the image from 1 to 5."
        decoded = byte_text(self.vlm.greedy(images, [f"{prompt} {t}" for t in texts], self.new_tokens).cpu())
        out = []
        for d, gt, t in zip(decoded, truths, texts):
            if self.mode == "ocr":
                ref = str(gt if gt is not None else t).strip().lower()
                hyp = d.strip().lower()
                out.append(1.0 - edit_distance(hyp, ref) / max(1, len(ref), len(hyp)))
            else:
                m = re.search(r"[1-5]", d)
                out.append((int(m.group()) - 1) / 4.0 if m else 0.0)
        return torch.tensor(out, dtype=torch.float32)


class CLAPScorer(nn.Module):
    def __init__(self, n_mels: int = 64, audio_dim: int = 768, audio_depth: int = 12, audio_heads: int = 12,
                 text_dim: int = 768, text_depth: int = 12, text_heads: int = 12, embed_dim: int = 512,
                 vocab: int = 50265, text_len: int = 77):
        super().__init__()
        self.audio_in = Linear(n_mels, audio_dim)
        self.audio = Tower(audio_dim, audio_depth, audio_heads, out_dim=embed_dim)
        self.text = TextTower(vocab, text_len, text_dim, text_depth, text_heads, embed_dim)

    @torch.no_grad()
    def score(self, mels: torch.Tensor, texts: Sequence[str]) -> torch.Tensor:
        """mels [B, frames, n_mels]."""
        a = self.audio(self.audio_in(mels.to(self.audio_in.weight.dtype))).mean(1)
        a = F.normalize(self.audio.out(a).float(), dim=-1)
        t = F.normalize(self.text(texts, mels.device).float(), dim=-1)
        return (a * t).sum(-1)


class ImageBindScorer(nn.Module):
    def __init__(self, image_size: int = 224, patch: int = 14, dim: int = 1024, depth: int = 24, heads: int = 16,
                 n_mels: int = 128, embed_dim: int = 1024, vocab: int = 49408, text_len: int = 77):
        super().__init__()
        self.visual = ImageEncoder(image_size, patch, dim, depth, heads, embed_dim)
        self.audio_in = Linear(n_mels, dim)
        self.audio = Tower(dim, max(1, depth // 2), heads, out_dim=embed_dim)
        self.text = TextTower(vocab, text_len, dim, max(1, depth // 2), heads, embed_dim)

    @torch.no_grad()
    def score(self, texts: Sequence[str], images: Optional[torch.Tensor] = None,
              mels: Optional[torch.Tensor] = None) -> torch.Tensor:
        dev = images.device if images is not None else mels.device
        t = F.normalize(self.text(texts, dev).float(), dim=-1)
        sims = []
        if images is not None:
            sims.append((F.normalize(self.visual(images).float(), dim=-1) * t).sum(-1))
        if mels is not None:
            a = self.audio.pooled(self.audio_in(mels.to(self.audio_in.weight.dtype)))
            sims.append((F.normalize(a.float(), dim=-1) * t).sum(-1))
        return torch.stack(sims, 0).mean(0)


def _normalise_answer(s: str) -> str:
    s = str(s or "").strip().lower()
    m = re.search(r"\\boxed\{([^}]*)\}", s)
    if m:
        s = m.group(1)
    return re.sub(r"[\s\.\$]+", "", s)


def mmk12_reward(responses: Sequence[str], truths: Sequence[Optional[str]]) -> torch.Tensor:
    """1 when the response's final answer (``\\boxed{}`` if present, else the last line) equals the truth."""
    out = []
    for r, gt in zip(responses, truths):
        lines = [ln for ln in str(r).strip().splitlines() if ln.strip()]
        ans = r if "\\boxed" in str(r) else (lines[-1] if lines else "")
        out.append(float(gt is not None and _normalise_answer(ans) == _normalise_answer(gt)))
    return torch.tensor(out, dtype=torch.float32)


def choice_reward(responses: Sequence[str], truths: Sequence[Optional[str]]) -> torch.Tensor:
    """1 when the last standalone option letter A-E of the response equals the ground-truth letter."""
    out = []
    for r, gt in zip(responses, truths):
        letters = re.findall(r"\b([A-E])\b", str(r).upper())
        out.append(float(bool(letters) and gt is not None and letters[-1] == str(gt).strip().upper()[:1]))
    return torch.tensor(out, dtype=torch.float32)
