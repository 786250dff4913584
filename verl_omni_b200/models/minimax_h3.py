"""MiniMax-H3-shaped single-stream audio-video DiT (packed text / audio / video rows).

Shape family of the model the reference fine-tunes with DiffusionNFT through
``verl_omni/pipelines/minimax_h3_diffusion_nft`` (``diffusers_training_adapter.py:38-141``,
``common.py:86-283``):

* the per-sample latent is one flat vector: video rows of width 96 (a 1x2x2 patch of 24 latent channels),
  then audio rows of width 32, packed and unpacked by :func:`pack_rows` / :func:`unpack_rows`;
* the transformer runs on one sequence ``[text | audio | video]`` with a learned tag embedding per
  modality and 3-axis rotary positions (time, row, column): text tokens on the time axis, audio rows on the
  time axis, video rows on their latent grid;
* H3's clock is the data fraction ``1 - sigma`` and its velocity has the opposite sign of the flow-matching
  convention (``common.py:76-83``); this module takes ``sigma * 1000`` and returns flow-matching velocities.

Blocks are single-stream AdaLN-Zero transformer layers (RMS q/k norms, GELU MLP) on the tcgen05 GEMM and FMHA.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import Linear, RMSWeight, TimestepMLP, rope_nd, timestep_embedding
from verl_omni_b200.ops.attention import attention
from verl_omni_b200.ops.norm import adaln_layernorm, qk_norm_split_into

VIDEO_ROW_WIDTH = 96
AUDIO_ROW_WIDTH = 32


@dataclass
class H3Config:
    video_grid: tuple = (8, 30, 52)  # latent frames, patch rows, patch columns
    audio_rows: int = 256
    hidden: int = 3072
    heads: int = 24
    depth: int = 40
    mlp_ratio: float = 4.0
    text_dim: int = 4096
    eps: float = 1e-6

    @staticmethod
    def h3() -> "H3Config":
        return H3Config()

    @staticmethod
    def tiny() -> "H3Config":
        return H3Config(video_grid=(2, 4, 4), audio_rows=8, hidden=128, heads=2, depth=2, text_dim=48)

    @property
    def video_rows(self) -> int:
        f, h, w = self.video_grid
        return f * h * w

    @property
    def flat(self) -> int:
        return self.video_rows * VIDEO_ROW_WIDTH + self.audio_rows * AUDIO_ROW_WIDTH


def pack_rows(video: torch.Tensor, audio: torch.Tensor) -> torch.Tensor:
    """[B, Vr, 96], [B, Ar, 32] -> [B, Vr*96 + Ar*32]."""
    B = video.shape[0]
    return torch.cat([video.reshape(B, -1), audio.reshape(B, -1)], 1)


def unpack_rows(flat: torch.Tensor, video_rows: int, audio_rows: int) -> tuple[torch.Tensor, torch.Tensor]:
    B = flat.shape[0]
    flat = flat.reshape(B, -1)
    n = video_rows * VIDEO_ROW_WIDTH
    return flat[:, :n].reshape(B, video_rows, VIDEO_ROW_WIDTH), flat[:, n:].reshape(B, audio_rows, AUDIO_ROW_WIDTH)


class H3Block(nn.Module):
    def __init__(self, cfg: H3Config):
        super().__init__()
        D = cfg.hidden
        self.H, self.dh, self.eps = cfg.heads, D // cfg.heads, cfg.eps
        self.mod = Linear(D, 6 * D)
        self.qkv = Linear(D, 3 * D)
        self.norm_q, self.norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.o = Linear(D, D)
        hid = int(D * cfg.mlp_ratio)
        self.ff_1, self.ff_2 = Linear(D, hid), Linear(hid, D)

    def forward(self, x, temb_act, rope):
        B, S, D = x.shape
        m = self.mod(temb_act)
        h = adaln_layernorm(x, m, 0, 1, 6, self.eps)
        mk = lambda: torch.empty(B, self.H, S, self.dh, device=x.device, dtype=x.dtype)  # noqa: E731
        q, k, v = qk_norm_split_into(mk(), mk(), mk(), self.qkv(h).reshape(B * S, 3 * D), self.norm_q.weight,
                                     self.norm_k.weight, S, 0, rope=rope, eps=self.eps)
        x = self.o(attention(q, k, v), epilogue="gate_res", gate=m.view(B, 6, D)[:, 2], res=x, S=S)
        hm = adaln_layernorm(x, m, 3, 4, 6, self.eps)
        return self.ff_2(self.ff_1(hm, epilogue="gelu"), epilogue="gate_res", gate=m.view(B, 6, D)[:, 5], res=x, S=S)


class MiniMaxH3DiT(nn.Module):
    """forward(latents [B, ...] holding the packed flat rows, timestep [B] = sigma * 1000,
    prompt_embeds [B, St, text_dim]) -> flow-matching velocity with the latents' shape (fp32)."""

    family = "minimax_h3"

    def __init__(self, cfg: H3Config):
        super().__init__()
        self.cfg = cfg
        D = cfg.hidden
        self.video_in, self.audio_in, self.text_in = (Linear(VIDEO_ROW_WIDTH, D), Linear(AUDIO_ROW_WIDTH, D),
                                                      Linear(cfg.text_dim, D))
        self.tag = nn.Parameter(torch.randn(3, D) * 0.02)  # text, audio, video
        self.time_embed = TimestepMLP(256, D)
        self.blocks = nn.ModuleList([H3Block(cfg) for _ in range(cfg.depth)])
        self.norm_out_linear = Linear(D, 2 * D)
        self.video_out, self.audio_out = Linear(D, VIDEO_ROW_WIDTH), Linear(D, AUDIO_ROW_WIDTH)
        self.gradient_checkpointing = False
        self._rope_cache: dict = {}

    def _rope(self, St: int, device):
        key = (St, str(device))
        if key not in self._rope_cache:
            cfg = self.cfg
            f, h, w = cfg.video_grid
            dh = cfg.hidden // cfg.heads
            d_s = 2 * (dh // 6)
            d_t = dh - 2 * d_s
            tt = torch.arange(St).float()
            ta = St + torch.arange(cfg.audio_rows).float() * (f / max(cfg.audio_rows, 1))
            ff, hh, ww = torch.meshgrid(torch.arange(f), torch.arange(h), torch.arange(w), indexing="ij")
            t_axis = torch.cat([tt, ta, St + ff.reshape(-1).float()])
            r_axis = torch.cat([torch.zeros(St + cfg.audio_rows), hh.reshape(-1).float()])
            c_axis = torch.cat([torch.zeros(St + cfg.audio_rows), ww.reshape(-1).float()])
            c, s = rope_nd([t_axis, r_axis, c_axis], [d_t, d_s, d_s])
            self._rope_cache[key] = (c.to(device).contiguous(), s.to(device).contiguous())
        return self._rope_cache[key]

    def forward(self, latents, timestep, prompt_embeds):
        cfg = self.cfg
        dt = self.video_out.weight.dtype
        B = latents.shape[0]
        video, audio = unpack_rows(latents.to(dt), cfg.video_rows, cfg.audio_rows)
        c = self.text_in(prompt_embeds.to(dt)) + self.tag[0].to(dt)
        a = self.audio_in(audio.contiguous()) + self.tag[1].to(dt)
        v = self.video_in(video.contiguous()) + self.tag[2].to(dt)
        x = torch.cat([c, a, v], 1)
        St = c.shape[1]
        t_h3 = 1000.0 - timestep.float()  # H3 clock: data fraction (1 - sigma) x 1000
        ta = F.silu(self.time_embed(timestep_embedding(t_h3, 256).to(dt)))
        rope = self._rope(St, x.device)
        for blk in self.blocks:
            if self.gradient_checkpointing and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(blk, x, ta, rope, use_reentrant=False)
            else:
                x = blk(x, ta, rope)
        x = adaln_layernorm(x[:, St:].contiguous(), self.norm_out_linear(ta), 1, 0, 2, cfg.eps)
        vo = self.video_out(x[:, cfg.audio_rows:].contiguous())
        ao = self.audio_out(x[:, :cfg.audio_rows].contiguous())
        # H3 velocity points from data to noise in its clock: flip to the flow-matching sign
        return (-pack_rows(vo, ao)).float().reshape(latents.shape)
