"""LTX-2-shaped joint audio-video DiT (asymmetric dual stream with cross-modal attention).

Shape family of the model the reference trains through ``verl_omni/pipelines/ltx2_flow_grpo``: the
denoiser sees one packed latent sequence per sample, video tokens first (``F' x H' x W'`` latent grid, 128
channels, patch 1) then audio tokens (latent frames, 128 channels); it returns the velocity of both and the
SDE step / log-probability run on the concatenation (``diffusers_training_adapter.py:141-190``).

Per layer, each stream has AdaLN-modulated self-attention (video: 3-axis RoPE, audio: 1-axis RoPE), text
cross-attention, a cross-modal attention (video queries over audio tokens and audio queries over video
tokens) and a GELU MLP, all with gated residuals.  Modulation is the Wan-style shared time projection plus a
learned per-block table.  Every projection runs on the tcgen05 GEMM; attention on the tcgen05 FMHA
(joint self-attention of the video stream is the long-sequence hot spot).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import Linear, RMSWeight, TimestepMLP, rope_nd, timestep_embedding
from verl_omni_b200.ops.attention import attention
from verl_omni_b200.ops.norm import adaln_layernorm, qk_norm_split_into


@dataclass
class LTX2Config:
    channels: int = 128          # latent channels of both streams (packed tokens)
    video_grid: tuple = (16, 16, 24)  # latent frames, rows, columns (121 frames at 512 x 768)
    audio_tokens: int = 126      # audio latent frames
    video_hidden: int = 4096
    video_heads: int = 32
    audio_hidden: int = 2048
    audio_heads: int = 32
    depth: int = 48
    mlp_ratio: float = 4.0
    text_dim: int = 3840
    eps: float = 1e-6

    @staticmethod
    def ltx2() -> "LTX2Config":
        return LTX2Config()

    @staticmethod
    def tiny() -> "LTX2Config":
        return LTX2Config(channels=16, video_grid=(2, 4, 4), audio_tokens=16, video_hidden=128, video_heads=2,
                          audio_hidden=64, audio_heads=2, depth=2, text_dim=48)

    @property
    def video_tokens(self) -> int:
        f, h, w = self.video_grid
        return f * h * w


def _attn(x2d_q, q_lin, kv_src, kv_lin, wq, wk, B, Sq, Skv, H, dh, eps, rope_q=None, rope_k=None, self_attn=False,
          qkv_lin=None):
    """Attention with per-head RMS q/k norms: self-attention from a fused [q|k|v] projection, or cross
    attention from separate q and [k|v] projections (keys/values from ``kv_src``)."""
    D = H * dh
    mk = lambda n: torch.empty(B, H, n, dh, device=x2d_q.device, dtype=x2d_q.dtype)  # noqa: E731
    if self_attn:
        qkv = qkv_lin(x2d_q).reshape(B * Sq, 3 * D)
        q, k, v = qk_norm_split_into(mk(Sq), mk(Sq), mk(Sq), qkv, wq, wk, Sq, 0, rope=rope_q, eps=eps)
        return attention(q, k, v)
    qc = q_lin(x2d_q).reshape(B * Sq, D)
    q, _, _ = qk_norm_split_into(mk(Sq), None, None, qc, wq, wk, Sq, 0, parts=(0, -1, -1), eps=eps)
    kv = kv_lin(kv_src).reshape(B * Skv, 2 * D)
    _, k, v = qk_norm_split_into(None, mk(Skv), mk(Skv), kv, wq, wk, Skv, 0, parts=(-1, 0, D), eps=eps)
    return attention(q, k, v)


class _Stream(nn.Module):
    """The per-stream weights of one layer (video or audio)."""

    def __init__(self, D: int, heads: int, other: int, mlp_ratio: float):
        super().__init__()
        self.D, self.H, self.dh = D, heads, D // heads
        self.modulation = nn.Parameter(torch.randn(9 * D) * 0.02)  # self-attn, MLP, cross-modal (shift, scale, gate)
        self.qkv = Linear(D, 3 * D)
        self.norm_q, self.norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.o = Linear(D, D)
        self.text_q, self.text_kv, self.text_o = Linear(D, D), Linear(D, 2 * D), Linear(D, D)
        self.text_norm_q, self.text_norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.av_q, self.av_kv, self.av_o = Linear(D, D), Linear(other, 2 * D), Linear(D, D)
        self.av_norm_q, self.av_norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.norm_text_w = nn.Parameter(torch.ones(D))
        self.norm_text_b = nn.Parameter(torch.zeros(D))
        hid = int(D * mlp_ratio)
        self.ff_1, self.ff_2 = Linear(D, hid), Linear(hid, D)


class LTX2Block(nn.Module):
    def __init__(self, cfg: LTX2Config):
        super().__init__()
        self.video = _Stream(cfg.video_hidden, cfg.video_heads, cfg.audio_hidden, cfg.mlp_ratio)
        self.audio = _Stream(cfg.audio_hidden, cfg.audio_heads, cfg.video_hidden, cfg.mlp_ratio)
        self.eps = cfg.eps

    def _self_and_text(self, s: _Stream, x, mod, ctx, rope):
        B, S, D = x.shape
        h = adaln_layernorm(x, mod, 0, 1, 9, self.eps)
        o = _attn(h, None, None, None, s.norm_q.weight, s.norm_k.weight, B, S, S, s.H, s.dh, self.eps, rope_q=rope,
                  self_attn=True, qkv_lin=s.qkv)
        x = s.o(o, epilogue="gate_res", gate=mod.view(B, 9, D)[:, 2], res=x, S=S)
        hn = F.layer_norm(x, (D,), s.norm_text_w.to(x.dtype), s.norm_text_b.to(x.dtype), self.eps)
        oc = _attn(hn, s.text_q, ctx, s.text_kv, s.text_norm_q.weight, s.text_norm_k.weight, B, S, ctx.shape[1], s.H,
                   s.dh, self.eps)
        return x + s.text_o(oc)

    def _cross_modal(self, s: _Stream, x, mod, other):
        B, S, D = x.shape
        h = adaln_layernorm(x, mod, 6, 7, 9, self.eps)
        o = _attn(h, s.av_q, other, s.av_kv, s.av_norm_q.weight, s.av_norm_k.weight, B, S, other.shape[1], s.H, s.dh,
                  self.eps)
        return s.av_o(o, epilogue="gate_res", gate=mod.view(B, 9, D)[:, 8], res=x, S=S)

    def _mlp(self, s: _Stream, x, mod):
        B, S, D = x.shape
        h = adaln_layernorm(x, mod, 3, 4, 9, self.eps)
        return s.ff_2(s.ff_1(h, epilogue="gelu"), epilogue="gate_res", gate=mod.view(B, 9, D)[:, 5], res=x, S=S)

    def forward(self, xv, xa, tv, ta, ctx_v, ctx_a, rope_v, rope_a):
        mv = tv + self.video.modulation.to(tv.dtype)[None]
        ma = ta + self.audio.modulation.to(ta.dtype)[None]
        xv = self._self_and_text(self.video, xv, mv, ctx_v, rope_v)
        xa = self._self_and_text(self.audio, xa, ma, ctx_a, rope_a)
        xv, xa = self._cross_modal(self.video, xv, mv, xa), self._cross_modal(self.audio, xa, ma, xv)
        return self._mlp(self.video, xv, mv), self._mlp(self.audio, xa, ma)


class LTX2AVDiT(nn.Module):
    """forward(latents [B, Sv + Sa, C], timestep [B] in [0, 1000], prompt_embeds [B, St, text_dim],
    audio_prompt_embeds [B, St, text_dim]) -> velocity [B, Sv + Sa, C] (fp32)."""

    family = "ltx2"

    def __init__(self, cfg: LTX2Config):
        super().__init__()
        self.cfg = cfg
        Dv, Da, C = cfg.video_hidden, cfg.audio_hidden, cfg.channels
        self.patchify_v, self.patchify_a = Linear(C, Dv), Linear(C, Da)
        self.caption_v, self.caption_a = Linear(cfg.text_dim, Dv), Linear(cfg.text_dim, Da)
        self.time_v, self.time_a = TimestepMLP(256, Dv), TimestepMLP(256, Da)
        self.time_proj_v, self.time_proj_a = Linear(Dv, 9 * Dv), Linear(Da, 9 * Da)
        self.blocks = nn.ModuleList([LTX2Block(cfg) for _ in range(cfg.depth)])
        self.head_mod_v, self.head_mod_a = Linear(Dv, 2 * Dv), Linear(Da, 2 * Da)
        self.head_v, self.head_a = Linear(Dv, C), Linear(Da, C)
        self.gradient_checkpointing = False
        self._rope_cache: dict = {}

    def _ropes(self, device):
        key = str(device)
        if key not in self._rope_cache:
            cfg = self.cfg
            f, h, w = cfg.video_grid
            dh = cfg.video_hidden // cfg.video_heads
            d_t = dh - 4 * (dh // 6)
            d_s = 2 * (dh // 6)
            ff, hh, ww = torch.meshgrid(torch.arange(f), torch.arange(h), torch.arange(w), indexing="ij")
            cv, sv = rope_nd([ff.reshape(-1), hh.reshape(-1), ww.reshape(-1)], [d_t, d_s, d_s])
            ca, sa = rope_nd([torch.arange(cfg.audio_tokens)], [cfg.audio_hidden // cfg.audio_heads])
            self._rope_cache[key] = ((cv.to(device).contiguous(), sv.to(device).contiguous()),
                                     (ca.to(device).contiguous(), sa.to(device).contiguous()))
        return self._rope_cache[key]

    def forward(self, latents, timestep, prompt_embeds, audio_prompt_embeds):
        cfg = self.cfg
        dt = self.head_v.weight.dtype
        Sv = cfg.video_tokens
        x = latents.to(dt)
        xv = self.patchify_v(x[:, :Sv].contiguous())
        xa = self.patchify_a(x[:, Sv:].contiguous())
        te = timestep_embedding(timestep, 256).to(dt)
        ev, ea = F.silu(self.time_v(te)), F.silu(self.time_a(te))
        tv, ta = self.time_proj_v(ev), self.time_proj_a(ea)
        ctx_v, ctx_a = self.caption_v(prompt_embeds.to(dt)), self.caption_a(audio_prompt_embeds.to(dt))
        rope_v, rope_a = self._ropes(x.device)
        for blk in self.blocks:
            if self.gradient_checkpointing and torch.is_grad_enabled():
                xv, xa = torch.utils.checkpoint.checkpoint(blk, xv, xa, tv, ta, ctx_v, ctx_a, rope_v, rope_a,
                                                           use_reentrant=False)
            else:
                xv, xa = blk(xv, xa, tv, ta, ctx_v, ctx_a, rope_v, rope_a)
        yv = self.head_v(adaln_layernorm(xv, self.head_mod_v(ev), 0, 1, 2, cfg.eps))
        ya = self.head_a(adaln_layernorm(xa, self.head_mod_a(ea), 0, 1, 2, cfg.eps))
        return torch.cat([yv, ya], 1).float()
