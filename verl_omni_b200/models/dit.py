"""Cross-attention DiT with AdaLN-Zero (the Wan2.1 video DiT family, and the tiny plumbing DiT).

Block (Wan2.1 layout, as reached through the reference's ``wan22_dance_grpo`` adapter):
self-attention with per-head RMS qk-norm and 1D/3D RoPE -> gated residual; cross-attention
from the (LayerNorm'd) tokens to the text context -> plain residual; GELU(tanh) FFN -> gated
residual.  Modulation ``[shift, scale, gate] x (msa, mlp)`` comes from one linear of ``silu(temb)``.

Latents are 4-D images ``[B, C, H, W]`` (patch ``p x p``) or 5-D videos ``[B, C, F, H, W]``
(patch ``pt x ph x pw``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import (Linear, RMSWeight, TimestepMLP, patchify, patchify_3d, rope_nd,
                                          timestep_embedding, unpatchify, unpatchify_3d)
from verl_omni_b200.ops.attention import attention
from verl_omni_b200.parallel import ulysses_fused as UF
from verl_omni_b200.parallel.ulysses import gather_sequence, local_rows, shard_sequence, ulysses_attention
from verl_omni_b200.ops.norm import adaln_layernorm, layer_norm, qk_norm_split_into


@dataclass
class DiTConfig:
    in_channels: int = 16
    out_channels: int = 16
    patch: tuple = (1, 2, 2)  # (pt, ph, pw); images use (1, p, p)
    hidden: int = 5120
    heads: int = 40
    depth: int = 40
    ffn: int = 13824
    text_dim: int = 4096
    freq_dim: int = 256
    rope: bool = True
    eps: float = 1e-6

    @staticmethod
    def wan21_14b() -> "DiTConfig":
        return DiTConfig()

    @staticmethod
    def tiny_plumbing() -> "DiTConfig":
        """4 blocks, hidden 256, 4 heads, patch 2 (image), text width 256."""
        return DiTConfig(in_channels=4, out_channels=4, patch=(1, 2, 2), hidden=256, heads=4, depth=4, ffn=1024,
                         text_dim=256, rope=False)


class DiTBlock(nn.Module):
    def __init__(self, cfg: DiTConfig):
        super().__init__()
        D = cfg.hidden
        self.D, self.H, self.dh = D, cfg.heads, D // cfg.heads
        # per-block learned offset added to the shared time projection (Wan2.1 layout)
        self.modulation = nn.Parameter(torch.randn(6 * D) * 0.02)
        self.qkv = Linear(D, 3 * D)
        self.norm_q, self.norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.o = Linear(D, D)
        self.norm3_w = nn.Parameter(torch.ones(D))
        self.norm3_b = nn.Parameter(torch.zeros(D))
        self.cross_q = Linear(D, D)
        self.cross_kv = Linear(D, 2 * D)
        self.cross_norm_q, self.cross_norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.cross_o = Linear(D, D)
        self.ffn_1, self.ffn_2 = Linear(D, cfg.ffn), Linear(cfg.ffn, D)
        self.eps = cfg.eps

    def forward(self, x, ctx, temb_proj, rope=None, sp_group=None, rope_full=None):
        B, S, D = x.shape
        St = ctx.shape[1]
        H, dh = self.H, self.dh
        mod = temb_proj + self.modulation.to(temb_proj.dtype)[None]
        h = adaln_layernorm(x, mod, 0, 1, 6, self.eps)
        mk = lambda n: torch.empty(B, H, n, dh, device=x.device, dtype=x.dtype)  # noqa: E731
        if type(self.qkv) is Linear and UF.enabled(sp_group, x, H, D):
            # sequence-parallel inference: both exchanges inside the QKV GEMM and attention kernels
            o, _ = UF.joint_attention_fused(h, None, self.qkv, None, (self.norm_q.weight, self.norm_k.weight), None,
                                            H, sp_group, rope=rope_full, eps=self.eps)
        else:
            qkv = self.qkv(h).reshape(B * S, 3 * D)
            q, k, v = qk_norm_split_into(mk(S), mk(S), mk(S), qkv, self.norm_q.weight, self.norm_k.weight, S, 0,
                                         rope=rope, eps=self.eps)
            o = ulysses_attention(q, k, v, sp_group)  # local queries; keys over the whole sequence
        x = self.o(o, epilogue="gate_res", gate=mod.view(B, 6, D)[:, 2], res=x, S=S)
        # cross attention (no gate)
        hn = layer_norm(x, self.norm3_w.to(x.dtype), self.norm3_b.to(x.dtype), self.eps)
        qc = self.cross_q(hn).reshape(B * S, D)
        kv = self.cross_kv(ctx).reshape(B * St, 2 * D)
        qc, _, _ = qk_norm_split_into(mk(S), None, None, qc, self.cross_norm_q.weight, self.cross_norm_k.weight, S, 0,
                                      parts=(0, -1, -1), eps=self.eps)
        _, kc, vc = qk_norm_split_into(None, mk(St), mk(St), kv, self.cross_norm_q.weight, self.cross_norm_k.weight, St,
                                       0, parts=(-1, 0, D), eps=self.eps)
        oc = attention(qc, kc, vc)
        x = x + self.cross_o(oc)
        hm = adaln_layernorm(x, mod, 3, 4, 6, self.eps)
        u = self.ffn_1(hm, epilogue="gelu")
        return self.ffn_2(u, epilogue="gate_res", gate=mod.view(B, 6, D)[:, 5], res=x, S=S)


class DiT(nn.Module):
    """forward(latents, timestep [B], context [B, St, text_dim]) -> velocity (fp32, same shape as latents)."""

    family = "wan"

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.cfg = cfg
        pt, ph, pw = cfg.patch
        D = cfg.hidden
        self.patch_embedding = Linear(cfg.in_channels * pt * ph * pw, D)
        self.text_embedding_1 = Linear(cfg.text_dim, D)
        self.text_embedding_2 = Linear(D, D)
        self.time_embedding = TimestepMLP(cfg.freq_dim, D)
        self.time_projection = Linear(D, 6 * D)
        self.blocks = nn.ModuleList([DiTBlock(cfg) for _ in range(cfg.depth)])
        self.head_mod = Linear(D, 2 * D)
        self.head = Linear(D, pt * ph * pw * cfg.out_channels)
        self.gradient_checkpointing = False
        self._rope_cache: dict = {}

    def _rope(self, f, h, w, device):
        key = (f, h, w, str(device))
        if key not in self._rope_cache:
            dh = self.cfg.hidden // self.cfg.heads
            d_t = dh - 4 * (dh // 6)
            d_h = d_w = 2 * (dh // 6)
            ff, hh, ww = torch.meshgrid(torch.arange(f), torch.arange(h), torch.arange(w), indexing="ij")
            c, s = rope_nd([ff.reshape(-1), hh.reshape(-1), ww.reshape(-1)], [d_t, d_h, d_w])
            self._rope_cache[key] = (c.to(device).contiguous(), s.to(device).contiguous())
        return self._rope_cache[key]

    def forward(self, latents, timestep, context):
        cfg = self.cfg
        pt, ph, pw = cfg.patch
        dt = self.head.weight.dtype
        video = latents.ndim == 5
        if video:
            B, C, Fr, Hh, Ww = latents.shape
            x = patchify_3d(latents.to(dt), pt, ph, pw)
            grid = (Fr // pt, Hh // ph, Ww // pw)
        else:
            B, C, Hh, Ww = latents.shape
            x = patchify(latents.to(dt), ph)
            grid = (1, Hh // ph, Ww // pw)
        x = self.patch_embedding(x)
        temb = self.time_embedding(timestep_embedding(timestep, cfg.freq_dim).to(dt))
        temb_act = F.silu(temb)
        temb_proj = self.time_projection(temb_act)
        ctx = self.text_embedding_2(F.gelu(self.text_embedding_1(context.to(dt)), approximate="tanh"))
        rope = self._rope(*grid, x.device) if cfg.rope else None
        sp = getattr(self, "sp_group", None)
        rope_full = rope
        if sp is not None:  # Ulysses: 1/sp of the video tokens per rank; the text context stays whole
            S = x.shape[1]
            x = shard_sequence(x, sp)
            if rope is not None:
                rope = (local_rows(rope[0], [S], sp), local_rows(rope[1], [S], sp))
        for blk in self.blocks:
            if self.gradient_checkpointing and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(blk, x, ctx, temb_proj, rope, sp, rope_full, use_reentrant=False)
            else:
                x = blk(x, ctx, temb_proj, rope, sp, rope_full)
        mod = self.head_mod(temb_act)
        x = adaln_layernorm(x, mod, 0, 1, 2, cfg.eps)
        out = self.head(x)
        if sp is not None:
            out = gather_sequence(out, sp)
        if video:
            return unpatchify_3d(out, pt, ph, pw, cfg.out_channels, Fr, Hh, Ww).float()
        return unpatchify(out, ph, cfg.out_channels, Hh, Ww).float()


class TextEncoder(nn.Module):
    """Small bidirectional transformer text encoder (token ids -> [B, L, D] hidden states)."""

    def __init__(self, vocab: int = 1000, dim: int = 256, layers: int = 2, heads: int = 4, max_len: int = 512):
        super().__init__()
        self.embed = nn.Embedding(vocab, dim)
        self.pos = nn.Parameter(torch.randn(max_len, dim) * 0.02)
        self.heads = heads
        self.layers = nn.ModuleList()
        for _ in range(layers):
            blk = nn.Module()
            blk.ln1_w, blk.ln1_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
            blk.qkv = Linear(dim, 3 * dim)
            blk.o = Linear(dim, dim)
            blk.ln2_w, blk.ln2_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
            blk.fc1, blk.fc2 = Linear(dim, 4 * dim), Linear(4 * dim, dim)
            self.layers.append(blk)
        self.ln_f_w, self.ln_f_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        B, Lt = ids.shape
        dt = self.pos.dtype
        x = self.embed(ids).to(dt) + self.pos[:Lt][None]
        D = x.shape[-1]
        H = self.heads
        for blk in self.layers:
            h = layer_norm(x, blk.ln1_w, blk.ln1_b)
            qkv = blk.qkv(h).view(B, Lt, 3, H, D // H).permute(2, 0, 3, 1, 4)
            o = attention(qkv[0].contiguous(), qkv[1].contiguous(), qkv[2].contiguous())
            x = x + blk.o(o)
            h = layer_norm(x, blk.ln2_w, blk.ln2_b)
            x = x + blk.fc2(blk.fc1(h, epilogue="gelu"))
        return layer_norm(x, self.ln_f_w, self.ln_f_b)
