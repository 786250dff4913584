"""Frozen random-init reward models and the VAE decoder used in rollout.

* ``LatentMLPReward``: scalar from a 2-layer MLP on the mean-pooled final latent (plumbing config).
* ``ViTScorer``: ViT-B/16-shaped image scorer (patch 16, width 768, 12 layers, 12 heads) on decoded
  images -> scalar (stands in for PickScore/HPS-style scorers, ``verl_omni/utils/reward_score/pickscore_reward.py``);
  with ``per_frame=True`` it scores each video frame and mean-pools (video reward).
* ``VAEDecoder``: SD/SD3-shaped VAE decoder (16 latent channels, 512-512-256-128 up path, x8
  upsampling) producing images in [-1, 1].  Convolutions and GroupNorm run through cuDNN / torch.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import Linear
from verl_omni_b200.ops.attention import attention
from verl_omni_b200.ops.norm import layer_norm


class LatentMLPReward(nn.Module):
    def __init__(self, channels: int = 4, hidden: int = 256):
        super().__init__()
        self.fc1 = nn.Linear(channels, hidden)
        self.fc2 = nn.Linear(hidden, 1)

    @torch.no_grad()
    def forward(self, latents: torch.Tensor) -> torch.Tensor:
        pooled = latents.float().flatten(2).mean(-1)  # [B, C]
        return self.fc2(torch.tanh(self.fc1(pooled.to(self.fc1.weight.dtype)))).squeeze(-1).float()


class ViTScorer(nn.Module):
    def __init__(self, image_size: int = 512, patch: int = 16, dim: int = 768, depth: int = 12, heads: int = 12,
                 mlp: int = 3072):
        super().__init__()
        self.patch, self.heads, self.dim = patch, heads, dim
        n = (image_size // patch) ** 2
        self.patch_embed = Linear(3 * patch * patch, dim)
        self.cls = nn.Parameter(torch.randn(1, 1, dim) * 0.02)
        self.pos = nn.Parameter(torch.randn(1, n + 1, dim) * 0.02)
        self.blocks = nn.ModuleList()
        for _ in range(depth):
            b = nn.Module()
            b.ln1_w, b.ln1_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
            b.qkv = Linear(dim, 3 * dim)
            b.proj = Linear(dim, dim)
            b.ln2_w, b.ln2_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
            b.fc1, b.fc2 = Linear(dim, mlp), Linear(mlp, dim)
            self.blocks.append(b)
        self.ln_w, self.ln_b = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.zeros(dim))
        self.head = Linear(dim, 1)

    @torch.no_grad()
    def forward(self, images: torch.Tensor) -> torch.Tensor:
        """images [B, 3, H, W] in [-1, 1] (or [B, 3, F, H, W] -> per-frame mean)."""
        if images.ndim == 5:
            B, C, Fr, H, W = images.shape
            s = self.forward(images.permute(0, 2, 1, 3, 4).reshape(B * Fr, C, H, W))
            return s.view(B, Fr).mean(1)
        dt = self.head.weight.dtype
        B, C, H, W = images.shape
        p = self.patch
        x = images.to(dt).view(B, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5).reshape(B, -1, C * p * p)
        x = self.patch_embed(x)
        x = torch.cat([self.cls.to(dt).expand(B, -1, -1), x], dim=1) + self.pos.to(dt)
        S, D, Hh = x.shape[1], self.dim, self.heads
        for b in self.blocks:
            h = layer_norm(x, b.ln1_w, b.ln1_b)
            qkv = b.qkv(h).view(B, S, 3, Hh, D // Hh).permute(2, 0, 3, 1, 4)
            o = attention(qkv[0].contiguous(), qkv[1].contiguous(), qkv[2].contiguous())
            x = x + b.proj(o)
            h = layer_norm(x, b.ln2_w, b.ln2_b)
            x = x + b.fc2(b.fc1(h, epilogue="gelu"))
        x = layer_norm(x[:, 0], self.ln_w, self.ln_b)
        return self.head(x).squeeze(-1).float()


def _gn(norm: nn.GroupNorm, x: torch.Tensor, silu: bool = False) -> torch.Tensor:
    """GroupNorm (+SiLU) on the NHWC kernel for channels-last bf16 activations."""
    from verl_omni_b200.ops.norm import group_norm_act

    return group_norm_act(x, norm.weight, norm.bias, norm.num_groups, norm.eps, silu)


class _ResBlock(nn.Module):
    def __init__(self, cin: int, cout: int):
        super().__init__()
        self.n1 = nn.GroupNorm(32, cin, eps=1e-6)
        self.c1 = nn.Conv2d(cin, cout, 3, padding=1)
        self.n2 = nn.GroupNorm(32, cout, eps=1e-6)
        self.c2 = nn.Conv2d(cout, cout, 3, padding=1)
        self.skip = nn.Conv2d(cin, cout, 1) if cin != cout else None

    def forward(self, x):
        h = self.c1(_gn(self.n1, x, silu=True))
        h = self.c2(_gn(self.n2, h, silu=True))
        return h + (self.skip(x) if self.skip is not None else x)


class _MidAttn(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.norm = nn.GroupNorm(32, c, eps=1e-6)
        self.qkv = nn.Linear(c, 3 * c)
        self.out = nn.Linear(c, c)

    def forward(self, x):
        B, C, H, W = x.shape
        h = _gn(self.norm, x).flatten(2).transpose(1, 2)
        q, k, v = self.qkv(h).chunk(3, dim=-1)
        o = attention(q[:, None].contiguous(), k[:, None].contiguous(), v[:, None].contiguous())
        return x + self.out(o).transpose(1, 2).reshape(B, C, H, W)


class VAEDecoder(nn.Module):
    def __init__(self, latent_channels: int = 16, block_out=(128, 256, 512, 512), layers_per_block: int = 2,
                 scaling_factor: float = 1.5305, shift_factor: float = 0.0609, mid_attention: bool = True):
        super().__init__()
        self.scaling_factor, self.shift_factor = scaling_factor, shift_factor
        ch = list(reversed(block_out))
        self.conv_in = nn.Conv2d(latent_channels, ch[0], 3, padding=1)
        self.mid1 = _ResBlock(ch[0], ch[0])
        self.mid_attn = _MidAttn(ch[0]) if mid_attention else None
        self.mid2 = _ResBlock(ch[0], ch[0])
        self.ups = nn.ModuleList()
        cin = ch[0]
        for i, c in enumerate(ch):
            stage = nn.Module()
            stage.res = nn.ModuleList([_ResBlock(cin if j == 0 else c, c) for j in range(layers_per_block + 1)])
            stage.up = nn.Conv2d(c, c, 3, padding=1) if i < len(ch) - 1 else None
            self.ups.append(stage)
            cin = c
        self.norm_out = nn.GroupNorm(32, ch[-1], eps=1e-6)
        self.conv_out = nn.Conv2d(ch[-1], 3, 3, padding=1)

    @torch.no_grad()
    def forward(self, latents: torch.Tensor) -> torch.Tensor:
        dt = self.conv_in.weight.dtype
        z = latents.to(dt) / self.scaling_factor + self.shift_factor
        x = self.conv_in(z.contiguous(memory_format=torch.channels_last))
        x = self.mid1(x)
        if self.mid_attn is not None:
            x = self.mid_attn(x)
        x = self.mid2(x)
        for st in self.ups:
            for r in st.res:
                x = r(x)
            if st.up is not None:
                x = st.up(F.interpolate(x, scale_factor=2.0, mode="nearest"))
        x = self.conv_out(_gn(self.norm_out, x, silu=True))
        return x.clamp(-1, 1)

    def decode_video(self, latents: torch.Tensor) -> torch.Tensor:
        """[B, C, F, h, w] -> frames decoded independently -> [B, 3, F, 8h, 8w]."""
        B, C, Fr, h, w = latents.shape
        imgs = self.forward(latents.permute(0, 2, 1, 3, 4).reshape(B * Fr, C, h, w))
        return imgs.view(B, Fr, 3, imgs.shape[-2], imgs.shape[-1]).permute(0, 2, 1, 3, 4)
