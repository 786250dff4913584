"""Building blocks shared by the DiT families (parameters only; math lives in ``verl_omni_b200.ops``)."""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.ops import linear as L


class Linear(nn.Module):
    """``y = x W^T + b`` on the tcgen05 GEMM, with the fused epilogues of ``ops.linear``."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, std: float = 0.02):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.empty(out_features)) if bias else None
        self.std = std
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.normal_(self.weight, std=self.std)
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def forward(self, x, epilogue: str = "none", gate=None, res=None, S: int = 1):
        return L.linear(x, self.weight, self.bias, epilogue=epilogue, gate=gate, res=res, S=S)


def linear_pair(m0: nn.Module, x0, m1: nn.Module, x1, epilogue: str = "none", gate0=None, res0=None, S0: int = 1,
                gate1=None, res1=None, S1: int = 1):
    """``(m0(x0, ...), m1(x1, ...))``; two plain :class:`Linear` modules share one grouped GEMM launch per
    pass (forward, dgrad, wgrad), adapters and other module types run one after the other."""
    if type(m0) is Linear and type(m1) is Linear:
        return L.linear_pair(x0, m0.weight, m0.bias, x1, m1.weight, m1.bias, epilogue=epilogue, gate0=gate0,
                             res0=res0, S0=S0, gate1=gate1, res1=res1, S1=S1)
    return m0(x0, epilogue, gate0, res0, S0), m1(x1, epilogue, gate1, res1, S1)


class RMSWeight(nn.Module):
    """Learned per-channel scale of an RMSNorm (the normalisation itself is fused elsewhere)."""

    def __init__(self, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0,
                       flip_sin_to_cos: bool = True) -> torch.Tensor:
    """Sinusoidal embedding of (continuous) timesteps in [0, 1000]."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    args = t.float()[:, None] * freqs[None]
    emb = torch.cat([torch.sin(args), torch.cos(args)], dim=-1)
    if flip_sin_to_cos:
        emb = torch.cat([emb[:, half:], emb[:, :half]], dim=-1)
    return emb


class TimestepMLP(nn.Module):
    def __init__(self, in_dim: int, dim: int):
        super().__init__()
        self.in_dim = in_dim
        self.linear_1 = Linear(in_dim, dim)
        self.linear_2 = Linear(dim, dim)

    def forward(self, x):
        return self.linear_2(F.silu(self.linear_1(x)))


def sincos_2d(embed_dim: int, grid_h: int, grid_w: int, base_size: Optional[int] = None) -> torch.Tensor:
    """Fixed 2D sin-cos positional table [grid_h*grid_w, embed_dim] (MAE/DiT style)."""
    gh = torch.arange(grid_h, dtype=torch.float64)
    gw = torch.arange(grid_w, dtype=torch.float64)
    if base_size is not None:
        gh = gh / (grid_h / base_size)
        gw = gw / (grid_w / base_size)
    yy, xx = torch.meshgrid(gh, gw, indexing="ij")

    def one(dim, pos):
        omega = 1.0 / 10000 ** (torch.arange(dim // 2, dtype=torch.float64) / (dim / 2.0))
        out = pos.reshape(-1)[:, None] * omega[None]
        return torch.cat([torch.sin(out), torch.cos(out)], dim=1)

    emb = torch.cat([one(embed_dim // 2, yy), one(embed_dim // 2, xx)], dim=1)
    return emb.float()


def rope_table(positions: torch.Tensor, dim: int, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [S, dim/2] for 1-D positions (interleaved pairs)."""
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    ang = positions.double()[:, None] * inv[None]
    return torch.cos(ang).float(), torch.sin(ang).float()


def rope_nd(grid: list[torch.Tensor], dims: list[int], theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Multi-axis RoPE (2D FLUX / 3D Wan): axis ``i`` uses ``dims[i]`` channels of each head."""
    cs, ss = [], []
    for pos, d in zip(grid, dims):
        c, s = rope_table(pos, d, theta)
        cs.append(c)
        ss.append(s)
    return torch.cat(cs, dim=-1), torch.cat(ss, dim=-1)


def patchify(x: torch.Tensor, p: int) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/p)*(W/p), p*p*C]."""
    B, C, H, W = x.shape
    x = x.view(B, C, H // p, p, W // p, p).permute(0, 2, 4, 3, 5, 1)
    return x.reshape(B, (H // p) * (W // p), p * p * C)


def unpatchify(x: torch.Tensor, p: int, C: int, H: int, W: int) -> torch.Tensor:
    B = x.shape[0]
    x = x.view(B, H // p, W // p, p, p, C).permute(0, 5, 1, 3, 2, 4)
    return x.reshape(B, C, H, W)


def patchify_3d(x: torch.Tensor, pt: int, ph: int, pw: int) -> torch.Tensor:
    """[B, C, F, H, W] -> [B, (F/pt)(H/ph)(W/pw), pt*ph*pw*C]."""
    B, C, Fr, H, W = x.shape
    x = x.view(B, C, Fr // pt, pt, H // ph, ph, W // pw, pw).permute(0, 2, 4, 6, 3, 5, 7, 1)
    return x.reshape(B, (Fr // pt) * (H // ph) * (W // pw), pt * ph * pw * C)


def unpatchify_3d(x: torch.Tensor, pt: int, ph: int, pw: int, C: int, Fr: int, H: int, W: int) -> torch.Tensor:
    B = x.shape[0]
    x = x.view(B, Fr // pt, H // ph, W // pw, pt, ph, pw, C).permute(0, 7, 1, 4, 2, 5, 3, 6)
    return x.reshape(B, C, Fr, H, W)
