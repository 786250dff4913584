"""FLUX.1-dev-shaped rectified-flow transformer (double-stream + single-stream blocks, 2D RoPE).

Shape family of diffusers' ``FluxTransformer2DModel`` (reached through the reference's diffusers
adapters): patchified 16-channel latents (2x2 -> 64 features), timestep + guidance + pooled-text MLPs
summed into ``temb``, ``depth_double`` MMDiT-style blocks with separate image/text weights and joint
attention, then ``depth_single`` parallel blocks on the concatenated sequence (attention and GELU MLP
side by side, one gated output projection).  Rotary embeddings on 3 axes (text id, row, column) with
``axes_dim = (16, 56, 56)``; text tokens sit at position 0 on every axis.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import (Linear, RMSWeight, TimestepMLP, linear_pair, patchify, rope_nd,
                                         timestep_embedding, unpatchify)
from verl_omni_b200.ops.attention import attention, attention_split  # noqa: F401
from verl_omni_b200.parallel import ulysses_fused as UF
from verl_omni_b200.parallel.ulysses import gather_sequence, joint_attention, local_rows, shard_sequence, ulysses_attention
from verl_omni_b200.ops.norm import adaln_layernorm, qk_norm_split_into


@dataclass
class FluxConfig:
    in_channels: int = 16
    patch_size: int = 2
    hidden: int = 3072
    heads: int = 24
    depth_double: int = 19
    depth_single: int = 38
    mlp_ratio: float = 4.0
    joint_attention_dim: int = 4096
    pooled_projection_dim: int = 768
    axes_dim: tuple = (16, 56, 56)
    guidance_embeds: bool = True
    eps: float = 1e-6

    @staticmethod
    def flux1_dev() -> "FluxConfig":
        return FluxConfig()

    @staticmethod
    def tiny() -> "FluxConfig":
        return FluxConfig(in_channels=4, hidden=128, heads=2, depth_double=1, depth_single=1,
                          joint_attention_dim=48, pooled_projection_dim=32, axes_dim=(16, 24, 24))


class DoubleBlock(nn.Module):
    def __init__(self, cfg: FluxConfig):
        super().__init__()
        D = cfg.hidden
        self.H, self.dh, self.eps = cfg.heads, D // cfg.heads, cfg.eps
        hid = int(D * cfg.mlp_ratio)
        for s in ("img", "txt"):
            setattr(self, f"{s}_mod", Linear(D, 6 * D))
            setattr(self, f"{s}_qkv", Linear(D, 3 * D))
            setattr(self, f"{s}_norm_q", RMSWeight(self.dh))
            setattr(self, f"{s}_norm_k", RMSWeight(self.dh))
            setattr(self, f"{s}_out", Linear(D, D))
            setattr(self, f"{s}_mlp_1", Linear(D, hid))
            setattr(self, f"{s}_mlp_2", Linear(hid, D))

    def forward(self, x, c, temb_act, rope, kv_len=None, sp_group=None, key_mask=None, rope_full=None):
        B, Si, D = x.shape
        St = c.shape[1]
        H, dh = self.H, self.dh
        mi, mt = self.img_mod(temb_act), self.txt_mod(temb_act)
        hi = adaln_layernorm(x, mi, 0, 1, 6, self.eps)
        ht = adaln_layernorm(c, mt, 0, 1, 6, self.eps)
        S = Si + St
        if (key_mask is None and kv_len is None and type(self.img_qkv) is Linear and type(self.txt_qkv) is Linear
                and UF.enabled(sp_group, x, H, D)):
            # sequence-parallel inference: both exchanges inside the QKV GEMM and attention kernels
            o_img, o_txt = UF.joint_attention_fused(hi, ht, self.img_qkv, self.txt_qkv,
                                                    (self.img_norm_q.weight, self.img_norm_k.weight),
                                                    (self.txt_norm_q.weight, self.txt_norm_k.weight), H, sp_group,
                                                    rope=rope_full, eps=self.eps)
        else:
            mk = lambda: torch.empty(B, H, S, dh, device=x.device, dtype=x.dtype)  # noqa: E731
            qkv_i, qkv_t = linear_pair(self.img_qkv, hi, self.txt_qkv, ht)
            q, k, v = qk_norm_split_into(mk(), mk(), mk(), qkv_i.reshape(B * Si, 3 * D), self.img_norm_q.weight,
                                         self.img_norm_k.weight, Si, 0, rope=rope, eps=self.eps)
            q, k, v = qk_norm_split_into(q, k, v, qkv_t.reshape(B * St, 3 * D), self.txt_norm_q.weight,
                                         self.txt_norm_k.weight, St, Si, rope=rope, eps=self.eps)
            o_img, o_txt = joint_attention(q, k, v, Si, sp_group=sp_group, kv_len=kv_len, key_mask=key_mask)
        vi, vt = mi.view(B, 6, D), mt.view(B, 6, D)
        x, c = linear_pair(self.img_out, o_img, self.txt_out, o_txt, "gate_res", vi[:, 2], x, Si, vt[:, 2], c, St)
        ui, ut = linear_pair(self.img_mlp_1, adaln_layernorm(x, mi, 3, 4, 6, self.eps), self.txt_mlp_1,
                             adaln_layernorm(c, mt, 3, 4, 6, self.eps), "gelu")
        x, c = linear_pair(self.img_mlp_2, ui, self.txt_mlp_2, ut, "gate_res", vi[:, 5], x, Si, vt[:, 5], c, St)
        return x, c


class SingleBlock(nn.Module):
    def __init__(self, cfg: FluxConfig):
        super().__init__()
        D = cfg.hidden
        self.H, self.dh, self.eps = cfg.heads, D // cfg.heads, cfg.eps
        hid = int(D * cfg.mlp_ratio)
        self.mod = Linear(D, 3 * D)
        self.qkv = Linear(D, 3 * D)
        self.mlp_in = Linear(D, hid)
        self.norm_q, self.norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.proj_out = Linear(D + hid, D)

    def forward(self, x, temb_act, rope, sp_group=None):
        B, S, D = x.shape
        m = self.mod(temb_act)
        h = adaln_layernorm(x, m, 0, 1, 3, self.eps)
        mk = lambda: torch.empty(B, self.H, S, self.dh, device=x.device, dtype=x.dtype)  # noqa: E731
        q, k, v = qk_norm_split_into(mk(), mk(), mk(), self.qkv(h).reshape(B * S, 3 * D), self.norm_q.weight,
                                     self.norm_k.weight, S, 0, rope=rope, eps=self.eps)
        o = ulysses_attention(q, k, v, sp_group)
        a = self.mlp_in(h, epilogue="gelu")
        return self.proj_out(torch.cat([o, a], -1), epilogue="gate_res", gate=m.view(B, 3, D)[:, 2], res=x, S=S)


class FluxDiT(nn.Module):
    """forward(latents [B,C,H,W], timestep [B], encoder_hidden_states [B,St,4096], pooled [B,768], guidance)."""

    family = "flux"

    def __init__(self, cfg: FluxConfig):
        super().__init__()
        self.cfg = cfg
        D, p = cfg.hidden, cfg.patch_size
        if sum(cfg.axes_dim) != D // cfg.heads:
            raise ValueError(f"RoPE axes {cfg.axes_dim} must cover the head dim {D // cfg.heads}")
        self.x_embedder = Linear(cfg.in_channels * p * p, D)
        self.time_embed = TimestepMLP(256, D)
        self.guidance_embed = TimestepMLP(256, D) if cfg.guidance_embeds else None
        self.text_embed = TimestepMLP(cfg.pooled_projection_dim, D)
        self.context_embedder = Linear(cfg.joint_attention_dim, D)
        self.transformer_blocks = nn.ModuleList([DoubleBlock(cfg) for _ in range(cfg.depth_double)])
        self.single_transformer_blocks = nn.ModuleList([SingleBlock(cfg) for _ in range(cfg.depth_single)])
        self.norm_out_linear = Linear(D, 2 * D)
        self.proj_out = Linear(D, p * p * cfg.in_channels)
        self.gradient_checkpointing = False
        self._rope_cache: dict = {}

    def _rope(self, h: int, w: int, St: int, device):
        key = (h, w, St, str(device))
        if key not in self._rope_cache:
            hh, ww = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
            img = [torch.zeros(h * w), hh.reshape(-1).float(), ww.reshape(-1).float()]
            txt = [torch.zeros(St)] * 3
            pos = [torch.cat([a, b]) for a, b in zip(img, txt)]  # buffer order: image tokens, then text
            c, s = rope_nd(pos, list(self.cfg.axes_dim))
            self._rope_cache[key] = (c.to(device).contiguous(), s.to(device).contiguous())
        return self._rope_cache[key]

    def forward(self, hidden_states, timestep, encoder_hidden_states, pooled_projections, guidance=None):
        cfg = self.cfg
        p = cfg.patch_size
        B, C, Hh, Ww = hidden_states.shape
        dt = self.proj_out.weight.dtype
        x = self.x_embedder(patchify(hidden_states.to(dt), p))
        temb = self.time_embed(timestep_embedding(timestep, 256).to(dt)) + self.text_embed(pooled_projections.to(dt))
        if self.guidance_embed is not None:
            g = guidance if guidance is not None else torch.full_like(timestep, 3.5)
            temb = temb + self.guidance_embed(timestep_embedding(g.float() * 1000.0, 256).to(dt))
        ta = F.silu(temb)
        c = self.context_embedder(encoder_hidden_states.to(dt))
        Si, St = x.shape[1], c.shape[1]
        rope = self._rope(Hh // p, Ww // p, St, x.device)
        sp = getattr(self, "sp_group", None)
        rope_full = rope
        if sp is not None:  # Ulysses: this rank keeps 1/sp of the image tokens and of the text tokens
            x, c = shard_sequence(x, sp), shard_sequence(c, sp)
            rope = (local_rows(rope[0], [Si, St], sp), local_rows(rope[1], [Si, St], sp))
        Sl = x.shape[1]
        ckpt = self.gradient_checkpointing and torch.is_grad_enabled()
        for blk in self.transformer_blocks:
            if ckpt:  # keep only block inputs; the block's activations are recomputed in backward
                x, c = torch.utils.checkpoint.checkpoint(blk, x, c, ta, rope, None, sp, None, rope_full,
                                                         use_reentrant=False)
            else:
                x, c = blk(x, c, ta, rope, sp_group=sp, rope_full=rope_full)
        xs = torch.cat([x, c], 1)
        for blk in self.single_transformer_blocks:
            if ckpt:
                xs = torch.utils.checkpoint.checkpoint(blk, xs, ta, rope, sp, use_reentrant=False)
            else:
                xs = blk(xs, ta, rope, sp_group=sp)
        x = xs[:, :Sl].contiguous()
        x = adaln_layernorm(x, self.norm_out_linear(ta), 1, 0, 2, cfg.eps)
        y = self.proj_out(x)
        if sp is not None:
            y = gather_sequence(y, sp)
        return unpatchify(y, p, cfg.in_channels, Hh, Ww).float()
