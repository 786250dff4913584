"""Qwen-Image-shaped MMDiT (all double-stream blocks, multi-scale 3-axis RoPE), plus the Edit variant.

Shape family of diffusers' ``QwenImageTransformer2DModel`` as driven by the reference's Qwen-Image
adapters (``verl_omni/pipelines/qwen_image_flow_grpo/diffusers_training_adapter.py:66-239``,
``verl_omni/pipelines/qwen_image_edit_flow_grpo/diffusers_training_adapter.py:31``):

* latents [B, 16, H, W] are packed 2x2 into 64-feature tokens and embedded by ``img_in``;
* text: Qwen2.5-VL hidden states [B, St, 3584] -> RMSNorm -> ``txt_in``; an optional per-token mask
  marks padded prompt positions (they are excluded from every attention);
* ``temb`` = MLP(sinusoidal(t)) (no pooled text, no guidance embedding);
* ``depth`` joint blocks with separate image / text weights (AdaLN-Zero modulation, LayerNorm without
  affine, per-head q/k RMSNorm, RoPE, joint attention, GELU(tanh) MLP, gated residuals) -- the same
  block as the FLUX double stream, so the grouped image/text GEMM launches apply unchanged;
* RoPE on (frame, row, column) with ``axes_dim = (16, 56, 56)``: image positions are centred on the
  grid (rows -H/2 .. H/2 - 1), text tokens sit on the diagonal after the largest image index;
* Edit (image-to-image): the reference image's latents are packed the same way and appended to the
  image tokens at frame position 1; only the generated tokens are returned.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.flux import DoubleBlock, FluxConfig
from verl_omni_b200.models.layers import Linear, TimestepMLP, patchify, rope_nd, timestep_embedding, unpatchify
from verl_omni_b200.ops.norm import adaln_layernorm
from verl_omni_b200.parallel.ulysses import gather_key_mask, gather_sequence, local_rows, shard_sequence


@dataclass
class QwenImageConfig:
    in_channels: int = 16  # latent channels (64 features after 2x2 packing)
    patch_size: int = 2
    hidden: int = 3072
    heads: int = 24
    depth: int = 60
    mlp_ratio: float = 4.0
    joint_attention_dim: int = 3584
    axes_dim: tuple = (16, 56, 56)
    eps: float = 1e-6

    @staticmethod
    def qwen_image() -> "QwenImageConfig":
        return QwenImageConfig()

    @staticmethod
    def tiny() -> "QwenImageConfig":
        return QwenImageConfig(in_channels=4, hidden=128, heads=2, depth=2, joint_attention_dim=48,
                               axes_dim=(16, 24, 24))

    def block_config(self) -> FluxConfig:
        return FluxConfig(in_channels=self.in_channels, patch_size=self.patch_size, hidden=self.hidden,
                          heads=self.heads, depth_double=self.depth, depth_single=0, mlp_ratio=self.mlp_ratio,
                          axes_dim=self.axes_dim, eps=self.eps)


class QwenImageDiT(nn.Module):
    """forward(latents [B,C,H,W], timestep [B] in [0, 1000], prompt_embeds [B,St,3584],
    prompt_mask [B,St] or None, image_latents [B,C,H,W] or None (Edit))."""

    family = "qwen_image"

    def __init__(self, cfg: QwenImageConfig):
        super().__init__()
        self.cfg = cfg
        D, p = cfg.hidden, cfg.patch_size
        if sum(cfg.axes_dim) != D // cfg.heads:
            raise ValueError(f"RoPE axes {cfg.axes_dim} must cover the head dim {D // cfg.heads}")
        self.img_in = Linear(cfg.in_channels * p * p, D)
        self.txt_norm_weight = nn.Parameter(torch.ones(cfg.joint_attention_dim))
        self.txt_in = Linear(cfg.joint_attention_dim, D)
        self.time_embed = TimestepMLP(256, D)
        bc = cfg.block_config()
        self.transformer_blocks = nn.ModuleList([DoubleBlock(bc) for _ in range(cfg.depth)])
        self.norm_out_linear = Linear(D, 2 * D)
        self.proj_out = Linear(D, p * p * cfg.in_channels)
        self.gradient_checkpointing = False
        self._rope_cache: dict = {}

    def _positions(self, h: int, w: int, frame: int) -> list[torch.Tensor]:
        rows = torch.arange(h).float() - (h // 2)
        cols = torch.arange(w).float() - (w // 2)
        hh, ww = torch.meshgrid(rows, cols, indexing="ij")
        return [torch.full((h * w,), float(frame)), hh.reshape(-1), ww.reshape(-1)]

    def _rope(self, h: int, w: int, n_ref: int, St: int, device):
        key = (h, w, n_ref, St, str(device))
        if key not in self._rope_cache:
            axes = self._positions(h, w, 0)
            for r in range(n_ref):
                axes = [torch.cat([a, b]) for a, b in zip(axes, self._positions(h, w, r + 1))]
            start = float(max(h // 2, w // 2))
            txt = torch.arange(St).float() + start
            pos = [torch.cat([a, txt]) for a in axes]  # buffer order: image tokens (+ reference), then text
            c, s = rope_nd(pos, list(self.cfg.axes_dim))
            self._rope_cache[key] = (c.to(device).contiguous(), s.to(device).contiguous())
        return self._rope_cache[key]

    def forward(self, hidden_states, timestep, prompt_embeds, prompt_mask: Optional[torch.Tensor] = None,
                image_latents: Optional[torch.Tensor] = None):
        cfg = self.cfg
        p = cfg.patch_size
        B, C, Hh, Ww = hidden_states.shape
        dt = self.proj_out.weight.dtype
        x = patchify(hidden_states.to(dt), p)
        Sg = x.shape[1]
        n_ref = 0
        if image_latents is not None:
            x = torch.cat([x, patchify(image_latents.to(dt), p)], 1)
            n_ref = 1
        x = self.img_in(x)
        ta = F.silu(self.time_embed(timestep_embedding(timestep, 256).to(dt)))
        e = prompt_embeds.float()
        e = e * torch.rsqrt(e.pow(2).mean(-1, keepdim=True) + cfg.eps) * self.txt_norm_weight.float()
        c = self.txt_in(e.to(dt))
        Si, St = x.shape[1], c.shape[1]
        masked = prompt_mask is not None and not bool(prompt_mask.all())
        rope = rope_full = self._rope(Hh // p, Ww // p, n_ref, St, x.device)
        sp = getattr(self, "sp_group", None)
        kv_len = key_mask = None
        pm = prompt_mask.to(x.device).bool() if masked else None
        # right-padded prompts (valid text tokens form a prefix): keys past the image tokens + valid text
        # tokens are masked by a per-sequence key count on the tcgen05 kernels; other masks use a key mask
        padded = masked and bool((pm.int().cumprod(1).bool() == pm).all())
        if padded:
            kv_len = (Si + pm.sum(1)).to(torch.int32)
        if sp is not None:  # Ulysses: this rank keeps 1/sp of the image tokens and of the text tokens
            x, c = shard_sequence(x, sp), shard_sequence(c, sp)
            rope = (local_rows(rope[0], [Si, St], sp), local_rows(rope[1], [Si, St], sp))
            # key counts: the gathered keys are reordered image-first, text in prompt order
            if masked and not padded:  # valid keys in the gathered order [img_0 txt_0 img_1 txt_1 ...]
                local = torch.cat([torch.ones(B, x.shape[1], dtype=torch.bool, device=x.device),
                                   shard_sequence(pm, sp)], 1)
                key_mask = gather_key_mask(local, sp)
        elif masked and not padded:
            key_mask = torch.cat([torch.ones(B, Si, dtype=torch.bool, device=x.device), pm], 1)
        for blk in self.transformer_blocks:
            x, c = blk(x, c, ta, rope, kv_len, sp_group=sp, key_mask=key_mask, rope_full=rope_full)
        x = adaln_layernorm(x, self.norm_out_linear(ta), 1, 0, 2, cfg.eps)
        y = self.proj_out(x)
        if sp is not None:
            y = gather_sequence(y, sp)
        y = y[:, :Sg].contiguous() if n_ref else y
        return unpatchify(y, p, cfg.in_channels, Hh, Ww).float()
