"""SD3 / SD3.5-shaped MMDiT (joint text+image attention transformer) built on the sm_100a ops.

Shape family of diffusers' ``SD3Transformer2DModel`` as used by the reference SD3.5 FlowGRPO
adapter (``verl_omni/pipelines/sd3_flow_grpo/diffusers_training_adapter.py:48-181``):

* patch embed (p=2) + fixed 2D sin-cos positions; timestep (256-d sinusoid) + pooled-text MLPs
  summed into ``temb``; ``context_embedder`` maps the joint CLIP+T5 token sequence to the width;
* ``depth`` joint blocks: per-stream AdaLN-Zero modulation, per-head RMS qk-norm, one joint
  attention over ``[image ; text]`` tokens, gated residual out-projections and GELU(tanh) MLPs.
  The first ``dual_attention_layers`` blocks add an image-only self-attention branch
  (SD3.5 "MMDiT-X"); the last block is ``context_pre_only`` (text stream feeds k/v only);
* AdaLN-continuous output norm + linear to ``p*p*C`` and unpatchify.

Every linear runs on the tcgen05 GEMM (gated residuals and GELU fused into the epilogue), the
AdaLN norms and the qk-norm/QKV split are fused kernels, and attention is the tcgen05 FMHA.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import (Linear, RMSWeight, TimestepMLP, linear_pair, patchify, sincos_2d,
                                         timestep_embedding, unpatchify)
from verl_omni_b200.ops.norm import adaln_layernorm, qk_norm_split_into
from verl_omni_b200.parallel import ulysses_fused as UF
from verl_omni_b200.parallel.ulysses import (gather_key_mask, gather_sequence, joint_attention, pad_to_multiple,
                                             shard_sequence, sp_info, ulysses_attention)


@dataclass
class MMDiTConfig:
    in_channels: int = 16
    out_channels: int = 16
    patch_size: int = 2
    hidden: int = 1536
    heads: int = 24
    depth: int = 24
    mlp_ratio: float = 4.0
    joint_attention_dim: int = 4096
    pooled_projection_dim: int = 2048
    pos_embed_max_size: int = 384
    sample_size: int = 64
    dual_attention_layers: int = 13
    qk_norm: bool = True
    eps: float = 1e-6

    @staticmethod
    def sd35_medium() -> "MMDiTConfig":
        return MMDiTConfig()

    @staticmethod
    def small() -> "MMDiTConfig":
        """Miniature with the full-size head width (64) and GEMMs of >= 128 rows: the smallest shape that
        runs every hot op of the full model on its native kernel (32x32 latents -> 256 image tokens)."""
        return MMDiTConfig(hidden=256, heads=4, depth=2, joint_attention_dim=256, pooled_projection_dim=128,
                           dual_attention_layers=1, sample_size=32, pos_embed_max_size=32)

    @staticmethod
    def tiny(hidden: int = 64, heads: int = 2, depth: int = 2) -> "MMDiTConfig":
        return MMDiTConfig(hidden=hidden, heads=heads, depth=depth, joint_attention_dim=48,
                           pooled_projection_dim=32, dual_attention_layers=1, sample_size=8, in_channels=4,
                           out_channels=4, pos_embed_max_size=16)


class JointBlock(nn.Module):
    def __init__(self, cfg: MMDiTConfig, context_pre_only: bool, dual: bool):
        super().__init__()
        D = cfg.hidden
        self.D, self.H = D, cfg.heads
        self.dh = D // cfg.heads
        self.cpo = context_pre_only
        self.dual = dual
        self.n_mod = 9 if dual else 6
        self.n_mod_c = 2 if context_pre_only else 6
        self.norm1_linear = Linear(D, self.n_mod * D)
        self.norm1_context_linear = Linear(D, self.n_mod_c * D)
        self.to_qkv = Linear(D, 3 * D)
        self.add_qkv = Linear(D, 3 * D)
        self.norm_q, self.norm_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.norm_added_q, self.norm_added_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.to_out = Linear(D, D)
        hid = int(D * cfg.mlp_ratio)
        self.ff_1, self.ff_2 = Linear(D, hid), Linear(hid, D)
        if not context_pre_only:
            self.to_add_out = Linear(D, D)
            self.ff_context_1, self.ff_context_2 = Linear(D, hid), Linear(hid, D)
        if dual:
            self.attn2_qkv = Linear(D, 3 * D)
            self.attn2_out = Linear(D, D)
            self.norm2_q, self.norm2_k = RMSWeight(self.dh), RMSWeight(self.dh)
        self.eps = cfg.eps

    def forward(self, x: torch.Tensor, c: torch.Tensor, temb_act: torch.Tensor, sp_group=None, key_mask=None):
        B, Si, D = x.shape
        St = c.shape[1]
        H, dh = self.H, self.dh
        mod = self.norm1_linear(temb_act)  # [B, n_mod*D]
        modc = self.norm1_context_linear(temb_act)
        # chunk order: 0 shift_msa, 1 scale_msa, 2 gate_msa, 3 shift_mlp, 4 scale_mlp, 5 gate_mlp,
        #              6 shift_msa2, 7 scale_msa2, 8 gate_msa2
        h = adaln_layernorm(x, mod, 0, 1, self.n_mod, self.eps)
        # AdaLayerNormZero chunks: shift, scale, ...; the context-pre-only block's AdaLayerNormContinuous: scale, shift
        hc = adaln_layernorm(c, modc, 1 if self.cpo else 0, 0 if self.cpo else 1, self.n_mod_c, self.eps)
        S = Si + St
        dev, dt = x.device, x.dtype
        if (key_mask is None and type(self.to_qkv) is Linear and type(self.add_qkv) is Linear
                and UF.enabled(sp_group, x, H, D)):
            # sequence-parallel inference: both exchanges inside the QKV GEMM and attention kernels
            o_img, o_txt = UF.joint_attention_fused(h, hc, self.to_qkv, self.add_qkv,
                                                    (self.norm_q.weight, self.norm_k.weight),
                                                    (self.norm_added_q.weight, self.norm_added_k.weight), H,
                                                    sp_group, eps=self.eps)
        else:
            qkv, qkvc = linear_pair(self.to_qkv, h, self.add_qkv, hc)
            qkv, qkvc = qkv.reshape(B * Si, 3 * D), qkvc.reshape(B * St, 3 * D)
            q = torch.empty(B, H, S, dh, device=dev, dtype=dt)
            k = torch.empty(B, H, S, dh, device=dev, dtype=dt)
            v = torch.empty(B, H, S, dh, device=dev, dtype=dt)
            q, k, v = qk_norm_split_into(q, k, v, qkv, self.norm_q.weight, self.norm_k.weight, Si, 0, eps=self.eps)
            q, k, v = qk_norm_split_into(q, k, v, qkvc, self.norm_added_q.weight, self.norm_added_k.weight, St, Si,
                                         eps=self.eps)
            o_img, o_txt = joint_attention(q, k, v, Si, sp_group=sp_group, key_mask=key_mask)  # [B, Si|St, D]
        gate_msa = mod.view(B, self.n_mod, D)[:, 2]
        mc = modc.view(B, self.n_mod_c, D)
        if self.cpo:
            x_new = self.to_out(o_img, epilogue="gate_res", gate=gate_msa, res=x, S=Si)
        else:
            x_new, c = linear_pair(self.to_out, o_img, self.to_add_out, o_txt, "gate_res", gate_msa, x, Si,
                                   mc[:, 2], c, St)
        if self.dual:
            h2 = adaln_layernorm(x, mod, 6, 7, self.n_mod, self.eps)
            if type(self.attn2_qkv) is Linear and UF.enabled(sp_group, x, H, D):
                o2, _ = UF.joint_attention_fused(h2, None, self.attn2_qkv, None,
                                                 (self.norm2_q.weight, self.norm2_k.weight), None, H, sp_group,
                                                 eps=self.eps)
            else:
                qkv2 = self.attn2_qkv(h2).reshape(B * Si, 3 * D)
                q2 = torch.empty(B, H, Si, dh, device=dev, dtype=dt)
                k2 = torch.empty_like(q2)
                v2 = torch.empty_like(q2)
                q2, k2, v2 = qk_norm_split_into(q2, k2, v2, qkv2, self.norm2_q.weight, self.norm2_k.weight, Si, 0,
                                                eps=self.eps)
                o2 = ulysses_attention(q2, k2, v2, sp_group)
            x_new = self.attn2_out(o2, epilogue="gate_res", gate=mod.view(B, self.n_mod, D)[:, 8], res=x_new, S=Si)
        x = x_new
        hm = adaln_layernorm(x, mod, 3, 4, self.n_mod, self.eps)
        gate_mlp = mod.view(B, self.n_mod, D)[:, 5]
        if self.cpo:
            u = self.ff_1(hm, epilogue="gelu")
            return self.ff_2(u, epilogue="gate_res", gate=gate_mlp, res=x, S=Si), None
        hcm = adaln_layernorm(c, modc, 3, 4, self.n_mod_c, self.eps)
        u, uc = linear_pair(self.ff_1, hm, self.ff_context_1, hcm, "gelu")
        x, c = linear_pair(self.ff_2, u, self.ff_context_2, uc, "gate_res", gate_mlp, x, Si, mc[:, 5], c, St)
        return x, c


class MMDiT(nn.Module):
    """Input latents ``[B, C, H, W]`` (fp32 or bf16), timesteps ``[B]`` in [0, 1000],
    ``encoder_hidden_states [B, St, joint_attention_dim]``, ``pooled_projections [B, pooled_dim]``.
    Returns the velocity prediction ``[B, C, H, W]`` in fp32."""

    family = "sd3"

    def __init__(self, cfg: MMDiTConfig):
        super().__init__()
        self.cfg = cfg
        D, p = cfg.hidden, cfg.patch_size
        self.pos_embed_proj = Linear(cfg.in_channels * p * p, D)
        grid = cfg.pos_embed_max_size
        self.register_buffer("pos_table", sincos_2d(D, grid, grid, base_size=cfg.sample_size // p), persistent=False)
        self.time_embed = TimestepMLP(256, D)
        self.text_embed = TimestepMLP(cfg.pooled_projection_dim, D)
        self.context_embedder = Linear(cfg.joint_attention_dim, D)
        self.transformer_blocks = nn.ModuleList([
            JointBlock(cfg, context_pre_only=(i == cfg.depth - 1), dual=(i < cfg.dual_attention_layers))
            for i in range(cfg.depth)])
        self.norm_out_linear = Linear(D, 2 * D)
        self.proj_out = Linear(D, p * p * cfg.out_channels)
        self.gradient_checkpointing = False

    def _pos(self, h: int, w: int) -> torch.Tensor:
        g = self.cfg.pos_embed_max_size
        top, left = (g - h) // 2, (g - w) // 2
        t = self.pos_table.view(g, g, -1)[top:top + h, left:left + w]
        return t.reshape(h * w, -1)

    def forward(self, hidden_states, timestep, encoder_hidden_states, pooled_projections):
        cfg = self.cfg
        p = cfg.patch_size
        B, C, Hh, Ww = hidden_states.shape
        dt = self.proj_out.weight.dtype
        x = patchify(hidden_states.to(dt), p)
        x = self.pos_embed_proj(x)
        x = x + self._pos(Hh // p, Ww // p).to(dt)[None]
        temb = self.time_embed(timestep_embedding(timestep, 256).to(dt)) + self.text_embed(pooled_projections.to(dt))
        temb_act = F.silu(temb)
        c = self.context_embedder(encoder_hidden_states.to(dt))
        sp = getattr(self, "sp_group", None)
        key_mask = None
        if sp is not None:
            # Ulysses: 1/sp of the image tokens and of the (zero-padded, masked) text tokens per rank
            St = c.shape[1]
            r, W = sp_info(sp)
            c = pad_to_multiple(c, W, 1)
            x, c = shard_sequence(x, sp), shard_sequence(c, sp)
            if c.shape[1] * W != St:
                txt_ok = (torch.arange(c.shape[1], device=c.device) + r * c.shape[1]) < St
                local = torch.cat([torch.ones(x.shape[1], dtype=torch.bool, device=x.device), txt_ok])
                key_mask = gather_key_mask(local[None].expand(B, -1), sp)
        for blk in self.transformer_blocks:
            if self.gradient_checkpointing and torch.is_grad_enabled():
                x, c = torch.utils.checkpoint.checkpoint(blk, x, c, temb_act, sp, key_mask, use_reentrant=False)
            else:
                x, c = blk(x, c, temb_act, sp, key_mask)
        mod = self.norm_out_linear(temb_act)
        h = adaln_layernorm(x, mod, 1, 0, 2, cfg.eps)
        out = self.proj_out(h)
        if sp is not None:
            out = gather_sequence(out, sp)
        return unpatchify(out, p, cfg.out_channels, Hh, Ww).float()
