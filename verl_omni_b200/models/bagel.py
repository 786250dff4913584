"""BAGEL-shaped Mixture-of-Transformers (MoT) image generator (non-diffusers model).

Shape family of the model trained by the reference's ``verl_omni/pipelines/bagel_flow_grpo``
(``bagel_model.py:201-339``): a Qwen2.5-7B-shaped decoder (hidden 3584, 28 layers, 28 query / 4 KV heads of
128, SwiGLU 18944) whose every layer has two weight sets -- the understanding expert for text tokens and the
generation expert for the noisy VAE-latent tokens -- sharing one attention:

* text (prompt) tokens attend causally among themselves;
* latent tokens attend to every prompt token and bidirectionally to each other.

Per layer both experts' projections run as grouped tcgen05 GEMM launches (text rows with the
understanding weights, latent rows with the generation weights in one launch); attention runs as two FMHA
calls (causal text block, then the latent queries over all keys).  Latents are 2x2-packed 16-channel VAE
tokens embedded by a linear layer plus a timestep embedding; the velocity head reads the latent tokens.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from verl_omni_b200.models.layers import (Linear, TimestepMLP, linear_pair, patchify, rope_nd, timestep_embedding,
                                         unpatchify)
from verl_omni_b200.ops import llm as LO
from verl_omni_b200.ops.attention import attention


@dataclass
class BagelConfig:
    vocab: int = 152064
    hidden: int = 3584
    layers: int = 28
    q_heads: int = 28
    kv_heads: int = 4
    head_dim: int = 128
    ffn: int = 18944
    latent_channels: int = 16
    patch_size: int = 2
    rope_theta: float = 1_000_000.0
    eps: float = 1e-6

    @staticmethod
    def bagel_7b_mot() -> "BagelConfig":
        return BagelConfig()

    @staticmethod
    def tiny() -> "BagelConfig":
        return BagelConfig(vocab=512, hidden=128, layers=2, q_heads=4, kv_heads=2, head_dim=32, ffn=256,
                           latent_channels=4)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return LO.rms_norm(x.contiguous(), w, eps)  # one fused kernel per row on CUDA


class _Expert(nn.Module):
    def __init__(self, cfg: BagelConfig):
        super().__init__()
        D, hd = cfg.hidden, cfg.head_dim
        self.ln1 = nn.Parameter(torch.ones(D))
        self.qkv = Linear(D, (cfg.q_heads + 2 * cfg.kv_heads) * hd)
        self.q_norm = nn.Parameter(torch.ones(hd))
        self.k_norm = nn.Parameter(torch.ones(hd))
        self.o = Linear(cfg.q_heads * hd, D, bias=False)
        self.ln2 = nn.Parameter(torch.ones(D))
        self.gate_up = Linear(D, 2 * cfg.ffn, bias=False)
        self.down = Linear(cfg.ffn, D, bias=False)


class MoTLayer(nn.Module):
    def __init__(self, cfg: BagelConfig):
        super().__init__()
        self.cfg = cfg
        self.und, self.gen = _Expert(cfg), _Expert(cfg)

    def _heads(self, qkv, e: _Expert, B, S, cos, sin):
        cfg = self.cfg
        hd, Hq, Hk = cfg.head_dim, cfg.q_heads, cfg.kv_heads
        # per-head RMSNorm + rotate-half RoPE read straight out of the QKV projection (one kernel each)
        x3 = qkv.view(B, S, (Hq + 2 * Hk) * hd)
        c2, s2 = cos.reshape(S, hd // 2), sin.reshape(S, hd // 2)
        q = LO.head_norm_rope(x3, 0, Hq, e.q_norm, c2, s2, cfg.eps)
        k = LO.head_norm_rope(x3, Hq * hd, Hk, e.k_norm, c2, s2, cfg.eps)
        v = qkv.view(B, S, Hq + 2 * Hk, hd)[:, :, Hq + Hk:]
        return q, k, v.transpose(1, 2)

    def forward(self, xt, xl, rope_t, rope_l):
        cfg = self.cfg
        B, St, D = xt.shape
        Sl = xl.shape[1]
        rep = cfg.q_heads // cfg.kv_heads
        qkv_t, qkv_l = linear_pair(self.und.qkv, _rms(xt, self.und.ln1, cfg.eps), self.gen.qkv,
                                   _rms(xl, self.gen.ln1, cfg.eps))
        qt, kt, vt = self._heads(qkv_t, self.und, B, St, *rope_t)
        ql, kl, vl = self._heads(qkv_l, self.gen, B, Sl, *rope_l)
        k_all = torch.cat([kt, kl], 2).repeat_interleave(rep, 1).contiguous()
        v_all = torch.cat([vt, vl], 2).repeat_interleave(rep, 1).contiguous()
        # prompt tokens: causal over the prompt; latent tokens: every prompt token and all latents
        ot = attention(qt.contiguous(), k_all[:, :, :St].contiguous(), v_all[:, :, :St].contiguous(), causal=True)
        ol = attention(ql.contiguous(), k_all, v_all)
        xt, xl = self._out(ot, ol, xt, xl)
        gu_t, gu_l = linear_pair(self.und.gate_up, _rms(xt, self.und.ln2, cfg.eps), self.gen.gate_up,
                                 _rms(xl, self.gen.ln2, cfg.eps))
        at, al = LO.swiglu(gu_t.contiguous()), LO.swiglu(gu_l.contiguous())
        dt_, dl_ = linear_pair(self.und.down, at, self.gen.down, al)
        return xt + dt_, xl + dl_

    def _out(self, ot, ol, xt, xl):
        yt, yl = linear_pair(self.und.o, ot, self.gen.o, ol)
        return xt + yt, xl + yl


class BagelMoT(nn.Module):
    """forward(latents [B, C, H, W], timestep [B] in [0, 1000], prompt_ids [B, St] int64) -> velocity."""

    family = "bagel"

    def __init__(self, cfg: BagelConfig):
        super().__init__()
        self.cfg = cfg
        D, p = cfg.hidden, cfg.patch_size
        self.embed_tokens = nn.Embedding(cfg.vocab, D)
        self.vae2llm = Linear(cfg.latent_channels * p * p, D)
        self.time_embedder = TimestepMLP(256, D)
        self.layers = nn.ModuleList([MoTLayer(cfg) for _ in range(cfg.layers)])
        self.norm_und = nn.Parameter(torch.ones(D))
        self.norm_gen = nn.Parameter(torch.ones(D))
        self.llm2vae = Linear(D, cfg.latent_channels * p * p)
        self.gradient_checkpointing = False
        self._rope_cache: dict = {}

    def _ropes(self, St: int, h: int, w: int, device):
        key = (St, h, w, str(device))
        if key not in self._rope_cache:
            hd = self.cfg.head_dim
            ct, stt = rope_nd([torch.arange(St).float()], [hd], theta=self.cfg.rope_theta)
            # latent tokens share the position after the prompt (one image "token" position), 2-D offsets
            # inside the image come from the latent position embedding in the generation expert's input
            pos = torch.full((h * w,), float(St))
            cl, sl = rope_nd([pos], [hd], theta=self.cfg.rope_theta)
            self._rope_cache[key] = ((ct.to(device)[None, :, None], stt.to(device)[None, :, None]),
                                     (cl.to(device)[None, :, None], sl.to(device)[None, :, None]))
        return self._rope_cache[key]

    def forward(self, latents, timestep, prompt_ids):
        cfg = self.cfg
        p = cfg.patch_size
        B, C, Hh, Ww = latents.shape
        dt = self.llm2vae.weight.dtype
        xt = self.embed_tokens(prompt_ids.long()).to(dt)
        xl = self.vae2llm(patchify(latents.to(dt), p))
        xl = xl + self.time_embedder(timestep_embedding(timestep, 256).to(dt))[:, None]
        h, w = Hh // p, Ww // p
        hh, ww = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
        pe = torch.cat(rope_nd([hh.reshape(-1).float(), ww.reshape(-1).float()], [cfg.hidden // 2, cfg.hidden // 2]),
                       -1)
        xl = xl + pe.to(xl.device, dt)[None] * 0.02
        rope_t, rope_l = self._ropes(xt.shape[1], h, w, xt.device)
        for layer in self.layers:
            if self.gradient_checkpointing and torch.is_grad_enabled():
                xt, xl = torch.utils.checkpoint.checkpoint(layer, xt, xl, rope_t, rope_l, use_reentrant=False)
            else:
                xt, xl = layer(xt, xl, rope_t, rope_l)
        out = self.llm2vae(_rms(xl, self.norm_gen, cfg.eps))
        return unpatchify(out, p, cfg.latent_channels, Hh, Ww).float()
