"""Qwen3-Omni-30B-A3B-shaped MoE "thinker" LLM with audio and vision encoders.

Architecture (random-init): ``layers`` decoder blocks of RMSNorm -> GQA attention (``q_heads`` query
heads, ``kv_heads`` key/value heads, per-head RMS q/k-norm, RoPE) -> RMSNorm -> sparse MoE
(softmax router, top-``k`` of ``experts`` SwiGLU experts of width ``expert_ffn``, renormalised gates);
tied-size LM head over ``vocab``.  Multimodal prompts carry placeholder ids (``audio_token`` /
``image_token``) whose embeddings are replaced by the projected outputs of an audio encoder over
128-dim log-mel frames and a ViT over image patches, as in the reference's Qwen3-Omni thinker
adapter (``verl_omni/pipelines/qwen3_omni/thinker_training_adapter.py:34-206``).

Expert computation groups tokens by expert (sort by expert id, one GEMM per non-empty expert on the
tcgen05 GEMM; combine weighted by the gates).  ``ExpertParallel`` dispatches token groups to the
expert-owning ranks with all-to-all and combines the results back (see ``parallel/expert_parallel.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from verl_omni_b200.models.layers import Linear, rope_table
from verl_omni_b200.ops import llm as LO
from verl_omni_b200.ops.attention import attention
from verl_omni_b200.ops import linear as L
from verl_omni_b200.ops.decode import KVCache, PagedView, decode_attention
from verl_omni_b200.parallel import dist as D_


@dataclass
class MoEConfig:
    vocab: int = 151936
    hidden: int = 2048
    layers: int = 48
    q_heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    expert_ffn: int = 768
    rope_theta: float = 1_000_000.0
    audio_layers: int = 32
    audio_dim: int = 1280
    audio_mel: int = 128
    vision_layers: int = 27
    vision_dim: int = 1152
    vision_patch_dim: int = 3 * 16 * 16
    audio_token: int = 151646
    image_token: int = 151655
    eps: float = 1e-6

    @staticmethod
    def qwen3_omni_30b_a3b() -> "MoEConfig":
        return MoEConfig()

    @staticmethod
    def tiny() -> "MoEConfig":
        return MoEConfig(vocab=512, hidden=64, layers=2, q_heads=4, kv_heads=2, head_dim=16, experts=8, top_k=2,
                         expert_ffn=32, audio_layers=1, audio_dim=32, audio_mel=16, vision_layers=1, vision_dim=32,
                         vision_patch_dim=48, audio_token=510, image_token=511)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Row RMSNorm: the fused kernel on bf16 CUDA tensors, the fp32 oracle otherwise."""
    return LO.rms_norm(x.contiguous(), w, eps)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, H, S, D] (rotate-half convention), cos/sin [S, D/2]."""
    d2 = x.shape[-1] // 2
    x1, x2 = x[..., :d2], x[..., d2:]
    c, s = cos.to(x.dtype)[None, None], sin.to(x.dtype)[None, None]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1)


class MoEBlock(nn.Module):
    def __init__(self, cfg: MoEConfig, ep=None):
        super().__init__()
        self.cfg = cfg
        D, hd = cfg.hidden, cfg.head_dim
        self.ln1 = nn.Parameter(torch.ones(D))
        self.q_proj = Linear(D, cfg.q_heads * hd, bias=False)
        self.kv_proj = Linear(D, 2 * cfg.kv_heads * hd, bias=False)
        self.o_proj = Linear(cfg.q_heads * hd, D, bias=False)
        self.q_norm = nn.Parameter(torch.ones(hd))
        self.k_norm = nn.Parameter(torch.ones(hd))
        self.ln2 = nn.Parameter(torch.ones(D))
        self.router = Linear(D, cfg.experts, bias=False)
        E, F_ = cfg.experts, cfg.expert_ffn
        # expert parallelism: this rank holds experts [e0, e0 + El) only; each expert's initial weights come
        # from its own seeded generator, so a sharded model equals the slices of the unsharded one
        El = E if ep is None else ep.per_rank
        self.e0 = 0 if ep is None else ep.rank * ep.per_rank
        base = int(torch.randint(0, 2 ** 31 - E, (1,)))
        self.w_gate_up = nn.Parameter(torch.empty(El, 2 * F_, D))  # [El, 2F, D]
        self.w_down = nn.Parameter(torch.empty(El, D, F_))  # [El, D, F]
        with torch.no_grad():
            for j in range(El):
                g = torch.Generator(device=self.w_gate_up.device).manual_seed(base + self.e0 + j)
                self.w_gate_up[j].normal_(0.0, 0.02, generator=g)
                self.w_down[j].normal_(0.0, 0.02, generator=g)
        if ep is not None and ep.ep > 1:
            self.w_gate_up._vo_expert = True  # sharded over the EP group: the engine's expert parameter set
            self.w_down._vo_expert = True

    def attn_tp(self, x, cos, sin, tp):
        """Tensor + sequence parallel attention: ``x`` [B, S_l, D] holds this rank's tokens (rank r: positions
        [r S_l, (r+1) S_l)); q/k/v of this rank's heads come from one all-gather->GEMM over the whole
        sequence, the output projection's partial sums are reduce-scattered back to the token owners
        (``parallel/tensor_parallel.py``).  ``cos`` / ``sin`` cover the full sequence."""
        from verl_omni_b200.parallel.tensor_parallel import column_parallel_linear, row_parallel_linear

        cfg = self.cfg
        B, Sl, D = x.shape
        W, r = tp.world, tp.rank
        hd, Hq, Hk = cfg.head_dim, cfg.q_heads // W, cfg.kv_heads // W
        S = Sl * W
        h = rms_norm(x, self.ln1, cfg.eps).reshape(B * Sl, D)
        kvw = self.kv_proj.weight.view(2, cfg.kv_heads * hd, D)
        w = torch.cat([self.q_proj.weight[r * Hq * hd:(r + 1) * Hq * hd],
                       kvw[0, r * Hk * hd:(r + 1) * Hk * hd], kvw[1, r * Hk * hd:(r + 1) * Hk * hd]], 0)
        y = column_parallel_linear(h, w, None, tp)  # [W*B*Sl, (Hq + 2Hk) hd], rank-major rows
        y = y.view(W, B, Sl, -1).permute(1, 0, 2, 3).reshape(B, S, -1)
        v = y[..., (Hq + Hk) * hd:].view(B, S, Hk, hd).transpose(1, 2)
        # per-head q/k RMSNorm + RoPE straight from the projection output (one kernel each)
        q = LO.head_norm_rope(y, 0, Hq, self.q_norm, cos, sin, cfg.eps)
        k = LO.head_norm_rope(y, Hq * hd, Hk, self.k_norm, cos, sin, cfg.eps)
        rep = Hq // Hk
        o = attention(q.contiguous(), k.repeat_interleave(rep, 1).contiguous(),
                      v.repeat_interleave(rep, 1).contiguous(), causal=True)  # [B, S, Hq hd]
        o = o.view(B, W, Sl, -1).permute(1, 0, 2, 3).reshape(W * B * Sl, -1)
        wo = self.o_proj.weight[:, r * Hq * hd:(r + 1) * Hq * hd]
        return x + row_parallel_linear(o, wo, None, tp).view(B, Sl, D)

    def _tp_weights(self, tp):
        """This rank's slices of the attention weights (q / k / v rows of its heads, o_proj columns),
        contiguous copies kept until the weights change (their version counter, shared with the flat
        parameter buffer, moves on every optimizer step)."""
        cfg = self.cfg
        hd, W, r = cfg.head_dim, tp.world, tp.rank
        Hq, Hk = cfg.q_heads // W, cfg.kv_heads // W
        key = (W, r, self.q_proj.weight._version, self.kv_proj.weight._version, self.o_proj.weight._version,
               self.q_proj.weight.data_ptr())
        c = getattr(self, "_tp_w", None)
        if c is None or c[0] != key:
            kvw = self.kv_proj.weight.detach().view(2, cfg.kv_heads * hd, -1)
            qkv = torch.cat([self.q_proj.weight.detach()[r * Hq * hd:(r + 1) * Hq * hd],
                             kvw[0, r * Hk * hd:(r + 1) * Hk * hd], kvw[1, r * Hk * hd:(r + 1) * Hk * hd]], 0)
            wo = self.o_proj.weight.detach()[:, r * Hq * hd:(r + 1) * Hq * hd].contiguous()
            c = self._tp_w = (key, qkv, wo)
        return c[1], c[2]

    def attn_tp_decode(self, x, cos, sin, cache: KVCache, tp):
        """Tensor-parallel attention for the rollout (no autograd): every rank of the TP group holds the
        group's whole batch; rank r projects q / k / v for its ``q_heads / W`` and ``kv_heads / W`` heads, keeps
        only those KV heads in its cache and attends over them; the output projection's partial sums (its
        columns of ``o_proj``) are summed over the group by one all-reduce, so every rank continues with the
        same hidden states (vLLM's tensor-parallel attention)."""
        cfg = self.cfg
        B, S, D = x.shape
        hd, W = cfg.head_dim, tp.world
        Hq, Hk = cfg.q_heads // W, cfg.kv_heads // W
        wqkv, wo = self._tp_weights(tp)
        h = rms_norm(x, self.ln1, cfg.eps)
        y = L.linear(h, wqkv)  # [B, S, (Hq + 2 Hk) hd]
        q = LO.head_norm_rope(y, 0, Hq, self.q_norm, cos, sin, cfg.eps)
        k = LO.head_norm_rope(y, Hq * hd, Hk, self.k_norm, cos, sin, cfg.eps)
        v = y[..., (Hq + Hk) * hd:].reshape(B, S, Hk, hd).transpose(1, 2)
        first = cache.len == 0
        cache.append(k, v)
        if S == 1 and not first:
            o = decode_attention(q[:, :, 0], cache.k, cache.v, cache.lens()).reshape(B, 1, Hq * hd)
        else:
            if not first:
                k, v = cache.k[:, :, :cache.len], cache.v[:, :, :cache.len]
            rep = Hq // Hk
            o = attention(q.contiguous(), k.repeat_interleave(rep, 1).contiguous(),
                          v.repeat_interleave(rep, 1).contiguous(), causal=first and S > 1)
        part = L.linear(o.reshape(B, S, Hq * hd), wo)
        D_.all_reduce(part, group=tp.group)
        return x + part

    def attn(self, x, cos, sin, cache: Optional[dict], pos0: int, pos_t: Optional[torch.Tensor] = None):
        """``pos_t`` (int64 ``[1]`` on the device, one-token steps on a :class:`KVCache`): the position comes
        from the device, nothing is read on the host (a step that can be captured in a CUDA graph)."""
        cfg = self.cfg
        B, S, D = x.shape
        hd = cfg.head_dim
        h = rms_norm(x, self.ln1, cfg.eps)
        qp = self.q_proj(h)  # [B, S, Hq hd]
        kvp = self.kv_proj(h)  # [B, S, 2 Hk hd]: k heads, then v heads
        q = LO.head_norm_rope(qp, 0, cfg.q_heads, self.q_norm, cos, sin, cfg.eps)  # [B, Hq, S, hd]
        k = LO.head_norm_rope(kvp, 0, cfg.kv_heads, self.k_norm, cos, sin, cfg.eps)  # [B, Hk, S, hd]
        v = kvp[..., cfg.kv_heads * hd:].view(B, S, cfg.kv_heads, hd).transpose(1, 2)
        if pos_t is not None:
            if not isinstance(cache, KVCache) or S != 1:
                raise ValueError("device-position steps take one token against a contiguous KVCache")
            cache.append_at(k, v, pos_t)
            o = decode_attention(q[:, :, 0], cache.k, cache.v, cache.lens_at(pos_t))  # [B, Hq, hd]
            return x + self.o_proj(o.reshape(B, 1, cfg.q_heads * hd))
        if isinstance(cache, KVCache):
            # preallocated cache: in-place append; one-token steps use the grouped-query decode kernel
            first = cache.len == 0
            cache.append(k, v)
            if S == 1 and not first:
                o = decode_attention(q[:, :, 0], cache.k, cache.v, cache.lens())  # [B, Hq, hd]
                return x + self.o_proj(o.reshape(B, 1, cfg.q_heads * hd))
            if not first:
                k, v = cache.k[:, :, :cache.len], cache.v[:, :, :cache.len]
        elif isinstance(cache, PagedView):
            # paged cache (block pool + block table): same steps through the block-table decode kernel
            first = cache.len == 0
            cache.append(k, v)
            if S == 1 and not first:
                o = cache.decode(q[:, :, 0])
                return x + self.o_proj(o.reshape(B, 1, cfg.q_heads * hd))
            if not first:
                k, v = cache.contiguous()
        elif cache is not None:
            if "k" in cache:
                k = torch.cat([cache["k"], k], 2)
                v = torch.cat([cache["v"], v], 2)
            cache["k"], cache["v"] = k, v
        rep = cfg.q_heads // cfg.kv_heads
        kk = k.repeat_interleave(rep, 1).contiguous()
        vv = v.repeat_interleave(rep, 1).contiguous()
        causal = S > 1 and (cache is None or pos0 == 0)
        if S == 1 or (cache is not None and pos0 > 0):
            causal = False  # decode: the new token sees every cached key
        o = attention(q.contiguous(), kk, vv, causal=causal)
        return x + self.o_proj(o)

    def moe(self, x, ep=None):
        cfg = self.cfg
        B, S, D = x.shape
        h = rms_norm(x, self.ln2, cfg.eps).reshape(B * S, D)
        # softmax + top-k + renormalised gates on the device (one kernel, no host sync)
        gates, idx, probs = LO.router_topk(self.router(h).float(), cfg.top_k)
        gates = gates.to(x.dtype)
        self.last_router = (probs, idx)
        if (ep is not None and ep.ep > 1 and not torch.is_grad_enabled() and S == 1
                and getattr(ep, "decode_combine", None) is not None):
            # one-token decode steps: fixed-size gather / reduce-scatter, no host synchronisation per layer
            out = ep.decode_combine(h, idx, gates, self.w_gate_up, self.w_down, self.e0)
        elif ep is not None and hasattr(ep, "fused_ok") and ep.fused_ok(h, self.w_gate_up, self.w_down):
            out = ep.dispatch_combine_fused(h, idx, gates, self.w_gate_up, self.w_down)  # peer-memory exchange
        elif ep is not None:
            out = ep.dispatch_combine(h, idx, gates, self.expert_ffn)
        else:
            out = grouped_expert_ffn(h, idx, gates, self.w_gate_up, self.w_down)
        return x + out.view(B, S, D)

    def expert_ffn(self, tokens: torch.Tensor, expert_ids: torch.Tensor) -> torch.Tensor:
        """SwiGLU of locally-owned experts for tokens already grouped by (global) expert id."""
        return _ffn_grouped(tokens, expert_ids - self.e0, self.w_gate_up, self.w_down)

    def forward(self, x, cos, sin, cache=None, pos0: int = 0, ep=None, tp=None, pos_t=None, tp_decode=None):
        if tp_decode is not None:
            return self.moe(self.attn_tp_decode(x, cos, sin, cache, tp_decode), ep)
        if tp is not None:
            return self.moe(self.attn_tp(x, cos, sin, tp), ep)
        return self.moe(self.attn(x, cos, sin, cache, pos0, pos_t), ep)


def _ffn_grouped(tokens, expert_ids, w_gate_up, w_down):
    from verl_omni_b200.ops import moe as MO

    if MO.native_ok(tokens, w_gate_up, w_down):  # one grouped GEMM launch per projection, no host syncs
        ones = torch.ones(tokens.shape[0], 1, device=tokens.device, dtype=tokens.dtype)
        return MO.moe_ffn(tokens, expert_ids.reshape(-1, 1), ones, w_gate_up, w_down)
    out = torch.empty_like(tokens)
    for e in torch.unique(expert_ids).tolist():
        sel = (expert_ids == e).nonzero(as_tuple=True)[0]
        t = tokens.index_select(0, sel)
        gu = L.linear(t, w_gate_up[e].to(t.dtype))
        g, u = gu.chunk(2, -1)
        out.index_copy_(0, sel, L.linear(F.silu(g) * u, w_down[e].to(t.dtype)))
    return out


def grouped_expert_ffn(h, idx, gates, w_gate_up, w_down):
    """Top-k routed SwiGLU experts: sort (token, slot) pairs by expert, run each expert once, combine."""
    from verl_omni_b200.ops import moe as MO

    if MO.native_ok(h, w_gate_up, w_down):
        return MO.moe_ffn(h, idx, gates, w_gate_up, w_down)
    T, K = idx.shape
    flat_e = idx.reshape(-1)
    tok = torch.arange(T, device=h.device).repeat_interleave(K)
    order = torch.argsort(flat_e, stable=True)
    y = _ffn_grouped(h.index_select(0, tok[order]), flat_e[order], w_gate_up, w_down)
    w = gates.reshape(-1)[order].unsqueeze(-1)
    out = torch.zeros_like(h)
    out.index_add_(0, tok[order], (y * w).to(h.dtype))
    return out


class _Encoder(nn.Module):
    """Small pre-norm transformer encoder used for both the audio and the vision tower."""

    def __init__(self, in_dim: int, dim: int, layers: int, out_dim: int, heads: int = 4):
        super().__init__()
        self.inp = Linear(in_dim, dim)
        self.heads = heads
        self.blocks = nn.ModuleList()
        for _ in range(layers):
            b = nn.Module()
            b.ln1, b.ln2 = nn.Parameter(torch.ones(dim)), nn.Parameter(torch.ones(dim))
            b.qkv, b.o = Linear(dim, 3 * dim), Linear(dim, dim)
            b.fc1, b.fc2 = Linear(dim, 4 * dim), Linear(4 * dim, dim)
            self.blocks.append(b)
        self.proj = Linear(dim, out_dim)

    def forward(self, x):
        x = self.inp(x)
        B, S, D = x.shape
        H = self.heads
        for b in self.blocks:
            qkv = b.qkv(rms_norm(x, b.ln1, 1e-6)).view(B, S, 3, H, D // H).permute(2, 0, 3, 1, 4)
            x = x + b.o(attention(qkv[0].contiguous(), qkv[1].contiguous(), qkv[2].contiguous()))
            x = x + b.fc2(b.fc1(rms_norm(x, b.ln2, 1e-6), epilogue="gelu"))
        return self.proj(x)


class MoELLM(nn.Module):
    def __init__(self, cfg: MoEConfig, ep=None):
        """``ep``: an :class:`~verl_omni_b200.parallel.expert_parallel.ExpertParallel` context; its rank then
        holds only its own experts' weights (``experts / ep`` per layer)."""
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Parameter(torch.randn(cfg.vocab, cfg.hidden) * 0.02)
        self.layers = nn.ModuleList([MoEBlock(cfg, ep) for _ in range(cfg.layers)])
        self.norm = nn.Parameter(torch.ones(cfg.hidden))
        self.lm_head = Linear(cfg.hidden, cfg.vocab, bias=False)
        self.audio_tower = _Encoder(cfg.audio_mel, cfg.audio_dim, cfg.audio_layers, cfg.hidden)
        self.visual = _Encoder(cfg.vision_patch_dim, cfg.vision_dim, cfg.vision_layers, cfg.hidden)
        self.ep = ep
        self.tp = None  # TPContext: tensor + sequence parallel training forwards (no KV cache)
        self._rope_cache = None  # (cos, sin) fp32 [n, head_dim / 2] on the model's device, grown on demand

    def rope(self, pos0: int, S: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        """cos / sin rows for positions [pos0, pos0 + S) from a device-resident table (built once, grown
        to the next power of two when a longer position is asked for)."""
        need = pos0 + S
        c = self._rope_cache
        if c is None or c[0].shape[0] < need or c[0].device != torch.device(device):
            n = 1 << max(12, (need - 1).bit_length())
            cos, sin = rope_table(torch.arange(n), self.cfg.head_dim, self.cfg.rope_theta)
            c = self._rope_cache = (cos.to(device), sin.to(device))
        return c[0][pos0:need], c[1][pos0:need]

    def embed_tokens(self, ids, audio_feats=None, image_patches=None):
        x = F.embedding(ids, self.embed)
        for feats, tower, tok in ((audio_feats, self.audio_tower, self.cfg.audio_token),
                                  (image_patches, self.visual, self.cfg.image_token)):
            if feats is None:
                continue
            emb = tower(feats.to(x.dtype))  # [B, n, hidden]; each prompt holds n placeholder tokens
            mask = ids == tok
            mask = mask & (mask.cumsum(1) <= emb.shape[1])  # only the prompt's n placeholders
            x = x.masked_scatter(mask.unsqueeze(-1), emb.reshape(-1, x.shape[-1]).to(x.dtype))
        return x

    def forward(self, ids, positions=None, caches=None, pos0: int = 0, audio_feats=None, image_patches=None,
                return_hidden: bool = False, targets: Optional[torch.Tensor] = None, temperature: float = 1.0,
                pos_t: Optional[torch.Tensor] = None, tp_decode=None):
        """Logits [B, S, V] (fp32); ``return_hidden``: the final hidden states; ``targets`` [B, S] (next-token
        ids per position): log p(target) [B, S] through the chunked vocabulary kernel, with no logits tensor
        (under tensor parallelism each rank scores its own tokens and the log-probs are gathered).

        ``pos_t`` (int64 ``[1]`` on the device): a one-token decode step at that position against contiguous
        caches, with the RoPE rows and the KV write position taken on the device (``rope`` must already
        cover the position: the caller sizes the table before the step is captured)."""
        from verl_omni_b200.ops.vocab_logprob import token_logprobs_from_hidden

        cfg = self.cfg
        B, S = ids.shape
        if tp_decode is not None:
            # tensor-parallel rollout: heads split over the group, KV caches of this rank's heads only
            if caches is None:
                raise ValueError("tensor-parallel decode runs against KV caches")
            x = self.embed_tokens(ids, audio_feats, image_patches) if pos0 == 0 else F.embedding(ids, self.embed)
            cos, sin = self.rope(pos0, S, ids.device)
            for i, blk in enumerate(self.layers):
                x = blk(x, cos, sin, caches[i], pos0, self.ep, tp_decode=tp_decode)
            h = rms_norm(x, self.norm, cfg.eps)
            return h if return_hidden else self.lm_head(h).float()
        if pos_t is not None:
            if caches is None or S != 1 or self._rope_cache is None:
                raise ValueError("device-position steps need caches, one token and a sized RoPE table")
            x = F.embedding(ids, self.embed)
            cos, sin = self._rope_cache[0].index_select(0, pos_t), self._rope_cache[1].index_select(0, pos_t)
            for i, blk in enumerate(self.layers):
                x = blk(x, cos, sin, caches[i], 0, self.ep, pos_t=pos_t)
            h = rms_norm(x, self.norm, cfg.eps)
            return h if return_hidden else self.lm_head(h).float()
        x = self.embed_tokens(ids, audio_feats, image_patches) if pos0 == 0 else F.embedding(ids, self.embed)
        cos, sin = self.rope(pos0, S, ids.device)
        tp = self.tp if (self.tp is not None and caches is None and pos0 == 0 and self.tp.world > 1) else None
        if tp is not None:
            from verl_omni_b200.parallel.ulysses import gather_sequence

            W = tp.world
            pad = (-S) % W  # causal: zero tokens appended at the end change no earlier position
            if pad:
                x = torch.cat([x, x.new_zeros(B, pad, x.shape[-1])], 1)
                cos, sin = self.rope(0, S + pad, ids.device)
            Sl = x.shape[1] // W
            x = x[:, tp.rank * Sl:(tp.rank + 1) * Sl]
            for blk in self.layers:
                x = blk(x, cos, sin, None, 0, self.ep, tp)
            h = rms_norm(x, self.norm, cfg.eps)
            if targets is not None:
                tl = F.pad(targets, (0, pad))[:, tp.rank * Sl:(tp.rank + 1) * Sl]
                lp = token_logprobs_from_hidden(h, self.lm_head.weight, tl, temperature)
                return gather_sequence(lp.unsqueeze(-1), tp.group)[:, :S, 0]
            if return_hidden:
                return gather_sequence(h, tp.group)[:, :S]
            # the vocabulary projection stays partitioned by tokens; the logits are gathered
            return gather_sequence(self.lm_head(h).float(), tp.group)[:, :S]
        for i, blk in enumerate(self.layers):
            x = blk(x, cos, sin, None if caches is None else caches[i], pos0, self.ep)
        h = rms_norm(x, self.norm, cfg.eps)
        if targets is not None:
            return token_logprobs_from_hidden(h, self.lm_head.weight, targets, temperature)
        if return_hidden:
            return h
        return self.lm_head(h).float()


class MoEStage(nn.Module):
    """One pipeline stage of a :class:`MoELLM`: layers ``[lo, hi)``; the first stage also holds the token
    embedding and the audio / vision towers, the last the final norm and the vocabulary head.

    Built from a whole model (the stages then hold exactly the parameters of the unsplit model, initialised
    from the same generator state) whose other parts are dropped.  Counterpart of Megatron's
    ``pipeline_model_parallel_size`` layer split used by the reference's omni Megatron trainer
    (``trainer/config/_generated_omni_megatron_trainer.yaml:34-67``)."""

    def __init__(self, full: MoELLM, lo: int, hi: int, first: bool, last: bool):
        super().__init__()
        self.cfg, self.lo, self.hi, self.first, self.last = full.cfg, int(lo), int(hi), bool(first), bool(last)
        self.layers = nn.ModuleList(list(full.layers[lo:hi]))
        if first:
            self.embed, self.audio_tower, self.visual = full.embed, full.audio_tower, full.visual
        if last:
            self.norm, self.lm_head = full.norm, full.lm_head
        self.ep, self.tp, self._rope_cache = full.ep, None, None

    rope = MoELLM.rope
    embed_tokens = MoELLM.embed_tokens

    def forward(self, x, pos0: int = 0, caches=None, audio_feats=None, image_patches=None,
                targets: Optional[torch.Tensor] = None, temperature: float = 1.0, last_only: bool = False):
        """``x``: token ids ``[B, S]`` on the first stage, the previous stage's hidden states ``[B, S, D]``
        otherwise.  Returns the hidden states on every stage but the last; there: log p(``targets``) when
        given, else fp32 logits (of the last position only with ``last_only``)."""
        from verl_omni_b200.ops.vocab_logprob import token_logprobs_from_hidden

        cfg = self.cfg
        if self.first:
            ids = x
            x = self.embed_tokens(ids, audio_feats, image_patches) if pos0 == 0 else F.embedding(ids, self.embed)
        cos, sin = self.rope(pos0, x.shape[1], x.device)
        for i, blk in enumerate(self.layers):
            x = blk(x, cos, sin, None if caches is None else caches[i], pos0, self.ep)
        if not self.last:
            return x
        h = rms_norm(x, self.norm, cfg.eps)
        if targets is not None:
            return token_logprobs_from_hidden(h, self.lm_head.weight, targets, temperature)
        if last_only:
            h = h[:, -1:].contiguous()
        return self.lm_head(h).float()


def token_logprobs(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    """log p(target) per position: logits [B, S, V] (fp32), targets [B, S]."""
    lp = torch.log_softmax(logits / temperature, -1)
    return lp.gather(-1, targets.unsqueeze(-1)).squeeze(-1)
