"""Autoregressive decode helpers: preallocated KV cache, grouped-query decode attention, device sampling.

* :class:`KVCache` -- one ``[B, Hk, Lmax, hd]`` K and V buffer per layer written in place (no per-token
  concatenation), with per-sequence lengths;
* :func:`decode_attention` -- one new query token per sequence against the cache (``csrc/decode_attn.cu``:
  each CTA reads a (sequence, KV head) slice of the cache once for all query heads of its group,
  flash-decoding splits for long caches); fp32 torch oracle on CPU;
* :func:`sample_tokens` -- temperature / top-k / top-p sampling and the sampled tokens' log-probs on the
  device (Gumbel-max over the filtered logits with a seeded device generator): no host round trip per token.

Counterpart of vLLM's paged decode attention and sampler used by the reference's AR rollout
(``verl_omni/workers/rollout/vllm_rollout/vllm_omni_async_server.py:537-579,640-671``).
"""

from __future__ import annotations

import math
from typing import Optional

import torch


def _ext():
    from verl_omni_b200.ops._ext import ext

    return ext()


class KVCache:
    """Per-layer K / V buffers ``[B, Hk, Lmax, hd]`` and the number of valid positions (same for every row)."""

    def __init__(self, batch: int, kv_heads: int, max_len: int, head_dim: int, device, dtype=torch.bfloat16):
        self.k = torch.zeros(batch, kv_heads, max_len, head_dim, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.len = 0
        self.max_len = max_len

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """k / v [B, Hk, S, hd] for positions [len, len + S)."""
        S = k.shape[2]
        if self.len + S > self.max_len:
            raise ValueError(f"KV cache full ({self.len} + {S} > {self.max_len})")
        self.k[:, :, self.len:self.len + S].copy_(k)
        self.v[:, :, self.len:self.len + S].copy_(v)
        self.len += S

    def lens(self) -> torch.Tensor:
        return torch.full((self.k.shape[0],), self.len, dtype=torch.int32, device=self.k.device)


def decode_attention_reference(q, k_cache, v_cache, lens, scale: float) -> torch.Tensor:
    """q [B, Hq, hd]; caches [B, Hk, Lmax, hd]; lens [B] -> [B, Hq, hd] (fp32 math)."""
    B, Hq, hd = q.shape
    Hk = k_cache.shape[1]
    rep = Hq // Hk
    out = torch.empty(B, Hq, hd, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(lens[b])
        k = k_cache[b, :, :L].float().repeat_interleave(rep, 0)  # [Hq, L, hd]
        v = v_cache[b, :, :L].float().repeat_interleave(rep, 0)
        s = torch.einsum("hd,hld->hl", q[b].float(), k) * scale
        out[b] = torch.einsum("hl,hld->hd", torch.softmax(s, -1), v)
    return out.to(q.dtype)


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
                     scale: Optional[float] = None, splits: int = 0) -> torch.Tensor:
    hd = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    rep = q.shape[1] // k_cache.shape[1]
    if not q.is_cuda or hd not in (64, 128) or rep not in (1, 2, 4, 8) or q.dtype != torch.bfloat16:
        return decode_attention_reference(q, k_cache, v_cache, lens, scale)
    if splits <= 0:  # enough CTAs to cover the SMs a few times over
        n = q.shape[0] * k_cache.shape[1]
        splits = max(1, min(16, (4 * torch.cuda.get_device_properties(q.device).multi_processor_count) // max(n, 1)))
        splits = min(splits, max(1, int(k_cache.shape[2]) // 256))
    return _ext().decode_attention(q.contiguous(), k_cache, v_cache, lens.to(torch.int32).contiguous(), float(scale),
                                   int(splits))


def sample_tokens(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                  generator: Optional[torch.Generator]) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (token ids [B], log-probs of the sampled tokens under the temperature-scaled distribution)."""
    lf = logits.float()
    if temperature <= 0:
        ids = lf.argmax(-1)
        return ids, torch.zeros_like(ids, dtype=torch.float32)
    l = lf / temperature
    logp_full = torch.log_softmax(l, -1)
    if top_k and top_k > 0:
        kth = torch.topk(l, min(top_k, l.shape[-1]), dim=-1).values[..., -1:]
        l = l.masked_fill(l < kth, float("-inf"))
    if top_p < 1.0:
        sl, si = torch.sort(l, descending=True, dim=-1)
        p = torch.softmax(sl, -1)
        drop = (p.cumsum(-1) - p) > top_p
        sl = sl.masked_fill(drop, float("-inf"))
        l = torch.full_like(l, float("-inf")).scatter(-1, si, sl)
    u = torch.rand(l.shape, device=l.device, generator=generator).clamp_(1e-20, 1.0)
    ids = (l - torch.log(-torch.log(u))).argmax(-1)  # Gumbel-max: a draw from softmax(l)
    return ids, logp_full.gather(-1, ids[:, None]).squeeze(-1)
