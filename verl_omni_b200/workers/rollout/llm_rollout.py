"""Autoregressive rollout for the omni thinker (the vLLM-Omni AR mode of the reference,
``verl_omni/workers/rollout/vllm_rollout/vllm_omni_async_server.py:537-579``).

Batched prefill of the (multimodal) prompts, then token-by-token decode against preallocated per-layer KV
caches (grouped-query decode kernel); sampling with temperature / top-k / top-p on the device from a
seeded generator; returns the response ids, their log-probs under the sampling distribution
(``rollout_log_probs``) and an EOS-aware response mask.
"""

from __future__ import annotations

from typing import Optional

import torch

from verl_omni_b200.models.moe_llm import MoELLM
from verl_omni_b200.ops.decode import KVCache, PagedKVCache, sample_tokens
from verl_omni_b200.utils.dataproto import DataProto


def sample_next(logits: torch.Tensor, temperature: float, top_k: int, top_p: float, generator) -> torch.Tensor:
    if temperature <= 0:
        return logits.argmax(-1)
    l = logits / temperature
    if top_k and top_k > 0:
        kth = torch.topk(l, min(top_k, l.shape[-1]), dim=-1).values[..., -1:]
        l = l.masked_fill(l < kth, float("-inf"))
    if top_p < 1.0:
        sl, si = torch.sort(l, descending=True, dim=-1)
        cp = torch.softmax(sl, -1).cumsum(-1)
        drop = cp - torch.softmax(sl, -1) > top_p
        sl = sl.masked_fill(drop, float("-inf"))
        l = torch.full_like(l, float("-inf")).scatter(-1, si, sl)
    probs = torch.softmax(l.float(), -1)
    return torch.multinomial(probs.cpu(), 1, generator=generator).squeeze(-1).to(logits.device)


class LLMRolloutEngine:
    def __init__(self, module: MoELLM, *, max_new_tokens: int = 256, temperature: float = 1.0, top_k: int = 0,
                 top_p: float = 1.0, eos_id: Optional[int] = None, device=None, kv_block_size: int = 0):
        self.module = module
        self.kv_block_size = kv_block_size  # > 0: paged KV cache with blocks of this many positions
        self.max_new_tokens = max_new_tokens
        self.temperature, self.top_k, self.top_p = temperature, top_k, top_p
        self.eos_id = eos_id
        self.device = device

    @torch.no_grad()
    def generate(self, batch: DataProto, seed: int = 0) -> DataProto:
        ids = batch.batch["input_ids"].to(self.device)
        B, P = ids.shape
        dev = ids.device
        g = torch.Generator(device=dev).manual_seed(int(seed))  # sampling stays on the device
        cfg = self.module.cfg
        if self.kv_block_size > 0:
            bs = self.kv_block_size
            per_seq = -(-(P + self.max_new_tokens) // bs)
            caches = []
            for _ in self.module.layers:
                pool = PagedKVCache(B * per_seq, cfg.kv_heads, bs, cfg.head_dim, dev, self.module.embed.dtype,
                                    max_blocks_per_seq=per_seq)
                caches.append(pool.view([pool.add_sequence() for _ in range(B)]))
        else:
            caches = [KVCache(B, cfg.kv_heads, P + self.max_new_tokens, cfg.head_dim, dev, self.module.embed.dtype)
                      for _ in self.module.layers]
        # prefill: the vocabulary projection of the last prompt position only
        af, ip = batch.batch.get("audio_feats"), batch.batch.get("image_patches")
        h = self.module(ids, caches=caches, pos0=0, audio_feats=af.to(dev) if af is not None else None,
                        image_patches=ip.to(dev) if ip is not None else None, return_hidden=True)
        logits = self.module.lm_head(h[:, -1:].contiguous()).float()[:, -1]
        out_ids, out_lp = [], []
        done = torch.zeros(B, dtype=torch.bool, device=ids.device)
        mask = []
        for t in range(self.max_new_tokens):
            nxt, lp = sample_tokens(logits, self.temperature, self.top_k, self.top_p, g)
            if self.temperature <= 0:
                lp = torch.log_softmax(logits.float(), -1).gather(-1, nxt[:, None]).squeeze(-1)
            out_ids.append(nxt)
            out_lp.append(lp)
            mask.append(~done)
            if self.eos_id is not None:
                done = done | (nxt == self.eos_id)
            if t + 1 < self.max_new_tokens:
                logits = self.module(nxt[:, None], caches=caches, pos0=P + t)[:, -1]
        resp = torch.stack(out_ids, 1)
        out = DataProto({"prompts": ids, "responses": resp, "rollout_log_probs": torch.stack(out_lp, 1),
                         "response_mask": torch.stack(mask, 1).float(),
                         "input_ids": torch.cat([ids, resp], 1)}, dict(batch.non_tensor_batch))
        for k in ("audio_feats", "image_patches"):
            if k in batch.batch:
                out.batch[k] = batch.batch[k]
        return out
