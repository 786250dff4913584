"""Qwen-Image Dual-GRPO: the text encoder samples a response, the DiT images the prompt + response, and one
group advantage trains both policies (reference
``verl_omni/pipelines/qwen_image_dual_grpo/vllm_omni_rollout_adapter.py:56-340``).

Rollout, per prompt row:
1. the causal text-encoder LM (Qwen2.5-VL-shaped; its hidden states are Qwen-Image's 3584-d prompt
   embeddings) samples ``max_new_tokens`` response tokens with their log-probs;
2. the final hidden states of ``[prompt ; response]`` become the DiT's ``prompt_embeds`` (with a mask over
   the valid tokens), and the DiT rollout records the SDE trajectory and its log-probs.
Training (:func:`dual_grpo_loss`): the PPO-clip objective on the DiT step log-ratios plus, weighted by
``llm_coef``, the token-level PPO-clip objective on the text-encoder log-ratios, both with the sample's
group-normalised advantage.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from verl_omni_b200.models.layers import Linear
from verl_omni_b200.models.scorers import Tower
from verl_omni_b200.utils.dataproto import DataProto


class TextEncoderLM(nn.Module):
    """Causal transformer LM whose final hidden states are the diffusion prompt embeddings
    (Qwen2.5-VL-7B shape: hidden 3584, 28 layers, 28 heads, vocab 152064)."""

    def __init__(self, vocab: int = 152064, dim: int = 3584, depth: int = 28, heads: int = 28, max_len: int = 1024):
        super().__init__()
        self.vocab, self.dim = vocab, dim
        self.embed = nn.Embedding(vocab, dim)
        self.pos = nn.Parameter(torch.randn(max_len, dim) * 0.02)
        self.body = Tower(dim, depth, heads, causal=True)
        self.lm_head = Linear(dim, vocab, bias=False)

    def hidden(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.embed(ids).to(self.pos.dtype) + self.pos[:ids.shape[1]][None]
        return self.body(x)

    def token_logprobs(self, ids: torch.Tensor, P: int, temperature: float = 1.0) -> torch.Tensor:
        """log p(ids[:, t] | ids[:, :t]) for the response positions t >= P -> [B, S - P] fp32."""
        from verl_omni_b200.ops.vocab_logprob import token_logprobs_from_hidden

        h = self.hidden(ids[:, :-1])
        return token_logprobs_from_hidden(h[:, P - 1:], self.lm_head.weight, ids[:, P:], temperature)

    @torch.no_grad()
    def sample(self, ids: torch.Tensor, max_new_tokens: int, temperature: float, generator) -> tuple:
        """Ancestral sampling (full recompute per token: the responses are short); returns (response ids
        [B, n], their log-probs [B, n])."""
        out, lps = [], []
        cur = ids
        for _ in range(max_new_tokens):
            logits = self.lm_head(self.hidden(cur)[:, -1:].contiguous()).float()[:, -1] / max(temperature, 1e-6)
            logp = torch.log_softmax(logits, -1)
            nxt = torch.multinomial(logp.exp(), 1, generator=generator)[:, 0]
            out.append(nxt)
            lps.append(logp.gather(1, nxt[:, None])[:, 0])
            cur = torch.cat([cur, nxt[:, None]], 1)
        return torch.stack(out, 1), torch.stack(lps, 1)


class DualGRPORollout:
    def __init__(self, text_lm: TextEncoderLM, dit_rollout, *, max_new_tokens: int = 32, temperature: float = 1.0):
        self.lm, self.dit = text_lm, dit_rollout
        self.max_new_tokens, self.temperature = max_new_tokens, temperature

    @torch.no_grad()
    def generate(self, prompt_ids: torch.Tensor, *, seed: int = 0, row_seeds: Optional[torch.Tensor] = None) -> DataProto:
        dev = next(self.lm.parameters()).device
        ids = prompt_ids.to(dev)
        g = torch.Generator(device=dev).manual_seed(int(seed))
        resp, lps = self.lm.sample(ids, self.max_new_tokens, self.temperature, g)
        full = torch.cat([ids, resp], 1)
        emb = self.lm.hidden(full)  # [B, P + n, dim]: the DiT's prompt embeddings
        cond = DataProto({"prompt_embeds": emb, "prompt_embeds_mask": torch.ones(emb.shape[:2], device=dev)})
        out = self.dit.generate(cond, seed=seed, row_seeds=row_seeds, decode=self.dit.decoder is not None)
        out.batch.update({"llm_input_ids": full, "llm_response_ids": resp, "llm_log_probs": lps})
        out.meta_info["llm_prompt_len"] = int(ids.shape[1])
        return out


def dual_grpo_loss(dit_logp: torch.Tensor, dit_old: torch.Tensor, llm_logp: torch.Tensor, llm_old: torch.Tensor,
                   advantages: torch.Tensor, *, clip: float = 1e-4, llm_clip: float = 0.2, llm_coef: float = 1.0,
                   llm_mask: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, dict]:
    """PPO-clip on one DiT step's log-ratio [B] + ``llm_coef`` x token-mean PPO-clip on the text-encoder
    tokens [B, n]; ``advantages`` [B] shared by both."""
    a = advantages.detach()
    r = torch.exp(dit_logp - dit_old)
    dit = torch.maximum(-a * r, -a * torch.clamp(r, 1 - clip, 1 + clip)).mean()
    rl = torch.exp(llm_logp - llm_old)
    tok = torch.maximum(-a[:, None] * rl, -a[:, None] * torch.clamp(rl, 1 - llm_clip, 1 + llm_clip))
    m = torch.ones_like(tok) if llm_mask is None else llm_mask.to(tok.dtype)
    llm = (tok * m).sum() / m.sum().clamp_min(1)
    with torch.no_grad():
        metrics = {"actor/dit_pg_loss": dit.detach(), "actor/llm_pg_loss": llm.detach(),
                   "actor/llm_ratio_mean": ((rl * m).sum() / m.sum().clamp_min(1)).detach()}
    return dit + llm_coef * llm, metrics
