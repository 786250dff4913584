"""Autoregressive rollout for the omni thinker (the vLLM-Omni AR mode of the reference,
``verl_omni/workers/rollout/vllm_rollout/vllm_omni_async_server.py:537-579``).

Batched prefill of the (multimodal) prompts, then token-by-token decode against preallocated per-layer KV
caches (grouped-query decode kernel); sampling with temperature / top-k / top-p on the device from a
seeded generator; returns the response ids, their log-probs under the sampling distribution
(``rollout_log_probs``) and an EOS-aware response mask.
"""

from __future__ import annotations

import os
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


def _graph_ok(module: MoELLM, caches, dev) -> bool:
    """CUDA-graph decode applies to contiguous caches on a GPU.  With experts sharded over ranks the step holds
    collectives; those are captured only on request (``VO_DECODE_GRAPH_EP=1``), since every rank of the group
    must then replay in step."""
    if os.environ.get("VO_DECODE_GRAPH", "1") == "0" or torch.device(dev).type != "cuda":
        return False
    if not all(isinstance(c, KVCache) for c in caches):
        return False
    ep = getattr(module, "ep", None)
    if ep is not None and getattr(ep, "ep", 1) > 1 and os.environ.get("VO_DECODE_GRAPH_EP", "0") != "1":
        return False
    return True


class _DecodeStep:
    """The one-token decode step of the thinker (embedding, every layer's attention against the KV cache and
    experts, final norm, vocabulary projection) as one CUDA graph.

    A decode step is launch-bound: each layer issues a few dozen small kernels whose launch cost exceeds their
    run time at rollout batch sizes.  The step reads its token ids and its position from two static device
    tensors (``MoELLM.forward(pos_t=...)``: KV write position, RoPE rows and key lengths all come from the
    device), so one capture replays at every position.  The first step runs eagerly (it sets up the lazily
    built kernel state and the allocator's blocks), the second is captured and replayed, later steps replay.
    Sampling stays outside the graph (it draws from the caller's generator).  The extension's launch counter
    is advanced by the captured count on every replay."""

    def __init__(self, module: MoELLM, caches, batch: int, dev):
        self.module, self.caches = module, caches
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.graph, self.out, self.calls, self.launches = None, None, 0, 0

    def _run(self):
        return self.module(self.ids, caches=self.caches, pos_t=self.pos)[:, -1]

    def __call__(self, nxt: torch.Tensor, pos: int) -> torch.Tensor:
        from verl_omni_b200.ops._ext import ext

        self.ids.copy_(nxt.view(-1, 1))
        self.pos.fill_(pos)
        self.calls += 1
        if self.graph is None and self.calls == 1:
            out = self._run()
        elif self.graph is None:
            e = ext()
            n0 = e.launch_count()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.out = self._run()
            self.launches = e.launch_count() - n0  # counted at capture, which ran nothing: this replay's count
            self.graph.replay()
            out = self.out
        else:
            self.graph.replay()
            ext().count_launches(self.launches)
            out = self.out
        for c in self.caches:
            c.len = pos + 1
        return out


class LLMRolloutEngine:
    def __init__(self, module: MoELLM, *, max_new_tokens: int = 256, temperature: float = 1.0, top_k: int = 0,
                 top_p: float = 1.0, eos_id: Optional[int] = None, device=None, kv_block_size: int = 0,
                 pp=None, tp=None):
        """``pp``: a :class:`~verl_omni_b200.parallel.pipeline.PipeLink` when ``module`` is one pipeline stage
        (:class:`~verl_omni_b200.models.moe_llm.MoEStage`): every step's hidden states travel down the stages
        and the last stage's sampled tokens are broadcast back."""
        self.module = module
        self.pp = pp
        # ``tp``: a TPContext -- tensor-parallel decode (vLLM's rollout tensor_model_parallel_size): the ranks of
        # the group decode their prompts together, heads (and KV caches) split over the group
        self.tp = tp if tp is not None and tp.world > 1 else None
        self.kv_block_size = kv_block_size  # > 0: paged KV cache with blocks of this many positions
        self.max_new_tokens = max_new_tokens
        self.temperature, self.top_k, self.top_p = temperature, top_k, top_p
        self.eos_id = eos_id
        self.device = device

    @torch.no_grad()
    def generate(self, batch: DataProto, seed: int = 0) -> DataProto:
        if self.pp is not None:
            return self._generate_pp(batch, seed)
        tp = self.tp
        ids = batch.batch["input_ids"].to(self.device)
        af, ip = batch.batch.get("audio_feats"), batch.batch.get("image_patches")
        af = af.to(ids.device) if af is not None else None
        ip = ip.to(ids.device) if ip is not None else None
        B_own = ids.shape[0]
        if tp is not None:
            # the group's prompts in group-rank order; every rank decodes all of them (same seed on every rank,
            # identical logits after the all-reduces, so the same draws) and keeps its own rows at the end
            ids, af, ip = (self._gather(t, tp) if t is not None else None for t in (ids, af, ip))
        B, P = ids.shape
        dev = ids.device
        g = torch.Generator(device=dev).manual_seed(int(seed))  # sampling stays on the device
        cfg = self.module.cfg
        if tp is not None:
            caches = [KVCache(B, cfg.kv_heads // tp.world, P + self.max_new_tokens, cfg.head_dim, dev,
                              self.module.embed.dtype) for _ in self.module.layers]
        elif self.kv_block_size > 0:
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
        h = self.module(ids, caches=caches, pos0=0, audio_feats=af, image_patches=ip, return_hidden=True,
                        **({"tp_decode": tp} if tp is not None else {}))
        logits = self.module.lm_head(h[:, -1:].contiguous()).float()[:, -1]
        out_ids, out_lp = [], []
        done = torch.zeros(B, dtype=torch.bool, device=ids.device)
        mask = []
        step = None
        if self.max_new_tokens > 1 and tp is None and _graph_ok(self.module, caches, dev):
            self.module.rope(0, P + self.max_new_tokens, dev)  # the table covers every decode position
            step = _DecodeStep(self.module, caches, B, dev)
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
                if step is not None:
                    logits = step(nxt, P + t)
                elif tp is not None:
                    logits = self.module(nxt[:, None], caches=caches, pos0=P + t, tp_decode=tp)[:, -1]
                else:
                    logits = self.module(nxt[:, None], caches=caches, pos0=P + t)[:, -1]
        lp = torch.stack(out_lp, 1)
        if tp is not None:
            own = slice(tp.rank * B_own, (tp.rank + 1) * B_own)
            ids, lp = ids[own], lp[own]
            out_ids, mask = [t[own] for t in out_ids], [t[own] for t in mask]
        return self._pack(batch, ids, out_ids, lp, mask)

    @staticmethod
    def _gather(t: torch.Tensor, tp) -> torch.Tensor:
        from verl_omni_b200.parallel import dist as D

        t = t.contiguous()
        out = torch.empty((tp.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        D.all_gather_into(out, t, tp.group)
        return out

    @staticmethod
    def _pack(batch: DataProto, ids, out_ids, lp, mask) -> DataProto:
        resp = torch.stack(out_ids, 1)
        out = DataProto({"prompts": ids, "responses": resp, "rollout_log_probs": lp,
                         "response_mask": torch.stack(mask, 1).float(),
                         "input_ids": torch.cat([ids, resp], 1)}, dict(batch.non_tensor_batch))
        for k in ("audio_feats", "image_patches"):
            if k in batch.batch:
                out.batch[k] = batch.batch[k]
        return out

    def _generate_pp(self, batch: DataProto, seed: int) -> DataProto:
        """Pipelined decode: prefill and every token step run stage after stage (hidden states sent to the
        next stage), the last stage samples with the seeded generator and broadcasts the token ids, so every
        stage writes its own layers' KV caches and ends with the same responses; the sampled log-probs are
        broadcast once at the end.  Same tokens as the unsplit model given the same seed."""
        link, m = self.pp, self.module
        ids = batch.batch["input_ids"].to(self.device)
        B, P = ids.shape
        dev = ids.device
        cfg = m.cfg
        dt = next(m.layers[0].parameters()).dtype if len(m.layers) else torch.float32
        caches = [KVCache(B, cfg.kv_heads, P + self.max_new_tokens, cfg.head_dim, dev, dt) for _ in m.layers]
        g = torch.Generator(device=dev).manual_seed(int(seed)) if link.last else None
        af, ip = batch.batch.get("audio_feats"), batch.batch.get("image_patches")
        af = af.to(dev) if af is not None and link.first else None
        ip = ip.to(dev) if ip is not None and link.first else None

        def run(tok, pos0):
            x = tok if link.first else link.recv_prev((B, tok.shape[1], cfg.hidden), dt)
            y = m(x, pos0=pos0, caches=caches, audio_feats=af if pos0 == 0 else None,
                  image_patches=ip if pos0 == 0 else None, last_only=True)
            if not link.last:
                link.send_next(y)
                return None
            return y[:, -1]

        logits = run(ids, 0)
        out_ids, out_lp, mask = [], [], []
        done = torch.zeros(B, dtype=torch.bool, device=dev)
        for t in range(self.max_new_tokens):
            if link.last:
                nxt, lp = sample_tokens(logits, self.temperature, self.top_k, self.top_p, g)
                if self.temperature <= 0:
                    lp = torch.log_softmax(logits.float(), -1).gather(-1, nxt[:, None]).squeeze(-1)
                out_lp.append(lp)
            else:
                nxt = torch.zeros(B, dtype=torch.long, device=dev)
            nxt = link.bcast_last(nxt)
            out_ids.append(nxt)
            mask.append(~done)
            if self.eos_id is not None:
                done = done | (nxt == self.eos_id)
            if t + 1 < self.max_new_tokens:
                logits = run(nxt[:, None], P + t)
        lp = torch.stack(out_lp, 1) if link.last else torch.zeros(B, self.max_new_tokens, device=dev)
        return self._pack(batch, ids, out_ids, link.bcast_last(lp.float()), mask)
