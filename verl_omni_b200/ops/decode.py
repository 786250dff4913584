"""Autoregressive decode helpers: preallocated KV cache, grouped-query decode attention, device sampling.

* :class:`KVCache` -- one ``[B, Hk, Lmax, hd]`` K and V buffer per layer written in place (no per-token
  concatenation), with per-sequence lengths;
* :class:`PagedKVCache` -- a pool of fixed-size blocks ``[blocks, Hk, block, hd]`` shared by sequences of
  different lengths, a free list and one block table per sequence (vLLM's paged layout): sequences that
  finish return their blocks at once, memory follows the tokens actually cached;
* :func:`decode_attention` -- one new query token per sequence against the cache: at head_dim 128 a tcgen05
  kernel (``csrc/decode_attn_sm100.cu``: TMA-staged 128-key tiles, S^T = K Q^T and O^T = V^T P^T on the
  tensor cores with the query heads of a KV group as N), else the CUDA-core kernel (``csrc/decode_attn.cu``);
  each CTA reads a (sequence, KV head) slice of the cache once for all query heads of its group,
  flash-decoding splits for long caches; fp32 torch oracle on CPU;
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

    def append_at(self, k: torch.Tensor, v: torch.Tensor, pos_t: torch.Tensor) -> None:
        """One-token step written at the position held on the device (``pos_t`` int64 ``[1]``): k / v
        ``[B, Hk, 1, hd]``.  Neither the host counter nor any host value is read, so the step can be captured
        in a CUDA graph once and replayed at every later position; the caller keeps ``len`` in step and keeps
        the position below ``max_len``."""
        self.k.index_copy_(2, pos_t, k)
        self.v.index_copy_(2, pos_t, v)

    def lens_at(self, pos_t: torch.Tensor) -> torch.Tensor:
        """Valid rows after a step at ``pos_t``: ``pos_t + 1`` for every sequence, int32 ``[B]`` (device)."""
        return (pos_t + 1).to(torch.int32).expand(self.k.shape[0]).contiguous()


class PagedKVCache:
    """Paged K / V storage of one layer: pools ``[num_blocks, Hk, block_size, hd]``, a host-side free list and
    per-sequence block lists (the block manager runs on the host, as vLLM's does; the kernels only read the
    block table)."""

    def __init__(self, num_blocks: int, kv_heads: int, block_size: int, head_dim: int, device,
                 dtype=torch.bfloat16, max_blocks_per_seq: Optional[int] = None):
        self.k = torch.zeros(num_blocks, kv_heads, block_size, head_dim, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.block = block_size
        self.max_blocks = max_blocks_per_seq or num_blocks
        self.free: list[int] = list(range(num_blocks - 1, -1, -1))
        self.blocks: dict[int, list[int]] = {}
        self.length: dict[int, int] = {}
        self._next = 0

    def add_sequence(self) -> int:
        sid = self._next
        self._next += 1
        self.blocks[sid], self.length[sid] = [], 0
        return sid

    def free_sequence(self, sid: int) -> None:
        self.free.extend(reversed(self.blocks.pop(sid)))
        del self.length[sid]

    def _reserve(self, sid: int, n: int) -> None:
        need = -(-(self.length[sid] + n) // self.block) - len(self.blocks[sid])
        if need > len(self.free) or len(self.blocks[sid]) + need > self.max_blocks:
            raise RuntimeError(f"paged KV cache out of blocks (sequence {sid} needs {need} more)")
        for _ in range(need):
            self.blocks[sid].append(self.free.pop())

    def append(self, sids: list[int], k: torch.Tensor, v: torch.Tensor) -> None:
        """k / v ``[len(sids), Hk, S, hd]``: the next S positions of each listed sequence."""
        S = k.shape[2]
        blk, off = [], []
        for sid in sids:
            self._reserve(sid, S)
            L, bl = self.length[sid], self.blocks[sid]
            for t in range(L, L + S):
                blk.append(bl[t // self.block])
                off.append(t % self.block)
            self.length[sid] = L + S
        bi = torch.tensor(blk, device=self.k.device)
        oi = torch.tensor(off, device=self.k.device)
        Hk, hd = k.shape[1], k.shape[3]
        self.k[bi, :, oi] = k.permute(0, 2, 1, 3).reshape(-1, Hk, hd).to(self.k.dtype)
        self.v[bi, :, oi] = v.permute(0, 2, 1, 3).reshape(-1, Hk, hd).to(self.v.dtype)

    def view(self, sids: list[int]) -> "PagedView":
        return PagedView(self, list(sids))

    def block_table(self, sids: list[int]) -> torch.Tensor:
        width = max(1, max(len(self.blocks[s]) for s in sids))
        t = torch.zeros(len(sids), width, dtype=torch.int32)
        for i, s in enumerate(sids):
            t[i, :len(self.blocks[s])] = torch.tensor(self.blocks[s], dtype=torch.int32)
        return t.to(self.k.device)

    def lens(self, sids: list[int]) -> torch.Tensor:
        return torch.tensor([self.length[s] for s in sids], dtype=torch.int32, device=self.k.device)


class PagedView:
    """The sequences of one batch in a :class:`PagedKVCache` (what a model layer receives as its cache)."""

    def __init__(self, pool: PagedKVCache, sids: list[int]):
        self.pool, self.sids = pool, sids

    @property
    def len(self) -> int:
        return max(self.pool.length[s] for s in self.sids)

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        self.pool.append(self.sids, k, v)

    def decode(self, q: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
        """One query token per sequence ``[B, Hq, hd]`` against its cached rows."""
        p = self.pool
        return decode_attention(q, p.k, p.v, p.lens(self.sids), scale, block_table=p.block_table(self.sids))

    def contiguous(self) -> tuple[torch.Tensor, torch.Tensor]:
        """``[B, Hk, len, hd]`` K and V (prefill continuing an earlier prefix)."""
        p = self.pool
        t, ln = p.block_table(self.sids), p.lens(self.sids)
        return gather_paged(p.k, t, ln), gather_paged(p.v, t, ln)


def gather_paged(pool: torch.Tensor, table: torch.Tensor, lens: torch.Tensor) -> torch.Tensor:
    """Contiguous ``[B, Hk, max(lens), hd]`` copy of paged rows (oracle / debugging)."""
    B, L = table.shape[0], int(lens.max())
    t = torch.arange(L, device=pool.device)
    blk = table.long()[:, t // pool.shape[2]]  # [B, L]
    rows = pool[blk, :, (t % pool.shape[2])[None, :].expand(B, L)]  # [B, L, Hk, hd]
    return rows.permute(0, 2, 1, 3)


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
                     scale: Optional[float] = None, splits: int = 0,
                     block_table: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q ``[B, Hq, hd]`` against caches ``[B, Hk, Lmax, hd]``, or block pools ``[blocks, Hk, block, hd]`` with
    ``block_table`` ``[B, max_blocks]`` (:class:`PagedKVCache`)."""
    hd = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    rep = q.shape[1] // k_cache.shape[1]
    reps = (1, 2, 4, 8, 16) if hd == 128 else (1, 2, 4, 8)
    if not q.is_cuda or hd not in (64, 128) or rep not in reps or q.dtype != torch.bfloat16:
        if block_table is not None:
            k_cache, v_cache = gather_paged(k_cache, block_table, lens), gather_paged(v_cache, block_table, lens)
        return decode_attention_reference(q, k_cache, v_cache, lens, scale)
    # splits <= 0: the extension picks the key split count for the kernel that runs (tcgen05 at head_dim 128)
    bt = block_table.to(torch.int32).contiguous() if block_table is not None else None
    return _ext().decode_attention(q.contiguous(), k_cache, v_cache, lens.to(torch.int32).contiguous(), float(scale),
                                   int(splits), bt)


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
