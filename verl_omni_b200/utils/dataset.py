"""Synthetic prompt datasets and a resumable sampler.

No datasets or checkpoints are reachable offline, so prompts are generated deterministically from
``(seed, prompt_id)``: token-id prompts (uniform ids for a text encoder) or random text-encoder
output embeddings of the model's conditioning shapes.  The sampler reproduces the reference's
``StatefulDataLoader`` role (``ray_diffusion_trainer.py:256-276``): epoch-seeded shuffling and a
``state_dict`` saved as ``data.pt`` with each checkpoint.
"""

from __future__ import annotations

from typing import Optional

import zlib

import numpy as np
import torch

from verl_omni_b200.utils.dataproto import DataProto


class SyntheticPromptDataset:
    def __init__(self, num_prompts: int, *, seed: int = 0, token_len: int = 0, vocab: int = 1000,
                 cond_shapes: Optional[dict] = None, embed_dtype=torch.float32):
        self.n = int(num_prompts)
        self.seed = int(seed)
        self.token_len = token_len
        self.vocab = vocab
        self.cond_shapes = dict(cond_shapes or {})
        self.embed_dtype = embed_dtype

    def __len__(self) -> int:
        return self.n

    def _gen(self, idx: int) -> torch.Generator:
        g = torch.Generator()
        g.manual_seed(self.seed * 1_000_003 + int(idx))
        return g

    def get_batch(self, ids: list[int]) -> DataProto:
        tensors = {}
        if self.token_len:
            rows = [torch.randint(0, self.vocab, (self.token_len,), generator=self._gen(i)) for i in ids]
            tensors["input_ids"] = torch.stack(rows)
        for k, shape in self.cond_shapes.items():
            if k.endswith("_ids"):  # token ids of a model that embeds its own prompt
                rows = [torch.randint(0, self.vocab, shape, generator=self._gen(i * 31 + 3)) for i in ids]
                tensors[k] = torch.stack(rows)
                continue
            if k.endswith("_mask"):
                # right-padded prompt: a per-prompt valid length in [L/2, L]
                L = shape[0]
                lens = [int(torch.randint(L // 2, L + 1, (1,), generator=self._gen(i * 31 + 7)).item()) for i in ids]
                tensors[k] = (torch.arange(L)[None, :] < torch.tensor(lens)[:, None]).to(self.embed_dtype)
                continue
            rows = [torch.randn(shape, generator=self._gen(i * 31 + zlib.crc32(k.encode()) % 17)) for i in ids]
            tensors[k] = torch.stack(rows).to(self.embed_dtype)
        return DataProto(tensors, {"prompt_id": np.array(ids, dtype=object),
                                   "raw_prompt": np.array([f"prompt-{i}" for i in ids], dtype=object)})


class ResumableSampler:
    """Yields global batches of prompt ids; epoch-shuffled with ``seed + epoch``."""

    def __init__(self, n: int, batch_size: int, seed: int = 0, shuffle: bool = True, drop_last: bool = True):
        self.n, self.bs, self.seed, self.shuffle, self.drop_last = n, batch_size, seed, shuffle, drop_last
        self.epoch, self.pos = 0, 0

    def _order(self) -> np.ndarray:
        if not self.shuffle:
            return np.arange(self.n)
        return np.random.default_rng(self.seed + self.epoch).permutation(self.n)

    def next_batch(self) -> list[int]:
        if self.pos + self.bs > self.n:
            self.epoch += 1
            self.pos = 0
        ids = self._order()[self.pos:self.pos + self.bs].tolist()
        self.pos += self.bs
        return ids

    def __len__(self) -> int:
        return self.n // self.bs

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "pos": self.pos}

    def load_state_dict(self, sd: dict) -> None:
        self.epoch, self.pos = int(sd["epoch"]), int(sd["pos"])
