"""Parquet-backed datasets with the same ``get_batch(ids) -> DataProto`` interface as the synthetic ones.

* :class:`ParquetPromptDataset` -- RLHF prompts (reference ``verl_omni/utils/dataset/rl_dataset.py:65-153``
  on verl's ``RLHFDataset``): one row per prompt with ``prompt`` (a string or chat messages),
  optional ``negative_prompt``, ``data_source``, ``reward_model.ground_truth``; precomputed conditioning
  columns (``prompt_embeds``, ``pooled_prompt_embeds``, ...) are served as tensors when present, otherwise
  the prompt text is tokenized into ``input_ids`` (a model-supplied tokenizer callable, or a byte-level
  fallback: UTF-8 bytes mod vocab, right-padded / truncated to ``max_prompt_length``).
* :class:`ParquetOfflineDPODataset` -- offline diffusion DPO pairs (reference
  ``utils/dataset/offline_dpo_dataset.py:170-315``): ``img_win_latents`` / ``img_lose_latents`` plus the
  prompt conditioning; rows come out interleaved ``[chosen, rejected, ...]`` with ``rm_scores`` win / lose.
* :class:`ParquetMLLMDPODataset` -- offline omni DPO (reference ``utils/dataset/offline_mllm_dpo_dataset.py``):
  ``prompt_ids``, ``chosen_ids``, ``rejected_ids`` (+ optional ``audio_feats`` / ``image_patches``).
* :class:`ParquetOmniRLDataset` -- online omni RL prompts (reference ``utils/dataset/omni_rl_datasets.py``):
  ``prompt_ids`` (token ids holding the audio / image placeholder tokens) or ``prompt`` text, with optional
  ``audio_feats`` / ``image_patches`` arrays, ``data_source`` and ``reward_model.ground_truth``.

Tensor columns hold nested lists (any depth) or flat lists with a ``<col>_shape`` column.
"""

from __future__ import annotations

import json
from typing import Callable, Optional, Sequence

import numpy as np
import torch

from verl_omni_b200.utils.dataproto import DataProto


def _read(files) -> "object":
    import pyarrow.parquet as pq
    import pyarrow as pa

    files = [files] if isinstance(files, str) else list(files)
    return pa.concat_tables([pq.read_table(f) for f in files]).to_pandas()


def _tensor(row, key: str, dtype=torch.float32) -> Optional[torch.Tensor]:
    if key not in row or row[key] is None:
        return None
    v = row[key]
    shape_key = f"{key}_shape"
    arr = np.asarray(v.tolist() if hasattr(v, "tolist") else v)
    if arr.dtype == object:  # nested lists read back as arrays of arrays
        arr = np.stack([np.asarray(x) for x in arr])
        while arr.dtype == object:
            arr = np.stack([np.stack([np.asarray(y) for y in x]) for x in arr])
    t = torch.as_tensor(arr)
    if shape_key in row and row[shape_key] is not None:
        t = t.reshape([int(x) for x in row[shape_key]])
    return t.to(dtype)


def _prompt_text(v) -> str:
    """A plain string, or the concatenated contents of chat messages."""
    if isinstance(v, str):
        return v
    try:
        msgs = list(v)
        return "\n".join(str(m.get("content", "")) if isinstance(m, dict) else str(m) for m in msgs)
    except TypeError:
        return str(v)


def byte_tokenizer(vocab: int, length: int) -> Callable[[str], list[int]]:
    def tok(text: str) -> list[int]:
        ids = [b % vocab for b in text.encode("utf-8")][:length]
        return ids + [0] * (length - len(ids))

    return tok


class ParquetPromptDataset:
    def __init__(self, files, *, cond_keys: Sequence[str] = (), token_len: int = 0, vocab: int = 1000,
                 tokenizer: Optional[Callable[[str], list[int]]] = None, prompt_key: str = "prompt",
                 negative_prompt_key: str = "negative_prompt", max_samples: int = -1):
        self.df = _read(files)
        if max_samples and max_samples > 0:
            self.df = self.df.iloc[:max_samples]
        if prompt_key not in self.df.columns:
            raise ValueError(f"parquet prompts need a {prompt_key!r} column; have {list(self.df.columns)}")
        self.cond_keys = tuple(cond_keys)
        self.token_len = int(token_len)
        self.tok = tokenizer or byte_tokenizer(vocab, max(1, self.token_len))
        self.prompt_key, self.negative_prompt_key = prompt_key, negative_prompt_key

    def __len__(self) -> int:
        return len(self.df)

    def get_batch(self, ids: list[int]) -> DataProto:
        rows = [self.df.iloc[int(i)].to_dict() for i in ids]
        tensors = {}
        if self.token_len:
            tensors["input_ids"] = torch.tensor([self.tok(_prompt_text(r[self.prompt_key])) for r in rows])
        for k in self.cond_keys:
            ts = [_tensor(r, k) for r in rows]
            if any(t is None for t in ts):
                raise KeyError(f"conditioning column {k!r} missing in some rows (precompute it into the parquet)")
            tensors[k] = torch.stack(ts)
        nt = {"prompt_id": np.array(ids, dtype=object),
              "raw_prompt": np.array([_prompt_text(r[self.prompt_key]) for r in rows], dtype=object),
              "data_source": np.array([r.get("data_source", "unknown") for r in rows], dtype=object)}
        if self.negative_prompt_key in self.df.columns:
            nt["raw_negative_prompt"] = np.array([_prompt_text(r.get(self.negative_prompt_key) or "")
                                                  for r in rows], dtype=object)
        gts = []
        for r in rows:
            rm = r.get("reward_model")
            if isinstance(rm, str):
                try:
                    rm = json.loads(rm)
                except ValueError:
                    rm = None
            gts.append(rm.get("ground_truth") if isinstance(rm, dict) else None)
        nt["ground_truth"] = np.array(gts, dtype=object)
        return DataProto(tensors, nt)


class ParquetOfflineDPODataset:
    def __init__(self, files, *, cond_keys: Sequence[str] = ("prompt_embeds", "pooled_prompt_embeds"),
                 win_key: str = "img_win_latents", lose_key: str = "img_lose_latents", max_samples: int = -1):
        self.df = _read(files)
        if max_samples and max_samples > 0:
            self.df = self.df.iloc[:max_samples]
        need = {win_key, lose_key, *cond_keys}
        missing = need - set(self.df.columns)
        if missing:
            raise ValueError(f"offline DPO parquet is missing columns {sorted(missing)}")
        self.cond_keys, self.win_key, self.lose_key = tuple(cond_keys), win_key, lose_key

    def __len__(self) -> int:
        return len(self.df)

    def get_batch(self, ids: list[int]) -> DataProto:
        rows = [self.df.iloc[int(i)].to_dict() for i in ids]
        lat, scores, uids = [], [], []
        cond = {k: [] for k in self.cond_keys}
        for i, r in zip(ids, rows):
            ws, ls = float(r.get("win_score", 1.0)), float(r.get("lose_score", 0.0))
            if ws < ls:
                raise ValueError(f"offline DPO row {i}: win_score {ws} < lose_score {ls}")
            lat += [_tensor(r, self.win_key), _tensor(r, self.lose_key)]
            scores += [ws, ls]
            uids += [str(r.get("uid") or f"pair-{i}")] * 2
            for k in self.cond_keys:
                t = _tensor(r, k)
                cond[k] += [t, t]
        tensors = {"latents_clean": torch.stack(lat), "rm_scores": torch.tensor(scores)}
        tensors.update({k: torch.stack(v) for k, v in cond.items()})
        return DataProto(tensors, {"uid": np.array(uids, dtype=object)})


class ParquetMLLMDPODataset:
    def __init__(self, files, *, pad_id: int = 0, max_samples: int = -1):
        self.df = _read(files)
        if max_samples and max_samples > 0:
            self.df = self.df.iloc[:max_samples]
        missing = {"prompt_ids", "chosen_ids", "rejected_ids"} - set(self.df.columns)
        if missing:
            raise ValueError(f"MLLM DPO parquet is missing columns {sorted(missing)}")
        self.pad = pad_id

    def __len__(self) -> int:
        return len(self.df)

    def get_pairs(self, ids: list[int]) -> tuple[DataProto, DataProto]:
        """(chosen, rejected) batches: ``input_ids`` = prompt + response (right-padded), ``prompts``,
        ``response_mask``, and the prompt's ``audio_feats`` / ``image_patches`` when present."""
        rows = [self.df.iloc[int(i)].to_dict() for i in ids]
        P = max(len(r["prompt_ids"]) for r in rows)
        out = []
        for key in ("chosen_ids", "rejected_ids"):
            R = max(len(r[key]) for r in rows)
            prompts = torch.full((len(rows), P), self.pad, dtype=torch.long)
            resp = torch.full((len(rows), R), self.pad, dtype=torch.long)
            mask = torch.zeros(len(rows), R)
            for j, r in enumerate(rows):
                p = list(r["prompt_ids"])
                prompts[j, P - len(p):] = torch.tensor(p)  # left-pad prompts
                c = list(r[key])
                resp[j, :len(c)] = torch.tensor(c)
                mask[j, :len(c)] = 1.0
            t = {"prompts": prompts, "responses": resp, "response_mask": mask,
                 "input_ids": torch.cat([prompts, resp], 1)}
            for feat in ("audio_feats", "image_patches"):
                if feat in self.df.columns:
                    t[feat] = torch.stack([_tensor(r, feat) for r in rows])
            out.append(DataProto(t, {"uid": np.array([f"pair-{i}" for i in ids], dtype=object)}))
        return out[0], out[1]


class ParquetOmniRLDataset:
    """Prompts for the omni GRPO / GSPO trainer.  Each batch is left-padded to ``max_prompt_length`` with
    ``pad_id`` (the thinker attends over the padding like any other prompt token, identically in the rollout
    and the log-prob recompute); longer prompts keep their last ``max_prompt_length`` tokens.  Text prompts
    without ids are tokenized byte-level.  Feature arrays are stacked per batch (equal counts per row)."""

    def __init__(self, files, *, vocab: int, max_prompt_length: int, pad_id: int = 0, max_samples: int = -1,
                 tokenizer: Optional[Callable[[str], list[int]]] = None):
        self.df = _read(files)
        if max_samples and max_samples > 0:
            self.df = self.df.iloc[:max_samples]
        if "prompt_ids" not in self.df.columns and "prompt" not in self.df.columns:
            raise ValueError("omni RL parquet needs a 'prompt_ids' or a 'prompt' column")
        self.L, self.pad = int(max_prompt_length), int(pad_id)
        self.tok = tokenizer or (lambda text: [b % vocab for b in text.encode("utf-8")])

    def __len__(self) -> int:
        return len(self.df)

    def get_batch(self, ids: list[int], uid_prefix: str = "") -> DataProto:
        rows = [self.df.iloc[int(i) % len(self.df)].to_dict() for i in ids]
        out = torch.full((len(rows), self.L), self.pad, dtype=torch.long)
        for j, r in enumerate(rows):
            toks = list(r["prompt_ids"]) if r.get("prompt_ids") is not None else self.tok(_prompt_text(r["prompt"]))
            toks = [int(t) for t in toks][-self.L:]
            out[j, self.L - len(toks):] = torch.tensor(toks, dtype=torch.long)
        t = {"input_ids": out}
        for feat in ("audio_feats", "image_patches"):
            if feat in self.df.columns:
                t[feat] = torch.stack([_tensor(r, feat) for r in rows])
        gts = []
        for r in rows:
            rm = r.get("reward_model")
            if isinstance(rm, str):
                try:
                    rm = json.loads(rm)
                except ValueError:
                    rm = None
            gts.append(rm.get("ground_truth") if isinstance(rm, dict) else None)
        nt = {"uid": np.array([f"{uid_prefix}{i}" for i in ids], dtype=object),
              "data_source": np.array([r.get("data_source", "unknown") for r in rows], dtype=object),
              "ground_truth": np.array(gts, dtype=object)}
        return DataProto(t, nt)
