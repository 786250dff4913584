"""Request packing for the in-process diffusion rollout server.

Many single-sample requests (one per agent loop) are packed into device batches of up to
``max_num_seqs`` rows.  Packing must not change any sample's result, so:

* every request carries its own seed; the engine keys that sample's initial noise and SDE noise by
  it (``row_seeds``), never by its row position;
* requests are only packed together when they share the parameters that shape a whole batch
  (number of steps, guidance, SDE type / noise level, and the SDE window that ``global_step`` and
  the window policy select) -- :func:`pack_key`;
* prompt-embedding rows of different lengths are right-padded to a common length with a matching
  attention mask (:func:`collate_requests`), and outputs are split back per request
  (:func:`split_batched_output`) inside a ``{payload, metadata}`` envelope.

Behavioural counterparts in the reference: ``verl_omni/pipelines/request_batch.py:32-254`` (per-sample
SDE windows under packing, prompt row/mask collation, per-request output split) and
``verl_omni/pipelines/diffusion_rollout_output.py:33-137`` (the output envelope).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional

import numpy as np
import torch

from verl_omni_b200.utils.dataproto import DataProto


@dataclass
class DiffusionRequest:
    """One sample to generate: conditioning tensors (no batch dim) + sampling parameters."""

    request_id: str
    cond: dict[str, torch.Tensor]
    sampling: dict[str, Any]
    seed: int
    global_step: int = 0


@dataclass
class RolloutOutput:
    """``payload``: per-sample tensors (no batch dim); ``metadata``: scalars / strings about the run."""

    payload: dict[str, torch.Tensor]
    metadata: dict[str, Any] = field(default_factory=dict)

    @property
    def aborted(self) -> bool:
        return bool(self.metadata.get("aborted", False))


_BATCH_SHAPING_KEYS = ("num_inference_steps", "guidance_scale", "sde_type", "noise_level", "sde_window_size",
                       "sde_window_range", "logprobs", "height", "width")


def pack_key(req: DiffusionRequest, window: Optional[tuple[int, int]] = None) -> tuple:
    """Requests with equal keys may share a device batch."""
    s = req.sampling
    parts = []
    for k in _BATCH_SHAPING_KEYS:
        v = s.get(k)
        parts.append(tuple(v) if isinstance(v, (list, tuple)) else v)
    shapes = tuple(sorted((k, tuple(v.shape[1:]) if v.dim() > 1 else ()) for k, v in req.cond.items()))
    return tuple(parts) + (window, shapes)


def collate_requests(reqs: list[DiffusionRequest], pad_keys: tuple[str, ...] = ()) -> tuple[DataProto, torch.Tensor]:
    """Stacks the requests' conditioning into one batch; returns ``(batch, row_seeds int64 [B])``.

    Keys in ``pad_keys`` are sequence tensors ``[L, D]`` of varying ``L``: they are right-padded with
    zeros to the longest and an ``<key>_mask`` ``[B, Lmax]`` (1 = real token) is added.
    """
    if not reqs:
        raise ValueError("empty request list")
    keys = list(reqs[0].cond.keys())
    tensors = {}
    for k in keys:
        rows = [r.cond[k] for r in reqs]
        if k in pad_keys:
            L = max(int(t.shape[0]) for t in rows)
            out = rows[0].new_zeros((len(rows), L) + tuple(rows[0].shape[1:]))
            mask = torch.zeros(len(rows), L, dtype=torch.int64, device=rows[0].device)
            for i, t in enumerate(rows):
                out[i, : t.shape[0]] = t
                mask[i, : t.shape[0]] = 1
            tensors[k] = out
            tensors[k + "_mask"] = mask
        else:
            tensors[k] = torch.stack(rows, 0)
    batch = DataProto(tensors, {"request_id": np.array([r.request_id for r in reqs], dtype=object)})
    seeds = torch.tensor([int(r.seed) for r in reqs], dtype=torch.int64)
    return batch, seeds


def split_batched_output(out: DataProto, request_ids: list[str], metadata: Optional[dict] = None) -> list[RolloutOutput]:
    """One :class:`RolloutOutput` per row of a batched engine output."""
    aborted = out.meta_info.get("aborted")
    res = []
    for i, rid in enumerate(request_ids):
        payload = {k: v[i] for k, v in out.batch.items()}
        md = dict(metadata or {})
        md["request_id"] = rid
        md["aborted"] = bool(aborted[i]) if aborted is not None else False
        for k in ("sde_window", "num_inference_steps"):
            if k in out.meta_info:
                md[k] = out.meta_info[k]
        res.append(RolloutOutput(payload, md))
    return res


def pad_prompt_extra_field(name: str, t: torch.Tensor, max_len: int) -> torch.Tensor:
    """Right-pad (or reject) a per-sample prompt-side sequence tensor ``[L, ...]`` to ``max_len`` rows."""
    if t.dim() == 0:
        return t
    L = int(t.shape[0])
    if L > max_len:
        raise ValueError(f"{name}: length {L} exceeds max_prompt_embed_length={max_len}")
    if L == max_len:
        return t
    pad = t.new_zeros((max_len - L,) + tuple(t.shape[1:]))
    return torch.cat([t, pad], 0)
