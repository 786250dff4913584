"""Batch container passed between the controller, workers, rollout and reward.

Plays the role of verl's ``DataProto`` (used throughout
``verl_omni/trainer/diffusion/ray_diffusion_trainer.py:1133-1361``): a dict of tensors that
share a leading batch dimension, a dict of per-sample numpy object arrays
(``uid``, raw prompts, ...) and free-form ``meta_info``.  It also stands in for the
TensorDict micro-batches the engines consume (``tu.get_non_tensor_data`` etc.).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Iterable, Optional, Sequence

import numpy as np
import torch


@dataclass
class DataProto:
    batch: dict = field(default_factory=dict)
    non_tensor_batch: dict = field(default_factory=dict)
    meta_info: dict = field(default_factory=dict)

    def __post_init__(self):
        self.check_consistency()

    # ------------------------------------------------------------------ basics
    def __len__(self) -> int:
        for v in self.batch.values():
            return int(v.shape[0])
        for v in self.non_tensor_batch.values():
            return len(v)
        return 0

    def check_consistency(self) -> None:
        n = None
        for k, v in list(self.batch.items()):
            if not isinstance(v, torch.Tensor):
                raise TypeError(f"batch[{k!r}] must be a tensor, got {type(v)}")
            if n is None:
                n = v.shape[0]
            elif v.shape[0] != n:
                raise ValueError(f"batch[{k!r}] has leading dim {v.shape[0]}, expected {n}")
        for k, v in list(self.non_tensor_batch.items()):
            if not isinstance(v, np.ndarray):
                arr = np.empty(len(v), dtype=object)
                arr[:] = list(v)
                self.non_tensor_batch[k] = v = arr
            if n is not None and len(v) != n:
                raise ValueError(f"non_tensor_batch[{k!r}] has length {len(v)}, expected {n}")

    @classmethod
    def from_dict(cls, tensors: Optional[dict] = None, non_tensors: Optional[dict] = None,
                  meta_info: Optional[dict] = None) -> "DataProto":
        return cls(dict(tensors or {}), dict(non_tensors or {}), dict(meta_info or {}))

    def __contains__(self, key: str) -> bool:
        return key in self.batch or key in self.non_tensor_batch

    def __getitem__(self, item):
        if isinstance(item, str):
            if item in self.batch:
                return self.batch[item]
            return self.non_tensor_batch[item]
        return self.select_idxs(item)

    def get(self, key: str, default: Any = None) -> Any:
        if key in self.batch:
            return self.batch[key]
        return self.non_tensor_batch.get(key, default)

    def keys(self):
        return list(self.batch.keys()) + list(self.non_tensor_batch.keys())

    # ------------------------------------------------------------------ transforms
    def select_idxs(self, idxs) -> "DataProto":
        if isinstance(idxs, slice):
            idx_np = np.arange(len(self))[idxs]
        elif isinstance(idxs, torch.Tensor):
            idx_np = idxs.cpu().numpy()
        else:
            idx_np = np.asarray(idxs)
        if idx_np.dtype == bool:
            idx_np = np.nonzero(idx_np)[0]
        idx_t = None
        batch = {}
        for k, v in self.batch.items():
            if idx_t is None or idx_t.device != v.device:
                idx_t = torch.as_tensor(idx_np, dtype=torch.long, device=v.device)
            batch[k] = v.index_select(0, idx_t)
        nt = {k: v[idx_np] for k, v in self.non_tensor_batch.items()}
        return DataProto(batch, nt, dict(self.meta_info))

    def select(self, batch_keys: Sequence[str] = (), non_tensor_batch_keys: Sequence[str] = (),
               meta_info_keys: Optional[Sequence[str]] = None) -> "DataProto":
        b = {k: self.batch[k] for k in batch_keys}
        nt = {k: self.non_tensor_batch[k] for k in non_tensor_batch_keys}
        mi = dict(self.meta_info) if meta_info_keys is None else {k: self.meta_info[k] for k in meta_info_keys}
        return DataProto(b, nt, mi)

    def pop(self, batch_keys: Sequence[str] = (), non_tensor_batch_keys: Sequence[str] = ()) -> "DataProto":
        b = {k: self.batch.pop(k) for k in batch_keys}
        nt = {k: self.non_tensor_batch.pop(k) for k in non_tensor_batch_keys}
        return DataProto(b, nt, dict(self.meta_info))

    def union(self, other: "DataProto") -> "DataProto":
        if len(self) and len(other) and len(self) != len(other):
            raise ValueError(f"union of batches with sizes {len(self)} and {len(other)}")
        for k, v in other.batch.items():
            if k in self.batch and self.batch[k] is not v and not torch.equal(self.batch[k].cpu(), v.cpu()):
                raise ValueError(f"union conflict on batch key {k!r}")
            self.batch[k] = v
        for k, v in other.non_tensor_batch.items():
            self.non_tensor_batch[k] = v
        self.meta_info.update(other.meta_info)
        self.check_consistency()
        return self

    def repeat(self, repeat_times: int, interleave: bool = True) -> "DataProto":
        if interleave:
            b = {k: v.repeat_interleave(repeat_times, dim=0) for k, v in self.batch.items()}
            nt = {k: np.repeat(v, repeat_times, axis=0) for k, v in self.non_tensor_batch.items()}
        else:
            b = {k: v.repeat(repeat_times, *([1] * (v.ndim - 1))) for k, v in self.batch.items()}
            nt = {k: np.tile(v, repeat_times) for k, v in self.non_tensor_batch.items()}
        return DataProto(b, nt, dict(self.meta_info))

    def chunk(self, chunks: int) -> list["DataProto"]:
        n = len(self)
        if n % chunks != 0:
            raise ValueError(f"batch of {n} does not split into {chunks} equal chunks")
        size = n // chunks
        return [self.select_idxs(slice(i * size, (i + 1) * size)) for i in range(chunks)]

    def split(self, size: int) -> list["DataProto"]:
        n = len(self)
        return [self.select_idxs(slice(i, min(i + size, n))) for i in range(0, n, size)]

    @staticmethod
    def concat(items: Iterable["DataProto"]) -> "DataProto":
        items = list(items)
        if not items:
            return DataProto()
        b = {k: torch.cat([it.batch[k] for it in items], dim=0) for k in items[0].batch}
        nt = {k: np.concatenate([it.non_tensor_batch[k] for it in items], axis=0)
              for k in items[0].non_tensor_batch}
        return DataProto(b, nt, dict(items[0].meta_info))

    def to(self, device) -> "DataProto":
        self.batch = {k: v.to(device, non_blocking=True) for k, v in self.batch.items()}
        return self

    def clone(self) -> "DataProto":
        return DataProto({k: v.clone() for k, v in self.batch.items()},
                         {k: v.copy() for k, v in self.non_tensor_batch.items()}, dict(self.meta_info))

    def reorder(self, indices: torch.Tensor) -> None:
        d = self.select_idxs(indices)
        self.batch, self.non_tensor_batch = d.batch, d.non_tensor_batch

    def nbytes(self) -> int:
        return sum(v.numel() * v.element_size() for v in self.batch.values())


def pad_dataproto_to_divisor(data: DataProto, size_divisor: int) -> tuple[DataProto, int]:
    n = len(data)
    pad = (-n) % size_divisor
    if pad == 0:
        return data, 0
    idx = list(range(n)) + list(range(pad))
    return data.select_idxs(np.asarray(idx) % n), pad


def unpad_dataproto(data: DataProto, pad_size: int) -> DataProto:
    if pad_size == 0:
        return data
    return data.select_idxs(slice(0, len(data) - pad_size))
