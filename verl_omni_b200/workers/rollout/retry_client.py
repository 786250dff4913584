"""Whole-sample retry client (``verl_omni/workers/rollout/diffusion_llm_server.py:29-102``).

Aborted diffusion samples (a rollout replica was drained / switched to training mode) are resubmitted
as whole samples up to ``max_attempts`` times with ``wait_s`` between attempts.  The weight versions
seen by each sample are recorded as ``min_global_steps`` / ``max_global_steps`` for the staleness
accounting of the async trainer; samples still aborted after the last attempt are returned with
status ``failure``.
"""

from __future__ import annotations

import time
from typing import Callable

import numpy as np
import torch

from verl_omni_b200.utils.dataproto import DataProto


class WholeSampleRetryClient:
    def __init__(self, generate_fn: Callable[[DataProto], DataProto], version_fn: Callable[[], int],
                 max_attempts: int = 50, wait_s: float = 1.0):
        self.generate_fn = generate_fn
        self.version_fn = version_fn
        self.max_attempts = max_attempts
        self.wait_s = wait_s
        self.retries = 0

    def generate(self, batch: DataProto) -> tuple[DataProto, np.ndarray, np.ndarray, np.ndarray]:
        """Returns (outputs, status[B] in {'finished','failure'}, min_steps[B], max_steps[B])."""
        B = len(batch)
        results: list = [None] * B
        status = np.array(["failure"] * B, dtype=object)
        vmin = np.full(B, 1 << 60, dtype=np.int64)
        vmax = np.full(B, -1, dtype=np.int64)
        todo = np.arange(B)
        for attempt in range(self.max_attempts):
            v0 = self.version_fn()
            out = self.generate_fn(batch.select_idxs(todo))
            v1 = self.version_fn()
            aborted = np.asarray(out.meta_info.get("aborted", np.zeros(len(out), dtype=bool)), dtype=bool)
            vmin[todo] = np.minimum(vmin[todo], v0)
            vmax[todo] = np.maximum(vmax[todo], v1)
            done = todo[~aborted]
            for j, i in enumerate(todo):
                if not aborted[j]:
                    results[i] = out.select_idxs([j])
                    status[i] = "finished"
            todo = todo[aborted]
            if len(todo) == 0:
                break
            self.retries += len(todo)
            if attempt + 1 < self.max_attempts and self.wait_s > 0:
                time.sleep(self.wait_s)
        ok = [r for r in results if r is not None]
        merged = DataProto.concat(ok) if ok else DataProto()
        return merged, status, vmin, vmax
