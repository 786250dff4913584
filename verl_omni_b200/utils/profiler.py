"""Step-gated profiling (``verl_omni/trainer/config/profiler/profiler.yaml``, ``ray_diffusion_trainer.py:958-997``).

``global_profiler.tool``: ``torch`` (torch.profiler traces to ``save_path``), ``torch_memory``
(CUDA allocator history snapshots), ``nsys`` (``cudaProfilerStart/Stop`` capture ranges for
``nsys --capture-range=cudaProfilerApi``) or null.  ``global_profiler.steps`` lists the steps to
capture; ``profile_continuous_steps`` merges consecutive steps into one capture.  ``mark(name)``
emits NVTX ranges around trainer phases for any external profiler.
"""

from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch


@contextlib.contextmanager
def mark(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class StepProfiler:
    def __init__(self, cfg, rank: int = 0):
        self.tool = cfg.get("tool") if cfg else None
        self.steps = set(cfg.get("steps") or []) if cfg else set()
        self.continuous = bool(cfg.get("profile_continuous_steps", False)) if cfg else False
        self.save_path = (cfg.get("save_path") if cfg else None) or "outputs/profile"
        self.rank = rank
        self._prof = None
        self._active = False

    def _want(self, step: int) -> bool:
        return self.tool is not None and step in self.steps

    def start(self, step: int) -> None:
        if not self._want(step) or self._active:
            return
        os.makedirs(self.save_path, exist_ok=True)
        if self.tool == "torch":
            acts = [torch.profiler.ProfilerActivity.CPU]
            if torch.cuda.is_available():
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self._prof = torch.profiler.profile(activities=acts, record_shapes=True)
            self._prof.__enter__()
        elif self.tool == "torch_memory" and torch.cuda.is_available():
            torch.cuda.memory._record_memory_history(max_entries=100000)
        elif self.tool == "nsys" and torch.cuda.is_available():
            torch.cuda.cudart().cudaProfilerStart()
        self._active = True

    def stop(self, step: int) -> Optional[str]:
        if not self._active:
            return None
        if self.continuous and (step + 1) in self.steps:
            return None
        out = None
        if self.tool == "torch" and self._prof is not None:
            self._prof.__exit__(None, None, None)
            out = os.path.join(self.save_path, f"trace_step{step}_rank{self.rank}.json")
            self._prof.export_chrome_trace(out)
            self._prof = None
        elif self.tool == "torch_memory" and torch.cuda.is_available():
            out = os.path.join(self.save_path, f"memory_step{step}_rank{self.rank}.pickle")
            torch.cuda.memory._dump_snapshot(out)
            torch.cuda.memory._record_memory_history(enabled=None)
        elif self.tool == "nsys" and torch.cuda.is_available():
            torch.cuda.cudart().cudaProfilerStop()
        self._active = False
        return out
