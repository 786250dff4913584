"""In-memory replay buffer for the v1 (sync / separate-async) diffusion trainers.

Plays the role of verl's ReplayBuffer + TransferQueue rows used by
``verl_omni/trainer/diffusion/v1/trainer_base.py:130-145,699-771`` and
``verl_omni/agent_loop/diffusion_agent_loop_tq.py:123-166``:

* trajectories are stored per prompt group (``uid``) with tags ``status`` (``finished`` /
  ``failure``), ``min_global_steps`` / ``max_global_steps`` (weight versions seen while generating);
* ``sample(global_steps, batch_size)`` returns ``batch_size`` complete groups, oldest first (``fifo``)
  or newest first (``lifo``); groups staler than ``max_off_policy_threshold`` optimizer versions are dropped;
* failed groups (any sibling aborted after retries) are evicted and replaced by exactly as many new
  prompts through ``refill_fn``, for at most ``max_refill_rounds`` rounds;
* staleness metrics: ``training/staleness/{mean,max}`` over the sampled groups.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Callable, Optional

from verl_omni_b200.utils.dataproto import DataProto


@dataclass
class Group:
    uid: str
    n: int
    rows: list = field(default_factory=list)  # list[DataProto] (one row each)
    failed: bool = False
    min_step: int = 1 << 60
    max_step: int = -1
    submit_step: int = 0

    @property
    def complete(self) -> bool:
        return self.failed or len(self.rows) == self.n


class ReplayBuffer:
    def __init__(self, max_off_policy_threshold: int = 0, strategy: str = "fifo", max_refill_rounds: int = 3):
        if strategy not in ("fifo", "lifo"):
            raise ValueError(f"unknown replay strategy {strategy!r}")
        self.max_off_policy = int(max_off_policy_threshold)
        self.strategy = strategy
        self.max_refill_rounds = max_refill_rounds
        self.groups: "OrderedDict[str, Group]" = OrderedDict()
        self._cv = threading.Condition()
        self.dropped_stale = 0

    # ------------------------------------------------------------------ producer side
    def register(self, uid: str, n: int, submit_step: int) -> None:
        with self._cv:
            self.groups[uid] = Group(uid, n, submit_step=submit_step)

    def put(self, uid: str, row: DataProto, *, status: str = "finished", min_global_steps: int = 0,
            max_global_steps: int = 0) -> None:
        with self._cv:
            g = self.groups[uid]
            if status == "failure":
                g.failed = True
            else:
                g.rows.append(row)
            g.min_step = min(g.min_step, min_global_steps)
            g.max_step = max(g.max_step, max_global_steps)
            self._cv.notify_all()

    def pending(self) -> int:
        with self._cv:
            return sum(1 for g in self.groups.values() if not g.complete)

    # ------------------------------------------------------------------ consumer side
    def _ready(self, global_steps: int) -> list[Group]:
        out = []
        for g in list(self.groups.values()):
            if not g.complete:
                continue
            if not g.failed and self.max_off_policy >= 0 and global_steps - g.min_step > self.max_off_policy > 0:
                del self.groups[g.uid]
                self.dropped_stale += 1
                continue
            out.append(g)
        out.sort(key=lambda g: g.submit_step, reverse=(self.strategy == "lifo"))
        return out

    def sample(self, global_steps: int, batch_size: int, refill_fn: Optional[Callable[[int], int]] = None,
               timeout: float = 3600.0) -> tuple[DataProto, dict]:
        """Blocks until ``batch_size`` complete, non-failed groups are available (refilling failures)."""
        metrics = {"training/rollout_failure/evicted_groups": 0, "training/rollout_failure/refill_rounds": 0}
        rounds = 0
        chosen: list[Group] = []
        with self._cv:
            while len(chosen) < batch_size:
                ready = self._ready(global_steps)
                need = batch_size - len(chosen)
                take = ready[:need]
                failed = [g for g in take if g.failed]
                good = [g for g in take if not g.failed]
                for g in good:
                    chosen.append(g)
                    del self.groups[g.uid]
                if failed:
                    if rounds >= self.max_refill_rounds:
                        raise RuntimeError(f"Exceeded max_incomplete_group_refill_rounds={self.max_refill_rounds} "
                                           "while replacing failed rollout groups")
                    for g in failed:
                        del self.groups[g.uid]
                    metrics["training/rollout_failure/evicted_groups"] += len(failed)
                    metrics["training/rollout_failure/refill_rounds"] += 1
                    rounds += 1
                    if refill_fn is None:
                        raise RuntimeError("failed groups present but no refill function")
                    self._cv.release()
                    try:
                        got = refill_fn(len(failed))
                    finally:
                        self._cv.acquire()
                    if got != len(failed):
                        raise RuntimeError(f"refill submitted {got} prompts, expected {len(failed)}")
                    continue
                if len(chosen) < batch_size and not self._cv.wait(timeout=timeout):
                    raise TimeoutError("replay buffer: timed out waiting for complete groups")
        rows = [r for g in chosen for r in g.rows]
        batch = DataProto.concat(rows)
        stale = [global_steps - g.min_step for g in chosen]
        metrics["training/staleness/mean"] = sum(stale) / len(stale)
        metrics["training/staleness/max"] = max(stale)
        metrics["training/replay/dropped_stale_groups"] = self.dropped_stale
        return batch, metrics
