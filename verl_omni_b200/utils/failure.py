"""Host-side failure detection: rank liveness heartbeats and capacity-expiration checkpoints.

* :class:`HeartbeatMonitor` - every rank publishes a monotonically increasing beat in a TCP key-value
  store from a daemon thread; :meth:`HeartbeatMonitor.check` (called between steps, before the next
  collective) raises :class:`RankFailure` naming the ranks whose beat has not advanced within the
  timeout.  A rank that crashed or hangs in host code is reported to the survivors instead of
  leaving them blocked in their next collective until the process-group timeout.
* :func:`should_save_ckpt_esi` - the training-plan / elastic-instance expiration rule of the
  reference trainer (``verl_omni/trainer/diffusion/ray_diffusion_trainer.py:1265-1285``): force a
  checkpoint when the capacity block expires within ``redundant_time`` plus the longest step seen.
  The expiration is read from the same environment variables as the reference's platform helpers.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Optional

_EXPIRATION_ENVS = ("MLP_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP",
                    "SAGEMAKER_CURRENT_CAPACITY_BLOCK_EXPIRATION_TIMESTAMP")


def should_save_ckpt_esi(max_steps_duration: float, redundant_time: float = 0.0,
                         now: Optional[float] = None) -> bool:
    """True when the capacity block ends before another step plus ``redundant_time`` seconds fit."""
    now = time.time() if now is None else now
    for name in _EXPIRATION_ENVS:
        v = os.environ.get(name)
        if not v:
            continue
        try:
            expire = float(v)
        except ValueError:
            continue
        if expire > 1e12:  # milliseconds
            expire /= 1000.0
        if now + float(redundant_time) + float(max_steps_duration) >= expire:
            return True
    return False


class RankFailure(RuntimeError):
    def __init__(self, ranks: list[int]):
        super().__init__(f"ranks {ranks} stopped sending heartbeats")
        self.ranks = ranks


class HeartbeatMonitor:
    """Liveness of every rank through a TCP store (``host:port``; rank 0 hosts it)."""

    def __init__(self, rank: int, world: int, host: str, port: int, interval_s: float = 0.5,
                 timeout_s: float = 30.0):
        import torch.distributed as dist

        self.rank, self.world = rank, world
        self.interval, self.timeout = interval_s, timeout_s
        self.store = dist.TCPStore(host, port, world, rank == 0, timeout=__import__("datetime").timedelta(
            seconds=max(30.0, timeout_s)))
        self._stop = threading.Event()
        self._beat = 0
        self._seen: dict[int, tuple[int, float]] = {}
        self.store.set(f"hb/{rank}", "0")
        self._thread = threading.Thread(target=self._run, name="heartbeat", daemon=True)
        self._thread.start()

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            self._beat += 1
            try:
                self.store.set(f"hb/{self.rank}", str(self._beat))
            except Exception:  # noqa: BLE001 - the store host itself died; check() reports it
                return

    def check(self) -> None:
        """Raises :class:`RankFailure` if some rank's beat has not advanced for ``timeout_s``."""
        now = time.monotonic()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                beat = int(self.store.get(f"hb/{r}"))
            except Exception:  # noqa: BLE001 - store unreachable: treat the host rank as failed
                dead.append(r)
                continue
            last = self._seen.get(r)
            if last is None or beat != last[0]:
                self._seen[r] = (beat, now)
            elif now - last[1] > self.timeout:
                dead.append(r)
        if dead:
            raise RankFailure(dead)

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)
