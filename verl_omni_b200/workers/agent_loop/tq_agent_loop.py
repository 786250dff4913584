"""Non-blocking agent-loop worker that streams finished trajectories into the replay buffer (v1).

Behaviour of the reference's ``verl_omni/agent_loop/diffusion_agent_loop_tq.py:40-264``: ``submit``
returns immediately; each of the ``rollout.n`` sessions of a prompt writes its row to the buffer as
it finishes, tagged ``status`` and the weight versions (``min/max_global_steps``) it saw.  A
session that comes back aborted (after the whole-sample retries) marks its group failed; the
failure is published only after every sibling of the group has settled, so the consumer never
sees a half-written group.  The buffer role of TransferQueue is played by
:class:`~verl_omni_b200.trainer.diffusion.v1.replay_buffer.ReplayBuffer`.
"""

from __future__ import annotations

import asyncio
import threading
from typing import Callable, Optional

import numpy as np

from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.agent_loop.diffusion_agent_loop import DiffusionAgentLoopWorker


class DiffusionAgentLoopWorkerTQ(DiffusionAgentLoopWorker):
    def __init__(self, *args, replay_buffer, version_fn: Callable[[], int], **kwargs):
        super().__init__(*args, **kwargs)
        self.buffer = replay_buffer
        self.version_fn = version_fn
        self._loop: Optional[asyncio.AbstractEventLoop] = None
        self._thread: Optional[threading.Thread] = None

    def _ensure_loop(self) -> asyncio.AbstractEventLoop:
        if self._loop is None:
            self._loop = asyncio.new_event_loop()
            self._thread = threading.Thread(target=self._loop.run_forever, name="agent-loop-tq", daemon=True)
            self._thread.start()
        return self._loop

    def submit(self, batch: DataProto, n: int) -> "asyncio.Future":
        """Registers the groups and schedules generation; returns a future that resolves when done."""
        uids = batch.non_tensor_batch["uid"]
        step = int(batch.meta_info.get("global_steps", 0))
        for u in dict.fromkeys(uids.tolist()):
            self.buffer.register(str(u), n, step)
        return asyncio.run_coroutine_threadsafe(self._generate_and_stream(batch), self._ensure_loop())

    async def _generate_and_stream(self, batch: DataProto) -> int:
        v0 = int(self.version_fn())
        out = await self.generate_sequences(batch)
        v1 = int(self.version_fn())
        uids = out.non_tensor_batch["uid"]
        aborted = out.non_tensor_batch.get("aborted", np.zeros(len(out), dtype=bool))
        failed_groups = {str(u) for u, a in zip(uids, aborted) if a}
        for i in range(len(out)):
            u = str(uids[i])
            if u in failed_groups:
                continue
            self.buffer.put(u, out.select_idxs([i]), status="finished", min_global_steps=v0, max_global_steps=v1)
        # all siblings have settled (generate_sequences gathered every session): publish failures last
        for u in failed_groups:
            self.buffer.put(u, None, status="failure", min_global_steps=v0, max_global_steps=v1)
        return len(out)

    def shutdown(self) -> None:
        if self._loop is not None:
            async def _stop():
                await self.server.stop()
                if self._reward is not None:
                    await self._reward.stop()

            asyncio.run_coroutine_threadsafe(_stop(), self._loop).result(timeout=30)
            self._loop.call_soon_threadsafe(self._loop.stop)
            self._thread.join(timeout=10)
            self._loop = None
