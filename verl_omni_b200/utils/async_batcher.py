"""Coalesces concurrent single-item awaits into batched calls of a synchronous function.

``AsyncBatcher(fn, max_batch)``: ``await batcher(item)`` queues the item; a drain task calls
``fn(list_of_items) -> list_of_results`` on a worker thread with everything queued (up to
``max_batch``) and resolves each caller with its own result.  Used by the agent loops to stream
per-sample reward computation into batched scorer calls.
"""

from __future__ import annotations

import asyncio
import concurrent.futures
from typing import Any, Callable, Optional


class AsyncBatcher:
    def __init__(self, fn: Callable[[list], list], max_batch: int = 64, wait_s: float = 0.001):
        self.fn = fn
        self.max_batch = max(1, int(max_batch))
        self.wait_s = wait_s
        self._queue: Optional[asyncio.Queue] = None
        self._task: Optional[asyncio.Task] = None
        self._pool = concurrent.futures.ThreadPoolExecutor(max_workers=1, thread_name_prefix="async-batcher")
        self.num_calls = 0

    def _ensure_started(self) -> None:
        loop = asyncio.get_running_loop()
        if self._task is None or self._task.done() or self._task.get_loop() is not loop:
            self._queue = asyncio.Queue()
            self._task = loop.create_task(self._serve())

    async def __call__(self, item: Any) -> Any:
        self._ensure_started()
        fut = asyncio.get_running_loop().create_future()
        await self._queue.put((item, fut))
        return await fut

    async def _serve(self) -> None:
        loop = asyncio.get_running_loop()
        while True:
            items = [await self._queue.get()]
            deadline = loop.time() + self.wait_s
            while len(items) < self.max_batch:
                try:
                    items.append(self._queue.get_nowait())
                    continue
                except asyncio.QueueEmpty:
                    pass
                left = deadline - loop.time()
                if left <= 0:
                    break
                try:
                    items.append(await asyncio.wait_for(self._queue.get(), left))
                except asyncio.TimeoutError:
                    break
            try:
                res = await loop.run_in_executor(self._pool, self.fn, [x for x, _ in items])
                self.num_calls += 1
            except Exception as e:  # noqa: BLE001
                for _, fut in items:
                    if not fut.done():
                        fut.set_exception(e)
                continue
            for (_, fut), r in zip(items, res):
                if not fut.done():
                    fut.set_result(r)

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass
            self._task = None
