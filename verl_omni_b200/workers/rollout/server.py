"""In-process asynchronous rollout server over the DiT engine (request batching front end).

Agent loops submit one :class:`DiffusionRequest` per sample and await a :class:`RolloutOutput`.
A single batching task drains the queue, groups requests that may share a device batch
(:func:`pack_key`), packs up to ``max_num_seqs`` rows per engine call and splits the result per
request.  Engine calls run on a worker thread (the GPU work releases the GIL) so the event loop
keeps accepting requests while a batch is on the device; one engine call is in flight at a time.

Plays the role of the reference's vLLM-Omni rollout replica + its async server
(``verl_omni/workers/rollout/vllm_rollout/vllm_omni_async_server.py``), without HTTP or a separate
process: trainer, server and engine share one process and one CUDA context per GPU.
"""

from __future__ import annotations

import asyncio
import concurrent.futures
import os
from typing import Optional

from verl_omni_b200.pipelines.request_batch import (DiffusionRequest, RolloutOutput, collate_requests, pack_key,
                                                    split_batched_output)


class DiffusionRolloutServer:
    def __init__(self, engine, *, max_num_seqs: Optional[int] = None, batch_wait_s: float = 0.002,
                 pad_keys: tuple[str, ...] = ()):
        self.engine = engine
        self.max_num_seqs = int(max_num_seqs or engine.cfg.max_num_seqs)
        self.batch_wait_s = batch_wait_s
        self.pad_keys = pad_keys
        self._queue: Optional[asyncio.Queue] = None
        self._task: Optional[asyncio.Task] = None
        self._pool = concurrent.futures.ThreadPoolExecutor(max_workers=1, thread_name_prefix="dit-rollout")
        self.num_engine_calls = 0
        self._inflight: Optional[asyncio.Future] = None
        self._pending: list = []  # taken off the queue, not yet in an engine call

    # ------------------------------------------------------------------ lifecycle
    def _ensure_started(self) -> None:
        loop = asyncio.get_running_loop()
        if self._task is None or self._task.done() or self._task.get_loop() is not loop:
            self._queue = asyncio.Queue()
            self._task = loop.create_task(self._serve())

    async def stop(self) -> None:
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass
            self._task = None

    def abort(self) -> None:
        """Stops the running engine call; its unfinished rows come back marked aborted."""
        self.engine.abort()

    async def abort_all_requests(self, drain_timeout_s: Optional[float] = None) -> int:
        """Drain, then hard abort (``vllm_omni_async_server.py:790-912`` of the reference).

        Requests still queued are answered at once with a synthesized aborted output; the engine call in
        flight gets ``drain_timeout_s`` (default ``VERL_OMNI_ABORT_DRAIN_TIMEOUT_S`` or 120 s) to finish,
        after which the engine is told to abort and returns its unfinished rows marked aborted.  Returns
        the number of queued requests answered without running, so callers never wait forever."""
        if drain_timeout_s is None:
            drain_timeout_s = float(os.environ.get("VERL_OMNI_ABORT_DRAIN_TIMEOUT_S", "120"))
        waiting = list(self._pending)
        if self._queue is not None:
            while True:
                try:
                    waiting.append(self._queue.get_nowait())
                except asyncio.QueueEmpty:
                    break
        n = 0
        for req, fut in waiting:
            if not fut.done():
                fut.set_result(RolloutOutput({}, {"aborted": True, "request_id": req.request_id,
                                                  "finish_reason": "abort"}))
                n += 1
        inflight = self._inflight
        if inflight is not None and not inflight.done():
            try:
                await asyncio.wait_for(asyncio.shield(inflight), drain_timeout_s)
            except asyncio.TimeoutError:
                self.engine.abort()
                try:
                    await inflight
                except Exception:  # noqa: BLE001 - the aborted call's error already reached its requests
                    pass
            except Exception:  # noqa: BLE001
                pass
        return n

    async def wake_up(self) -> None:
        self.engine.wake_up()

    async def sleep(self) -> None:
        self.engine.sleep()

    # ------------------------------------------------------------------ requests
    async def generate(self, req: DiffusionRequest) -> RolloutOutput:
        self._ensure_started()
        fut = asyncio.get_running_loop().create_future()
        await self._queue.put((req, fut))
        return await fut

    async def _serve(self) -> None:
        loop = asyncio.get_running_loop()
        while True:
            first = await self._queue.get()
            items = [first]
            # gather everything already queued, plus stragglers arriving within the batching window
            deadline = loop.time() + self.batch_wait_s
            while True:
                try:
                    items.append(self._queue.get_nowait())
                    continue
                except asyncio.QueueEmpty:
                    pass
                left = deadline - loop.time()
                if left <= 0 or len(items) >= self.max_num_seqs:
                    break
                try:
                    items.append(await asyncio.wait_for(self._queue.get(), left))
                except asyncio.TimeoutError:
                    break
            groups: dict[tuple, list] = {}
            for req, fut in items:
                groups.setdefault(pack_key(req, self._window(req)), []).append((req, fut))
            self._pending = list(items)
            for group in groups.values():
                for s in range(0, len(group), self.max_num_seqs):
                    chunk = [(r, f) for r, f in group[s:s + self.max_num_seqs] if not f.done()]
                    running = {id(f) for _, f in chunk}
                    self._pending = [it for it in self._pending if id(it[1]) not in running and not it[1].done()]
                    if not chunk:
                        continue
                    try:
                        self._inflight = loop.run_in_executor(self._pool, self._run, [r for r, _ in chunk])
                        outs = await self._inflight
                    except Exception as e:  # noqa: BLE001 - surface the failure to every waiting request
                        for _, fut in chunk:
                            if not fut.done():
                                fut.set_exception(e)
                        continue
                    for (_, fut), o in zip(chunk, outs):
                        if not fut.done():
                            fut.set_result(o)

    def _window(self, req: DiffusionRequest) -> tuple[int, int]:
        from verl_omni_b200.workers.rollout.dit_rollout import select_sde_window

        s = req.sampling
        return select_sde_window(self.engine.cfg.algo, int(self.engine.cfg.pipeline.num_inference_steps),
                                 int(req.global_step), int(s.get("window_seed", 0)))

    def _run(self, reqs: list[DiffusionRequest]) -> list[RolloutOutput]:
        batch, seeds = collate_requests(reqs, self.pad_keys)
        s = reqs[0].sampling
        out = self.engine.generate(
            batch, seed=int(s.get("window_seed", 0)), global_step=int(reqs[0].global_step),
            record_logprobs=bool(s.get("logprobs", True)), decode=bool(s.get("decode", True)), row_seeds=seeds,
            window=self._window(reqs[0]), noise_level=s.get("noise_level"), sde_type=s.get("sde_type"),
            guidance_scale=s.get("guidance_scale"))
        self.num_engine_calls += 1
        return split_batched_output(out, [r.request_id for r in reqs], {"global_step": int(reqs[0].global_step)})
