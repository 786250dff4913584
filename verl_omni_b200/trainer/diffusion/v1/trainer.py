"""v1 diffusion trainers: replay-buffer driven ``sync`` and ``separate_async`` modes.

Counterparts of ``verl_omni/trainer/diffusion/v1/trainer_base.py:104-386``,
``trainer_sync.py:44-67`` and ``trainer_separate_async.py:64-293``:

* a registry ``register_diffusion_trainer`` / ``get_diffusion_trainer_cls`` keyed by
  ``trainer.v1.trainer_mode``;
* the lifecycle hooks ``on_init_end / on_train_begin / on_step_begin / on_sample_begin /
  on_sample_end / on_step_end / on_train_end``;
* ``step`` runs ``parameter_sync_step`` local updates, each sampling complete prompt groups from the
  replay buffer (failed groups evicted and refilled), then ``on_step_end`` syncs weights;
* ``sync``: the rollout engine is colocated and shares the trainer's weights; generation for a step
  happens when it is sampled, so every batch is on-policy;
* ``separate_async``: a standalone rollout replica (its own weight copy) runs on a background thread
  and CUDA stream of the same rank, kept ``warmup_batches + 1`` batches ahead; weight pushes every
  ``parameter_sync_step`` updates (an in-process copy); in-flight generations are aborted at a push unless
  ``partial_rollout`` is set and the whole-sample retry client regenerates them on the new weights;
  staleness is tracked per group;
* ``trainer.v1.standalone_rollout_ranks = R > 0``: rollout on the last R ranks of the job instead, weights
  pushed across GPUs by one peer-store kernel (``trainer/diffusion/v1/standalone.py``).
"""

from __future__ import annotations

import contextlib
import copy
import queue
import threading
import time
from typing import Optional

import numpy as np
import torch

from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
from verl_omni_b200.trainer.diffusion.v1.replay_buffer import ReplayBuffer
from verl_omni_b200.utils import metrics as M
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.rollout.dit_rollout import DiTRolloutEngine
from verl_omni_b200.workers.rollout.retry_client import WholeSampleRetryClient

_TRAINERS: dict[str, type] = {}


def register_diffusion_trainer(name: str):
    def deco(cls):
        _TRAINERS[name] = cls
        return cls

    return deco


def get_diffusion_trainer_cls(name: str) -> type:
    if name not in _TRAINERS:
        raise ValueError(f"unknown v1 trainer_mode {name!r}; known: {sorted(_TRAINERS)}")
    return _TRAINERS[name]


def build_v1_trainer(config):
    if int(config.trainer.v1.get("standalone_rollout_ranks", 0) or 0) > 0:
        # rollout on dedicated ranks of the job (trainer ranks + rollout ranks, weights pushed across GPUs)
        from verl_omni_b200.trainer.diffusion.v1.standalone import build_standalone

        return build_standalone(config)
    return get_diffusion_trainer_cls(config.trainer.v1.trainer_mode)(config)


class PolicyGradientDiffusionTrainerV1:
    def __init__(self, config):
        self.config = config
        self.core = PolicyGradientTrainer(config)
        v1 = config.trainer.v1
        self.parameter_sync_step = int(v1.get("parameter_sync_step", 1))
        self.buffer = ReplayBuffer(int(v1.get("max_off_policy_threshold", 0)), v1.get("replay_strategy", "fifo"),
                                   int(v1.get("max_incomplete_group_refill_rounds", 3)))
        self.global_steps = 0
        self.weight_version = 0
        self._uid = 0
        self.rollout = self.core.rollout
        self.client = WholeSampleRetryClient(self._generate_rows, lambda: self.weight_version,
                                             max_attempts=int(v1.get("max_retry_attempts", 50)),
                                             wait_s=float(v1.get("retry_wait_s", 0.0)))
        self.total_steps = self.core.total_steps
        self._gen_lock = None
        self.on_init_end()

    # ------------------------------------------------------------------ hooks
    def on_init_end(self):
        pass

    def on_train_begin(self):
        pass

    def on_train_end(self):
        pass

    def on_step_begin(self):
        pass

    def on_sample_begin(self):
        pass

    def on_sample_end(self):
        pass

    def on_step_end(self):
        pass

    # ------------------------------------------------------------------ generation
    def _generate_rows(self, batch: DataProto) -> DataProto:
        """Generation of already-expanded samples (used by the retry client, one attempt)."""
        with (self._gen_lock if self._gen_lock is not None else contextlib.nullcontext()):
            return self._generate_rows_locked(batch)

    def _generate_rows_locked(self, batch: DataProto) -> DataProto:
        out = self.rollout.generate(batch, seed=1000003 * (self.weight_version + 1) + self._uid,
                                    global_step=self.weight_version)
        if len(out):
            scores, _ = self.core.reward_fn(out)
            out.batch["rm_scores"] = scores.to(out.batch["latents"].device)
        out.non_tensor_batch.update({k: v[: len(out)] for k, v in batch.non_tensor_batch.items()})
        return out

    def _prompt_ids(self, num_prompts: int) -> list[int]:
        ids = []
        while len(ids) < num_prompts:
            ids += self.core.local_prompt_ids(self.core.sampler.next_batch())
        return ids[:num_prompts]

    def generate_prompts(self, num_prompts: int) -> int:
        """Generate ``num_prompts`` groups of ``n`` samples into the replay buffer (blocking)."""
        core = self.core
        ids = self._prompt_ids(num_prompts)
        cond = core.encode_prompts(core.dataset.get_batch(ids))
        uids = []
        for _ in ids:
            self._uid += 1
            uids.append(f"g{self._uid}")
        cond.non_tensor_batch["uid"] = np.array(uids, dtype=object)
        for u in uids:
            self.buffer.register(u, core.n, submit_step=self.global_steps)
        gen = cond.repeat(core.n, interleave=True)
        out, status, vmin, vmax = self.client.generate(gen)
        k = 0
        for i in range(len(gen)):
            uid = gen.non_tensor_batch["uid"][i]
            if status[i] == "finished":
                self.buffer.put(uid, out.select_idxs([k]), min_global_steps=int(vmin[i]), max_global_steps=int(vmax[i]))
                k += 1
            else:
                self.buffer.put(uid, None, status="failure", min_global_steps=int(vmin[i]),
                                max_global_steps=int(vmax[i]))
        return num_prompts

    # ------------------------------------------------------------------ training
    def _step_once(self) -> dict:
        core = self.core
        timer = M.PhaseTimer(core.device)
        self.on_sample_begin()
        with timer("sample"):
            batch, smetrics = self.buffer.sample(self.global_steps, core.prompts_per_rank,
                                                 refill_fn=self.generate_prompts)
        self.on_sample_end()
        self.global_steps += 1
        core.global_step = self.global_steps
        m = core.train_on(batch, batch.batch["rm_scores"], timer)
        m.update(smetrics)
        m.update(M.compute_timing_metrics_diffusion(timer.timing, len(batch)))
        m["training/global_step"] = self.global_steps
        m["training/weight_version"] = self.weight_version
        return m

    def step(self) -> dict:
        self.on_step_begin()
        t0 = time.perf_counter()
        m = {}
        for _ in range(self.parameter_sync_step):
            m = self._step_once()
        self.on_step_end()
        dt = time.perf_counter() - t0
        n = self.core.prompts_per_rank * self.core.n * self.parameter_sync_step * self.core.world
        m.update(M.compute_throughput_metrics_diffusion(dt, n, self.core.world))
        return m

    def fit(self, steps: Optional[int] = None, log_fn=None) -> list[dict]:
        steps = steps or self.total_steps
        self.on_train_begin()
        hist = []
        try:
            while self.global_steps < steps:
                m = self.step()
                hist.append(m)
                if log_fn is not None and self.core.rank == 0:
                    log_fn(m)
        finally:
            self.on_train_end()
        return hist


@register_diffusion_trainer("sync")
class PolicyGradientDiffusionTrainerV1Sync(PolicyGradientDiffusionTrainerV1):
    """Colocated rollout: generate exactly the sampled batch with the current weights."""

    def on_sample_begin(self):
        self.generate_prompts(self.core.prompts_per_rank)

    def on_step_end(self):
        self.core.rollout.update_weights(self.core.actor.engine.get_per_tensor_param())
        self.weight_version = self.global_steps
        if self.core.rollout_cfg.free_cache_engine:
            self.core.rollout.sleep()


@register_diffusion_trainer("separate_async")
class PolicyGradientDiffusionTrainerV1SeparateAsync(PolicyGradientDiffusionTrainerV1):
    """Standalone rollout replica on a background thread; periodic weight pushes; bounded staleness."""

    def __init__(self, config):
        super().__init__(config)
        core = self.core
        if core.prompts_per_rank * core.world != int(config.data.train_batch_size):
            raise ValueError("separate_async requires train_batch_size == ppo mini batch")
        # standalone replica: its own weight copy (a separate rollout pool in a multi-process deployment)
        module = copy.deepcopy(core.actor.module)
        for p in module.parameters():
            p.requires_grad_(False)
        self.rollout = DiTRolloutEngine(module, core.adapter, core.rollout_cfg, core.model_cfg, device=core.device,
                                        latent_shape=core.spec.latent_shape, decoder=core.rollout.decoder)
        v1 = config.trainer.v1
        self.partial_rollout = bool(v1.get("partial_rollout", False))
        self.warmup_batches = int(v1.get("warmup_batches", 0))
        self._requests: "queue.Queue[Optional[int]]" = queue.Queue()
        self._lock = threading.Lock()
        self._gen_lock = self._lock
        self.client.wait_s = max(self.client.wait_s, 0.01)
        self._stop = False
        self._errors: list = []
        self._stream = torch.cuda.Stream(device=core.device) if core.device.type == "cuda" else None
        self._thread = threading.Thread(target=self._worker, daemon=True)

    def _worker(self):
        ctx = torch.cuda.stream(self._stream) if self._stream is not None else None
        try:
            if ctx is not None:
                ctx.__enter__()
            while not self._stop:
                req = self._requests.get()
                if req is None:
                    break
                self.generate_prompts(req)
        except Exception as e:  # noqa: BLE001
            self._errors.append(e)
        finally:
            if ctx is not None:
                ctx.__exit__(None, None, None)

    def _enqueue(self, n: int) -> int:
        self._requests.put(n)
        return n

    def on_train_begin(self):
        self._thread.start()
        for _ in range(self.warmup_batches + 1):
            self._enqueue(self.core.prompts_per_rank)

    def on_sample_begin(self):
        if self._errors:
            raise RuntimeError("rollout worker failed") from self._errors[0]
        self._enqueue(self.core.prompts_per_rank)  # keep the pipeline one batch ahead

    def _step_once(self) -> dict:
        core = self.core
        timer = M.PhaseTimer(core.device)
        self.on_sample_begin()
        with timer("sample"):
            batch, smetrics = self.buffer.sample(self.global_steps, core.prompts_per_rank, refill_fn=self._enqueue)
        if self._stream is not None:
            torch.cuda.current_stream(core.device).wait_stream(self._stream)
        self.global_steps += 1
        core.global_step = self.global_steps
        m = core.train_on(batch, batch.batch["rm_scores"], timer)
        m.update(smetrics)
        m.update(M.compute_timing_metrics_diffusion(timer.timing, len(batch)))
        m["training/global_step"] = self.global_steps
        m["training/weight_version"] = self.weight_version
        return m

    def on_step_end(self):
        """Push weights to the standalone replica (abort in-flight work unless partial rollout)."""
        if not self.partial_rollout:
            self.rollout.abort()
        with self._lock:
            if self._stream is not None:
                self._stream.wait_stream(torch.cuda.current_stream(self.core.device))
            self.rollout.update_weights(self.core.actor.engine.get_per_tensor_param())
            self.weight_version = self.global_steps

    def on_train_end(self):
        self._stop = True
        self.rollout.abort()
        self._requests.put(None)
        if self._thread.is_alive():
            self._thread.join(timeout=600)
