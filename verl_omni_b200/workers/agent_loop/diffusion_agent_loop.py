"""Diffusion agent loops: per-sample generation coroutines, the batch worker and the manager.

Behaviour follows the reference's ``verl_omni/agent_loop/diffusion_agent_loop.py:105-403`` and
``verl_omni/agent_loop/single_turn_agent_loop.py:65-125``:

* sampling parameters = rollout ``pipeline`` + ``algo`` config (+ ``val_kwargs`` overrides and a fixed
  seed when ``meta_info["validate"]``), ``logprobs`` from ``calculate_log_probs``;
* one seed per post-repeat row derived from ``meta_info["rollout_seed"]`` and the trainer-assigned
  global row index (``_rollout_seed_global_idx``) so worker splits and packing order never remap
  RNG state;
* one agent loop per sample, chosen by ``agent_name`` (default ``agent.default_agent_loop``),
  running concurrently; each sample's reward is computed as soon as it finishes (streamed into a
  batched scorer) and the outputs are collated into one :class:`DataProto` with ``rm_scores`` and
  per-sample metrics;
* prompt-side extra tensors are right-padded to ``max_prompt_embed_length``.

Here the "server" is the in-process :class:`DiffusionRolloutServer` (request packing onto the
tcgen05 DiT engine) instead of HTTP replicas, and the workers are coroutines on one event loop.
"""

from __future__ import annotations

import asyncio
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import numpy as np
import torch

from verl_omni_b200.pipelines.request_batch import DiffusionRequest, RolloutOutput
from verl_omni_b200.utils.async_batcher import AsyncBatcher
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.agent_loop.utils import maybe_per_rollout_seeds

_AGENT_LOOPS: dict[str, type] = {}


def register_agent_loop(name: str):
    def deco(cls):
        _AGENT_LOOPS[name] = cls
        cls.agent_name = name
        return cls

    return deco


def get_agent_loop_class(name: str) -> type:
    if name not in _AGENT_LOOPS:
        raise KeyError(f"agent loop {name!r} not registered; registered: {sorted(_AGENT_LOOPS)}")
    return _AGENT_LOOPS[name]


@dataclass
class AgentLoopMetrics:
    generate_sequences: float = 0.0
    compute_score: float = 0.0
    num_preempted: int = 0

    def model_dump(self) -> dict:
        return {"generate_sequences": self.generate_sequences, "compute_score": self.compute_score,
                "num_preempted": self.num_preempted}


@dataclass
class DiffusionAgentLoopOutput:
    """What one agent loop returns for one sample."""

    payload: dict[str, torch.Tensor]  # engine outputs for this sample (no batch dim)
    reward_score: Optional[float] = None
    num_turns: int = 1
    metrics: AgentLoopMetrics = field(default_factory=AgentLoopMetrics)
    extra_fields: dict[str, Any] = field(default_factory=dict)
    aborted: bool = False


class DiffusionAgentLoopBase:
    """One sample's generation; subclasses implement :meth:`run`."""

    agent_name = "base"

    def __init__(self, server, rollout_cfg, **kwargs):
        self.server = server
        self.rollout_cfg = rollout_cfg

    async def run(self, sampling_params: dict, **kwargs) -> DiffusionAgentLoopOutput:
        raise NotImplementedError


@register_agent_loop("diffusion_single_turn_agent")
class DiffusionSingleTurnAgentLoop(DiffusionAgentLoopBase):
    """Single request per sample: the prompt's conditioning tensors go straight to the server."""

    async def run(self, sampling_params: dict, *, cond: dict, request_id: str, global_step: int = 0,
                  **kwargs) -> DiffusionAgentLoopOutput:
        t0 = time.perf_counter()
        req = DiffusionRequest(request_id=request_id, cond=cond, sampling=dict(sampling_params),
                               seed=int(sampling_params.get("seed", 0)), global_step=int(global_step))
        res: RolloutOutput = await self.server.generate(req)
        m = AgentLoopMetrics(generate_sequences=time.perf_counter() - t0)
        return DiffusionAgentLoopOutput(payload=res.payload, metrics=m, aborted=res.aborted,
                                        extra_fields={"request_id": request_id, **{
                                            k: v for k, v in res.metadata.items() if k in ("sde_window",)}})


def sampling_params_from_config(rollout_cfg, validate: bool) -> dict:
    """pipeline + algo knobs of the rollout config (validation overrides from ``val_kwargs``)."""
    p, a = rollout_cfg.pipeline, rollout_cfg.algo
    sp = {"num_inference_steps": int(p.num_inference_steps), "guidance_scale": p.guidance_scale,
          "noise_level": float(a.noise_level), "sde_type": a.sde_type, "sde_window_size": a.sde_window_size,
          "sde_window_range": a.sde_window_range, "logprobs": bool(rollout_cfg.calculate_log_probs)}
    if validate:
        vk = rollout_cfg.get("val_kwargs", {}) if hasattr(rollout_cfg, "get") else {}
        for sect in ("pipeline", "algo"):
            for k, v in (vk.get(sect) or {}).items():
                sp[k] = v
        sp["seed"] = int(vk.get("seed", 42))
        sp["logprobs"] = False
    return sp


class DiffusionAgentLoopWorker:
    """Runs one agent loop per row of a (post-repeat) prompt batch and collates the results."""

    def __init__(self, server, rollout_cfg, reward_fn: Optional[Callable] = None, *, cond_keys: tuple[str, ...],
                 max_prompt_embed_length: Optional[int] = None, default_agent_loop: str = "diffusion_single_turn_agent",
                 reward_batch: int = 64):
        self.server = server
        self.rollout_cfg = rollout_cfg
        self.cond_keys = tuple(cond_keys)
        self.max_prompt_embed_length = max_prompt_embed_length
        self.default_agent_loop = default_agent_loop
        self.reward_fn = reward_fn
        self._reward = AsyncBatcher(self._score_batch, max_batch=reward_batch) if reward_fn is not None else None

    def _score_batch(self, items: list[DataProto]) -> list[tuple[float, dict]]:
        batch = DataProto.concat(items)
        scores, metrics = self.reward_fn(batch)
        scores = scores.detach().float().cpu().reshape(-1).tolist()
        return [(s, metrics) for s in scores]

    async def generate_sequences(self, batch: DataProto) -> DataProto:
        validate = bool(batch.meta_info.get("validate", False))
        sp = sampling_params_from_config(self.rollout_cfg, validate)
        seeds = None
        if not validate:
            gidx = batch.non_tensor_batch.get("_rollout_seed_global_idx")
            seeds = maybe_per_rollout_seeds(batch.meta_info, len(batch),
                                            None if gidx is None else np.asarray(gidx, dtype=np.int64).reshape(-1))
        names = batch.non_tensor_batch.get("agent_name")
        global_step = int(batch.meta_info.get("global_steps", 0))
        sp["window_seed"] = int(batch.meta_info.get("rollout_seed", 0) or 0)
        tasks = []
        for i in range(len(batch)):
            psp = dict(sp)
            if seeds is not None:
                psp["seed"] = seeds[i]
            elif "seed" not in psp:
                psp["seed"] = i
            cond = {k: batch.batch[k][i] for k in self.cond_keys if k in batch.batch}
            for k in list(batch.batch.keys()):
                if k.startswith("negative_") and k[len("negative_"):] in self.cond_keys:
                    cond[k] = batch.batch[k][i]
            name = str(names[i]) if names is not None else self.default_agent_loop
            loop = get_agent_loop_class(name)(self.server, self.rollout_cfg)
            rid = f"{global_step}-{i}"
            if "uid" in batch.non_tensor_batch:
                rid = f"{batch.non_tensor_batch['uid'][i]}-{i}"
            tasks.append(asyncio.create_task(self._run_one(loop, psp, cond, rid, global_step)))
        outs = await asyncio.gather(*tasks)
        return self._postprocess(outs, batch)

    async def _run_one(self, loop: DiffusionAgentLoopBase, sp: dict, cond: dict, rid: str,
                       global_step: int) -> DiffusionAgentLoopOutput:
        out = await loop.run(sp, cond=cond, request_id=rid, global_step=global_step)
        if self.max_prompt_embed_length:
            from verl_omni_b200.pipelines.request_batch import pad_prompt_extra_field

            for k in self.cond_keys:
                v = out.payload.get(k)
                if isinstance(v, torch.Tensor) and v.dim() >= 2:
                    out.payload[k] = pad_prompt_extra_field(k, v, self.max_prompt_embed_length)
        if self._reward is not None and out.reward_score is None and not out.aborted:
            t0 = time.perf_counter()
            one = DataProto({k: v.unsqueeze(0) for k, v in out.payload.items()})
            out.reward_score, info = await self._reward(one)
            out.metrics.compute_score = time.perf_counter() - t0
            out.extra_fields["reward_extra_info"] = {k: v for k, v in info.items() if isinstance(v, (int, float))}
        return out

    def _postprocess(self, outs: list[DiffusionAgentLoopOutput], inp: DataProto) -> DataProto:
        keys = [k for k in outs[0].payload.keys() if all(k in o.payload for o in outs)]
        tensors = {k: torch.stack([o.payload[k] for o in outs], 0) for k in keys}
        scores = [o.reward_score for o in outs]
        if all(s is not None for s in scores):
            tensors["rm_scores"] = torch.tensor(scores, dtype=torch.float32).unsqueeze(-1)
        non_tensor = dict(inp.non_tensor_batch)
        non_tensor["__num_turns__"] = np.array([o.num_turns for o in outs], dtype=np.int32)
        non_tensor["aborted"] = np.array([o.aborted for o in outs], dtype=bool)
        meta = {"metrics": [o.metrics.model_dump() for o in outs]}
        if "sde_window" in outs[0].extra_fields:
            meta["sde_window"] = outs[0].extra_fields["sde_window"]
        return DataProto(tensors, non_tensor, meta)


class DiffusionAgentLoopManager:
    """Splits a batch over ``num_workers`` agent-loop workers sharing one rollout server."""

    def __init__(self, server, rollout_cfg, reward_fn=None, *, cond_keys, num_workers: int = 8,
                 default_agent_loop: str = "diffusion_single_turn_agent", max_prompt_embed_length=None):
        self.server = server
        self.workers = [DiffusionAgentLoopWorker(server, rollout_cfg, reward_fn, cond_keys=cond_keys,
                                                 max_prompt_embed_length=max_prompt_embed_length,
                                                 default_agent_loop=default_agent_loop)
                        for _ in range(max(1, int(num_workers)))]

    async def generate_sequences_async(self, batch: DataProto) -> DataProto:
        n = len(batch)
        W = min(len(self.workers), n)
        bounds = [round(i * n / W) for i in range(W + 1)]
        parts = []
        for w in range(W):
            sub = batch.select_idxs(slice(bounds[w], bounds[w + 1]))
            sub.meta_info = dict(batch.meta_info)
            parts.append(self.workers[w].generate_sequences(sub))
        outs = await asyncio.gather(*parts)
        res = DataProto.concat(list(outs))
        res.meta_info["metrics"] = [m for o in outs for m in o.meta_info.get("metrics", [])]
        for k in ("sde_window",):
            if k in outs[0].meta_info:
                res.meta_info[k] = outs[0].meta_info[k]
        return res

    async def _run_and_stop(self, batch: DataProto) -> DataProto:
        try:
            return await self.generate_sequences_async(batch)
        finally:  # the drain tasks belong to this event loop: stop them before it closes
            await self.server.stop()
            for w in self.workers:
                if w._reward is not None:
                    await w._reward.stop()

    def generate_sequences(self, batch: DataProto) -> DataProto:
        """Synchronous entry for the trainer (one event loop per call)."""
        return asyncio.run(self._run_and_stop(batch))
