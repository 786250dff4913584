"""Composite agent loop: an autoregressive (LLM) stage feeding a diffusion stage.

Behaviour of the reference's ``verl_omni/agent_loop/composite_agent_loop.py:79-320``: the AR model
first continues the prompt (e.g. prompt rewriting / planning tokens) with sampled token log-probs,
the text conditioning of the DiT is computed from the AR output, the DiT generates, and the sample
carries both the AR response (``ar_response_ids``, ``ar_log_probs``) and the diffusion trajectory,
plus an optional AR reward handle.  Here both stages are in-process engines: the KV-cached MoE LLM
rollout (:class:`~verl_omni_b200.workers.rollout.llm_rollout.LLMRolloutEngine`) and the DiT rollout
server; ``encode_fn`` maps AR tokens to the DiT conditioning tensors.
"""

from __future__ import annotations

import asyncio
import time
from typing import Callable, Optional

import torch

from verl_omni_b200.pipelines.request_batch import DiffusionRequest
from verl_omni_b200.workers.agent_loop.diffusion_agent_loop import (AgentLoopMetrics, DiffusionAgentLoopBase,
                                                                     DiffusionAgentLoopOutput, register_agent_loop)


@register_agent_loop("composite_ar_dit_agent")
class CompositeAgentLoop(DiffusionAgentLoopBase):
    """``ar_engine``: an :class:`LLMRolloutEngine`; ``encode_fn(token_ids [1, L + T]) -> {cond key: [1, ...]}``."""

    ar_engine = None
    encode_fn: Optional[Callable[[torch.Tensor], dict]] = None
    ar_reward_fn: Optional[Callable[[torch.Tensor], float]] = None

    async def run(self, sampling_params: dict, *, cond: dict, request_id: str, global_step: int = 0,
                  **kwargs) -> DiffusionAgentLoopOutput:
        if self.ar_engine is None or self.encode_fn is None:
            raise RuntimeError("CompositeAgentLoop needs ar_engine and encode_fn (set on the class)")
        t0 = time.perf_counter()
        prompt_ids = cond["prompt_ids"].unsqueeze(0)
        seed = int(sampling_params.get("seed", 0))
        loop = asyncio.get_running_loop()
        from verl_omni_b200.utils.dataproto import DataProto

        ar = await loop.run_in_executor(None, lambda: self.ar_engine.generate(
            DataProto({"input_ids": prompt_ids}), seed=seed))
        toks, lps = ar.batch["responses"], ar.batch["rollout_log_probs"]
        t_ar = time.perf_counter() - t0
        dit_cond = self.encode_fn(torch.cat([prompt_ids.to(toks.device), toks], 1))
        req = DiffusionRequest(request_id=request_id, cond={k: v[0] for k, v in dit_cond.items()},
                               sampling=dict(sampling_params), seed=seed, global_step=int(global_step))
        res = await self.server.generate(req)
        payload = dict(res.payload)
        payload["ar_response_ids"] = toks[0]
        payload["ar_log_probs"] = lps[0].float()
        extra = {"request_id": request_id, "ar_time_s": t_ar}
        if self.ar_reward_fn is not None:
            extra["ar_reward"] = float(self.ar_reward_fn(toks[0]))
        m = AgentLoopMetrics(generate_sequences=time.perf_counter() - t0)
        return DiffusionAgentLoopOutput(payload=payload, metrics=m, aborted=res.aborted, num_turns=2,
                                        extra_fields=extra)
