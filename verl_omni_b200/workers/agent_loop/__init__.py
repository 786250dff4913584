"""Agent loops: per-sample generation coroutines over the in-process rollout server."""

from verl_omni_b200.workers.agent_loop.diffusion_agent_loop import (  # noqa: F401
    DiffusionAgentLoopBase, DiffusionAgentLoopManager, DiffusionAgentLoopOutput, DiffusionAgentLoopWorker,
    DiffusionSingleTurnAgentLoop, get_agent_loop_class, register_agent_loop, sampling_params_from_config)
