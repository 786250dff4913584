"""Agent loops (same package path as the reference's ``verl_omni/agent_loop``).

The implementations live in :mod:`verl_omni_b200.workers.agent_loop`.
"""

from verl_omni_b200.workers.agent_loop import *  # noqa: F401,F403
from verl_omni_b200.workers.agent_loop.composite_agent_loop import CompositeAgentLoop  # noqa: F401
from verl_omni_b200.workers.agent_loop.tq_agent_loop import DiffusionAgentLoopWorkerTQ  # noqa: F401
from verl_omni_b200.workers.agent_loop.utils import derive_rollout_seed, maybe_per_rollout_seeds  # noqa: F401
