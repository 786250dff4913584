"""Reward managers and scorers (same package path as the reference's ``verl_omni/reward_loop``).

The implementations live in :mod:`verl_omni_b200.workers.reward.reward_manager`.
"""

from verl_omni_b200.workers.reward.reward_manager import *  # noqa: F401,F403
