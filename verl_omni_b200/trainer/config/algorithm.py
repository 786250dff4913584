"""Algorithm configs (parity with ``verl_omni/trainer/config/algorithm.py:29-81``)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from verl_omni_b200.utils.base_config import BaseConfig

OLD_POLICY_DECAY_SCHEDULES = ("copy", "linear_to_0_5", "delayed_linear_to_0_999")


@dataclass
class RolloutCorrectionConfig(BaseConfig):
    """Importance-sampling / rejection-sampling correction between rollout and trainer policies."""

    bypass_mode: bool = False
    loss_type: str = "ppo_clip"
    rollout_is: Optional[str] = None
    rollout_is_threshold: object = 2.0
    rollout_is_batch_normalize: bool = False
    rollout_rs: Optional[str] = None
    rollout_rs_threshold: object = None

    def __post_init__(self):
        if self.rollout_is is not None and self.rollout_is not in ("token", "sequence"):
            raise ValueError(f"rollout_is must be null, 'token' or 'sequence', got {self.rollout_is!r}")
        if self.loss_type != "ppo_clip":
            raise ValueError(f"Only loss_type='ppo_clip' is supported, got {self.loss_type!r}")


@dataclass
class DiffusionAlgoConfig(BaseConfig):
    trainer_type: str = "policy_gradient"
    sample_source: str = "online"
    adv_estimator: str = "flow_grpo"
    norm_adv_by_std_in_grpo: bool = True
    global_std: bool = True
    old_policy_decay_schedule: str = "copy"
    old_policy_decay: Optional[float] = None
    old_policy_update_interval: int = 1
    timestep_fraction: float = 1.0
    adv_mode: str = "continuous"
    paired_preference: bool = False
    rollout_correction: RolloutCorrectionConfig = field(default_factory=RolloutCorrectionConfig)

    def __post_init__(self):
        valid_adv_modes = {"continuous", "positive_only", "negative_only", "one_only", "binary"}
        if self.adv_mode not in valid_adv_modes:
            raise ValueError(f"Invalid adv_mode: {self.adv_mode}. Must be one of {sorted(valid_adv_modes)}")
        if self.old_policy_decay_schedule not in OLD_POLICY_DECAY_SCHEDULES:
            raise ValueError(f"Invalid old_policy_decay_schedule: {self.old_policy_decay_schedule}")
        if self.old_policy_decay is not None and not 0 <= self.old_policy_decay <= 1:
            raise ValueError(f"old_policy_decay must be in [0, 1], got {self.old_policy_decay}.")
        if self.old_policy_update_interval <= 0:
            raise ValueError("old_policy_update_interval must be positive")
        if not 0 < self.timestep_fraction <= 1:
            raise ValueError(f"timestep_fraction must be in (0, 1], got {self.timestep_fraction}.")
        if self.trainer_type not in ("policy_gradient", "direct_preference"):
            raise ValueError(f"Invalid trainer_type {self.trainer_type!r}")
        if self.sample_source not in ("online", "offline"):
            raise ValueError(f"Invalid sample_source {self.sample_source!r}")


@dataclass
class OmniAlgoConfig(BaseConfig):
    trainer_type: str = "direct_preference"
    sample_source: str = "offline"
    paired_preference: bool = True
    adv_estimator: str = "dpo"
    norm_adv_by_std_in_grpo: bool = True
    global_std: bool = True

    def __post_init__(self):
        if self.trainer_type not in {"policy_gradient", "direct_preference"}:
            raise ValueError(f"Invalid trainer_type: {self.trainer_type}")
        if self.sample_source not in {"online", "offline"}:
            raise ValueError(f"Invalid sample_source: {self.sample_source}")


# (warm-up steps, ramp per step, cap) for each DiffusionNFT old-policy EMA schedule
# (``verl_omni/trainer/diffusion/diffusion_trainer_utils.py:19-23``).
OLD_POLICY_DECAY_TABLE = {
    "copy": (0, 0.0, 0.0),
    "linear_to_0_5": (0, 0.001, 0.5),
    "delayed_linear_to_0_999": (75, 0.0075, 0.999),
}


def old_policy_decay_at(schedule: str, step: int, fixed: Optional[float] = None) -> float:
    """EMA decay ``d`` for ``old <- d*old + (1-d)*current`` at optimizer step ``step``.

    ``copy`` is a hard copy (d=0); the ramps hold 0 for the warm-up steps, then grow linearly
    to their cap.  A fixed ``old_policy_decay`` overrides the schedule.
    """
    if fixed is not None:
        return float(fixed)
    if schedule not in OLD_POLICY_DECAY_TABLE:
        raise ValueError(f"Unsupported old_policy_decay_schedule: {schedule}")
    warm, rate, cap = OLD_POLICY_DECAY_TABLE[schedule]
    return 0.0 if step < warm else min((step - warm) * rate, cap)
