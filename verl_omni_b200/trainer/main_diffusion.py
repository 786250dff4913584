"""Diffusion RL entry point: ``python -m verl_omni_b200.trainer.main_diffusion key=value ...``.

Same override syntax and key paths as ``verl_omni/trainer/main_diffusion.py:54-66`` (Hydra
style); launch one process per GPU with ``torchrun`` (``--nproc-per-node N``) instead of Ray.
``trainer.use_v1=true`` routes to the v1 trainers (replay buffer; ``trainer.v1.trainer_mode`` =
``sync`` | ``separate_async``).
"""

from __future__ import annotations

import json
import logging
import sys

from verl_omni_b200.parallel import dist as D
from verl_omni_b200.utils.config import load_config


def run_diffusion(config) -> list[dict]:
    device = config.trainer.get("device", "cuda")
    D.init_distributed(device=device, timeout_s=int(config.actor_rollout_ref.nccl_timeout))
    if config.trainer.get("use_v1", False):
        from verl_omni_b200.trainer.diffusion.v1.trainer import build_v1_trainer

        trainer = build_v1_trainer(config)
    elif config.algorithm.get("trainer_type", "policy_gradient") == "direct_preference":
        from verl_omni_b200.trainer.diffusion.preference_trainer import DirectPreferenceTrainer

        trainer = DirectPreferenceTrainer(config)
    else:
        from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer

        trainer = PolicyGradientTrainer(config)

    def log(m):
        print(json.dumps({k: (round(v, 6) if isinstance(v, float) else v) for k, v in m.items()}), flush=True)

    hist = trainer.fit(log_fn=log if "console" in list(config.trainer.logger) else None)
    return hist


def main(argv=None) -> None:
    logging.basicConfig(level=logging.INFO)
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config("diffusion_trainer", argv)
    run_diffusion(cfg)
    D.destroy()


if __name__ == "__main__":
    main()
