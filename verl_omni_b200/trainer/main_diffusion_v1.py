"""v1 entry point: ``python -m verl_omni_b200.trainer.main_diffusion_v1 trainer.v1.trainer_mode=sync|separate_async``.

Same role as ``verl_omni/trainer/main_diffusion_v1.py:32-147``: forces the replay-buffer data path
(``trainer.use_v1=true``) and picks the trainer by ``trainer.v1.trainer_mode``.
"""

from __future__ import annotations

import logging
import sys

from verl_omni_b200.parallel import dist as D
from verl_omni_b200.trainer.main_diffusion import run_diffusion
from verl_omni_b200.utils.config import apply_overrides, load_config


def main(argv=None) -> None:
    logging.basicConfig(level=logging.INFO)
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config("diffusion_trainer", argv)
    if cfg.trainer.get("use_v1", True) is False and "trainer.use_v1=false" in argv:
        run_diffusion(cfg)  # explicit opt-out falls back to the v0 trainer
    else:
        apply_overrides(cfg, ["trainer.use_v1=true"])
        run_diffusion(cfg)
    D.destroy()


if __name__ == "__main__":
    main()
