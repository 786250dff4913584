"""Base class for custom (non-diffusers) models trained through the diffusion trainer.

Behaviour of the reference's ``verl_omni/pipelines/non_diffusers_model_base.py:40-240`` (used there for
BAGEL): a model that is not a diffusers ``ModelMixin`` declares how to build it from a checkpoint
directory, which submodules are whole units for sharding / activation checkpointing
(``_no_split_modules``), and opts in to gradient checkpointing.  Here the engine packs the trainable
parameters into its flat buffers itself, so ``_no_split_modules`` only drives activation
checkpointing granularity; checkpoints are safetensors files plus a JSON config.
"""

from __future__ import annotations

import json
import os
from typing import Optional

import torch
import torch.nn as nn


class NonDiffusersModelBase(nn.Module):
    """Subclasses set ``config_class`` (a dataclass) and build their layers in ``__init__(config)``."""

    config_class = None
    _no_split_modules: tuple[str, ...] = ()
    supports_gradient_checkpointing: bool = False

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.gradient_checkpointing = False

    # ------------------------------------------------------------------ construction / IO
    @classmethod
    def from_config(cls, config) -> "NonDiffusersModelBase":
        return cls(config)

    @classmethod
    def from_pretrained(cls, path: str, *, torch_dtype: Optional[torch.dtype] = None, device="cpu",
                        strict: bool = True) -> "NonDiffusersModelBase":
        """``path`` holds ``config.json`` (the config dataclass fields) and ``model.safetensors`` or
        ``model.pt``; without weights the model is random-initialised (the offline default here)."""
        with open(os.path.join(path, "config.json")) as f:
            fields = json.load(f)
        config = cls.config_class(**fields) if cls.config_class is not None else fields
        model = cls(config)
        st = os.path.join(path, "model.safetensors")
        pt = os.path.join(path, "model.pt")
        if os.path.exists(st):
            from safetensors.torch import load_file

            model.load_state_dict(load_file(st), strict=strict)
        elif os.path.exists(pt):
            model.load_state_dict(torch.load(pt, map_location="cpu", weights_only=True), strict=strict)
        if torch_dtype is not None:
            model = model.to(dtype=torch_dtype)
        return model.to(device)

    def save_pretrained(self, path: str) -> None:
        from dataclasses import asdict, is_dataclass

        from safetensors.torch import save_file

        os.makedirs(path, exist_ok=True)
        cfg = asdict(self.config) if is_dataclass(self.config) else dict(self.config)
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(cfg, f, indent=2)
        save_file({k: v.detach().contiguous().cpu() for k, v in self.state_dict().items()},
                  os.path.join(path, "model.safetensors"))

    # ------------------------------------------------------------------ activation checkpointing
    def enable_gradient_checkpointing(self) -> None:
        if not self.supports_gradient_checkpointing:
            raise ValueError(f"{type(self).__name__} does not support gradient checkpointing")
        self.gradient_checkpointing = True

    def disable_gradient_checkpointing(self) -> None:
        self.gradient_checkpointing = False

    def no_split_module_instances(self) -> list[nn.Module]:
        """Module instances whose class name is listed in ``_no_split_modules``."""
        names = set(self._no_split_modules)
        return [m for m in self.modules() if type(m).__name__ in names]

    def maybe_checkpoint(self, module: nn.Module, *args):
        """Runs ``module(*args)`` under activation checkpointing when enabled and training."""
        if self.gradient_checkpointing and torch.is_grad_enabled():
            return torch.utils.checkpoint.checkpoint(module, *args, use_reentrant=False)
        return module(*args)
