"""LoRA adapters with named adapter slots (``default`` / ``old`` / disabled-as-reference).

Behaviour of ``verl_omni/workers/engine/lora_adapter_mixin.py:26-172`` and the PEFT export of
``verl_omni/utils/fsdp_utils.py:218-274``:

* ``inject_lora(module, rank, alpha, target_modules, exclude_modules)`` wraps matching
  :class:`~verl_omni_b200.models.layers.Linear` layers (``"all-linear"`` or a list of name suffixes);
  base weights are frozen, each adapter holds ``A [r, in]`` (gaussian init) and ``B [out, r]`` (zeros);
* the forward adds ``(x A^T B^T) * alpha / r`` for the active adapter; ``use_adapter(module, None)`` runs
  the base model (the frozen reference policy when LoRA is on);
* ``copy_adapter(src, dst)`` and ``ema_update_adapter(src, dst, decay)`` (``dst <- decay*dst + (1-decay)*src``)
  maintain the DiffusionNFT old-policy adapter;
* ``export_peft_adapter(module, path)`` writes ``adapter_config.json`` + ``adapter_model.safetensors`` with
  PEFT key names (``base_model.model.<name>.lora_A.weight``).

The low-rank path is two skinny GEMMs on the same tcgen05 GEMM as the base layer.
"""

from __future__ import annotations

import contextlib
import json
import math
import os
from typing import Iterable, Optional

import torch
import torch.nn as nn

from verl_omni_b200.models.layers import Linear
from verl_omni_b200.ops import linear as L


class LoRALinear(nn.Module):
    def __init__(self, base: Linear, rank: int, alpha: float, adapters: Iterable[str] = ("default",),
                 init: str = "gaussian"):
        super().__init__()
        self.base = base
        for p in base.parameters():
            p.requires_grad_(False)
        self.rank, self.alpha = rank, alpha
        self.scaling = alpha / rank
        self.lora_A = nn.ParameterDict()
        self.lora_B = nn.ParameterDict()
        for name in adapters:
            self.add_adapter(name, init)
        self.active: Optional[str] = "default" if "default" in self.lora_A else None

    def add_adapter(self, name: str, init: str = "gaussian") -> None:
        a = torch.empty(self.rank, self.base.in_features, device=self.base.weight.device)
        if init == "gaussian":
            nn.init.normal_(a, std=1.0 / self.rank)
        else:
            nn.init.kaiming_uniform_(a, a=math.sqrt(5))
        self.lora_A[name] = nn.Parameter(a)
        self.lora_B[name] = nn.Parameter(torch.zeros(self.base.out_features, self.rank, device=a.device))
        trainable = name == "default"
        self.lora_A[name].requires_grad_(trainable)
        self.lora_B[name].requires_grad_(trainable)

    @property
    def in_features(self):
        return self.base.in_features

    @property
    def out_features(self):
        return self.base.out_features

    @property
    def weight(self):
        return self.base.weight

    def forward(self, x, epilogue: str = "none", gate=None, res=None, S: int = 1):
        if self.active is None:
            return self.base(x, epilogue=epilogue, gate=gate, res=res, S=S)
        A, B = self.lora_A[self.active], self.lora_B[self.active]
        if L.lora_linear_native_ok(x, self.base.weight, A) and B.dtype == x.dtype:
            # low-rank term reduced inside the base GEMM, epilogue fused (ops/linear.py)
            return L.lora_linear(x, self.base.weight, self.base.bias, A, B, self.scaling, epilogue=epilogue,
                                 gate=gate, res=res, S=S)
        delta = L.linear(L.linear(x, A.to(x.dtype)), B.to(x.dtype)) * self.scaling
        if epilogue == "none":
            return self.base(x) + delta
        if epilogue == "gelu":
            pre = self.base(x) + delta
            return torch.nn.functional.gelu(pre, approximate="tanh")
        if epilogue == "gate_res":
            y = self.base(x) + delta
            Bsz = gate.shape[0]
            return res + (y.view(Bsz, S, -1) * gate[:, None]).view_as(res)
        raise ValueError(epilogue)


def _match(name: str, targets, excludes) -> bool:
    if excludes and any(name.endswith(e) or e in name.split(".") for e in excludes):
        return False
    if targets in (None, "all-linear"):
        return True
    if isinstance(targets, str):
        targets = [targets]
    return any(name.endswith(t) for t in targets)


def inject_lora(module: nn.Module, rank: int, alpha: float, target_modules="all-linear", exclude_modules=None,
                adapters: Iterable[str] = ("default",), init: str = "gaussian") -> list[str]:
    """Replace matching Linear layers by LoRALinear in place; freezes every non-LoRA parameter."""
    for p in module.parameters():
        p.requires_grad_(False)
    replaced = []
    for name, sub in list(module.named_modules()):
        for cname, child in list(sub.named_children()):
            full = f"{name}.{cname}" if name else cname
            if isinstance(child, Linear) and _match(full, target_modules, exclude_modules):
                setattr(sub, cname, LoRALinear(child, rank, alpha, adapters, init))
                replaced.append(full)
    return replaced


def lora_layers(module: nn.Module):
    for name, m in module.named_modules():
        if isinstance(m, LoRALinear):
            yield name, m


def set_active_adapter(module: nn.Module, name: Optional[str]) -> None:
    for _, m in lora_layers(module):
        m.active = name


@contextlib.contextmanager
def use_adapter(module: nn.Module, name: Optional[str]):
    """Temporarily switch every LoRA layer to adapter ``name`` (None = base model / reference)."""
    prev = [(m, m.active) for _, m in lora_layers(module)]
    set_active_adapter(module, name)
    try:
        yield
    finally:
        for m, a in prev:
            m.active = a


@torch.no_grad()
def copy_adapter(module: nn.Module, src: str = "default", dst: str = "old") -> None:
    for _, m in lora_layers(module):
        if dst not in m.lora_A:
            m.add_adapter(dst)
        m.lora_A[dst].copy_(m.lora_A[src])
        m.lora_B[dst].copy_(m.lora_B[src])


@torch.no_grad()
def ema_update_adapter(module: nn.Module, src: str = "default", dst: str = "old", decay: float = 0.0) -> None:
    """``dst <- decay * dst + (1 - decay) * src`` (torch ``lerp_(src, 1 - decay)``)."""
    for _, m in lora_layers(module):
        if dst not in m.lora_A:
            m.add_adapter(dst)
        m.lora_A[dst].lerp_(m.lora_A[src].to(m.lora_A[dst].dtype), 1.0 - decay)
        m.lora_B[dst].lerp_(m.lora_B[src].to(m.lora_B[dst].dtype), 1.0 - decay)


def lora_state_dict(module: nn.Module, adapter: str = "default", peft_keys: bool = True) -> dict:
    out = {}
    for name, m in lora_layers(module):
        pre = f"base_model.model.{name}" if peft_keys else name
        out[f"{pre}.lora_A.weight"] = m.lora_A[adapter].detach()
        out[f"{pre}.lora_B.weight"] = m.lora_B[adapter].detach()
    return out


def lora_checksum(module: nn.Module, adapter: str = "default") -> float:
    """Sum of all adapter weights (consistency check across rollout replicas)."""
    return float(sum(v.double().sum() for v in lora_state_dict(module, adapter, False).values()))


def export_peft_adapter(module: nn.Module, path: str, adapter: str = "default", base_model: str = "") -> None:
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    layers = list(lora_layers(module))
    if not layers:
        raise ValueError("module has no LoRA layers")
    r, alpha = layers[0][1].rank, layers[0][1].alpha
    cfg = {"peft_type": "LORA", "r": r, "lora_alpha": alpha, "target_modules": sorted({n.split(".")[-1] for n, _ in layers}),
           "lora_dropout": 0.0, "bias": "none", "base_model_name_or_path": base_model, "task_type": None}
    with open(os.path.join(path, "adapter_config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    save_file({k: v.float().contiguous().cpu() for k, v in lora_state_dict(module, adapter).items()},
              os.path.join(path, "adapter_model.safetensors"))


def load_peft_adapter(module: nn.Module, path: str, adapter: str = "default") -> int:
    from safetensors.torch import load_file

    sd = load_file(os.path.join(path, "adapter_model.safetensors"))
    n = 0
    with torch.no_grad():
        for name, m in lora_layers(module):
            ka, kb = f"base_model.model.{name}.lora_A.weight", f"base_model.model.{name}.lora_B.weight"
            if ka in sd:
                m.lora_A[adapter].copy_(sd[ka])
                m.lora_B[adapter].copy_(sd[kb])
                n += 1
    return n


def export_peft_from_checkpoint(actor_dir: str, out_dir: str, adapter: str = "default", lora_alpha: Optional[float] = None,
                                base_model: str = "") -> int:
    """PEFT adapter directory from a sharded engine checkpoint, without building the model (reference
    ``verl_omni/utils/fsdp_utils.py:218-274``, which gathers the LoRA tensors of FSDP shards).

    ``actor_dir`` holds ``model_world_size_{W}_rank_{r}.pt`` (each rank's slice of the flat master); the
    adapter's ``lora_A`` / ``lora_B`` tensors are re-assembled across ranks and written with PEFT keys
    (``base_model.model.<module>.lora_{A,B}.weight``) plus ``adapter_config.json``.  ``lora_alpha`` defaults
    to the rank (scaling 1) when the checkpoint does not record it.  Returns the number of adapted modules."""
    import re

    from safetensors.torch import save_file

    from verl_omni_b200.workers.engine.base import read_full_state

    state = read_full_state(actor_dir)
    pat = re.compile(rf"^(.*)\.lora_([AB])\.{re.escape(adapter)}$")
    tensors, mods, rank = {}, set(), None
    for name, full in state.items():
        m = pat.match(name)
        if not m:
            continue
        mod, ab = m.group(1), m.group(2)
        mods.add(mod)
        tensors[f"base_model.model.{mod}.lora_{ab}.weight"] = full.float().contiguous()
        if ab == "A":
            rank = full.shape[0]
    if not tensors:
        raise ValueError(f"checkpoint has no LoRA tensors for adapter {adapter!r}")
    os.makedirs(out_dir, exist_ok=True)
    cfg = {"peft_type": "LORA", "r": rank, "lora_alpha": float(lora_alpha if lora_alpha is not None else rank),
           "target_modules": sorted({m.split(".")[-1] for m in mods}), "lora_dropout": 0.0, "bias": "none",
           "base_model_name_or_path": base_model, "task_type": None}
    with open(os.path.join(out_dir, "adapter_config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    save_file(tensors, os.path.join(out_dir, "adapter_model.safetensors"))
    return len(mods)
