"""Hugging Face weight import / export for the Qwen3-Omni MoE thinker's language model.

The thinker here fuses what the HF checkpoint keeps apart: one ``kv_proj`` [2 Hk hd, D] for ``k_proj`` /
``v_proj``, and every layer's experts stacked as ``w_gate_up`` [E, 2F, D] (gate rows, then up rows) and
``w_down`` [E, D, F].  Checkpoints come in two layouts and both load: the hub layout with one tensor per
expert (``mlp.experts.{e}.gate_proj`` / ``up_proj`` / ``down_proj``) and the fused layout of recent
transformers releases (``mlp.experts.gate_up_proj`` [E, 2F, D], ``mlp.experts.down_proj`` [E, D, F]).  Names
may carry the ``thinker.`` prefix of the full omni model and the ``model.`` prefix of the causal-LM wrapper.
Under expert parallelism each rank takes only its own experts' slices.

Export writes the hub layout with the ``thinker.`` prefix.  The audio and vision towers of this framework
are shape-compatible stand-ins, not the HF encoders, so their tensors are neither read nor written.

Counterpart of the reference's HF loading of ``Qwen3OmniMoeForConditionalGeneration``
(``verl_omni/workers/engine/fsdp/omni_impl.py:145-196``; names as in transformers'
``modeling_qwen3_omni_moe.py``).
"""

from __future__ import annotations

import os
import re
from typing import Optional

import torch

_LAYER = re.compile(r"^layers\.(\d+)\.(.+)$")
_PLAIN = {  # per-layer tensors that map one to one: HF suffix -> this module's suffix
    "input_layernorm.weight": "ln1",
    "post_attention_layernorm.weight": "ln2",
    "self_attn.q_proj.weight": "q_proj.weight",
    "self_attn.o_proj.weight": "o_proj.weight",
    "self_attn.q_norm.weight": "q_norm",
    "self_attn.k_norm.weight": "k_norm",
    "mlp.gate.weight": "router.weight",
}


def _text_key(k: str) -> Optional[str]:
    """The language-model part of an HF name without its wrapper prefixes, or None (towers, talker, ...)."""
    if k.startswith("thinker."):
        k = k[len("thinker."):]
    elif k.startswith(("talker.", "code2wav.")):
        return None
    if k.startswith("lm_head."):
        return k
    if k.startswith("model."):
        k = k[len("model."):]
    if k.startswith(("audio_tower.", "visual.")):
        return None
    return k


def thinker_from_hf(state: dict, module, layer_offset: int = 0) -> dict:
    """HF tensors -> ``{name in module: tensor}`` for a :class:`MoELLM` (or a pipeline stage whose first layer
    is global layer ``layer_offset``).  Tensors the module does not hold (other stages' layers, other EP
    ranks' experts) are left out."""
    cfg = module.cfg
    nl = len(module.layers)
    El = int(module.layers[0].w_gate_up.shape[0]) if nl else 0
    e0 = int(module.layers[0].e0) if nl else 0
    out: dict = {}
    kv: dict = {}
    per_expert: dict = {}
    holds = dict(module.named_parameters())
    for k0, t in state.items():
        k = _text_key(k0)
        if k is None:
            continue
        if k in ("embed_tokens.weight",) and "embed" in holds:
            out["embed"] = t
            continue
        if k == "norm.weight" and "norm" in holds:
            out["norm"] = t
            continue
        if k == "lm_head.weight" and "lm_head.weight" in holds:
            out["lm_head.weight"] = t
            continue
        m = _LAYER.match(k)
        if m is None:
            continue
        li = int(m.group(1)) - layer_offset
        if li < 0 or li >= nl:
            continue
        rest = m.group(2)
        pre = f"layers.{li}."
        if rest in _PLAIN:
            out[pre + _PLAIN[rest]] = t
        elif rest in ("self_attn.k_proj.weight", "self_attn.v_proj.weight"):
            kv.setdefault(li, {})[rest.split(".")[1]] = t
        elif rest == "mlp.experts.gate_up_proj":  # fused layout [E, 2F, D]
            out[pre + "w_gate_up"] = t[e0:e0 + El]
        elif rest == "mlp.experts.down_proj":  # fused layout [E, D, F]
            out[pre + "w_down"] = t[e0:e0 + El]
        else:
            me = re.match(r"^mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight$", rest)
            if me is not None:
                e = int(me.group(1)) - e0
                if 0 <= e < El:
                    per_expert.setdefault(li, {}).setdefault(e, {})[me.group(2)] = t
    for li, d in kv.items():
        if "k_proj" in d and "v_proj" in d:
            out[f"layers.{li}.kv_proj.weight"] = torch.cat([d["k_proj"], d["v_proj"]], 0)
    for li, experts in per_expert.items():
        if len(experts) != El or any(len(v) != 3 for v in experts.values()):
            raise KeyError(f"layer {li + layer_offset}: incomplete per-expert tensors "
                           f"({len(experts)} of {El} experts)")
        out[f"layers.{li}.w_gate_up"] = torch.stack(
            [torch.cat([experts[e]["gate_proj"], experts[e]["up_proj"]], 0) for e in range(El)])
        out[f"layers.{li}.w_down"] = torch.stack([experts[e]["down_proj"] for e in range(El)])
    return out


def thinker_to_hf(named: dict, module, layer_offset: int = 0) -> dict:
    """``{name in module: tensor}`` -> hub-layout HF names (``thinker.`` prefix, one tensor per expert)."""
    cfg = module.cfg
    hd = cfg.head_dim
    out: dict = {}
    inv = {v: k for k, v in _PLAIN.items()}
    for n, t in named.items():
        if n == "embed":
            out["thinker.model.embed_tokens.weight"] = t
        elif n == "norm":
            out["thinker.model.norm.weight"] = t
        elif n == "lm_head.weight":
            out["thinker.lm_head.weight"] = t
        else:
            m = re.match(r"^layers\.(\d+)\.(.+)$", n)
            if m is None:
                continue  # towers: not HF-shaped
            li = int(m.group(1)) + layer_offset
            rest = m.group(2)
            pre = f"thinker.model.layers.{li}."
            if rest in inv:
                out[pre + inv[rest]] = t
            elif rest == "kv_proj.weight":
                k, v = t.split(cfg.kv_heads * hd, 0)
                out[pre + "self_attn.k_proj.weight"], out[pre + "self_attn.v_proj.weight"] = k, v
            elif rest in ("w_gate_up", "w_down"):
                e0 = int(module.layers[int(m.group(1))].e0)
                for j in range(t.shape[0]):
                    ep = pre + f"mlp.experts.{e0 + j}."
                    if rest == "w_gate_up":
                        g, u = t[j].chunk(2, 0)
                        out[ep + "gate_proj.weight"], out[ep + "up_proj.weight"] = g, u
                    else:
                        out[ep + "down_proj.weight"] = t[j]
    return out


def load_thinker(module, path: str, strict: bool = True, layer_offset: int = 0) -> int:
    """Loads an HF checkpoint (a directory of ``*.safetensors`` files, or one file) into the thinker's
    language model; returns the number of tensors loaded.  ``strict``: every language-model parameter of
    ``module`` must be present."""
    from safetensors import safe_open

    files = [path] if path.endswith(".safetensors") else sorted(
        os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors files under {path}")
    state = {}
    for f in files:
        with safe_open(f, framework="pt") as h:
            for k in h.keys():
                if _text_key(k) is not None:
                    state[k] = h.get_tensor(k)
    ours = thinker_from_hf(state, module, layer_offset)
    params = dict(module.named_parameters())
    text = [n for n in params if not n.startswith(("audio_tower.", "visual."))]
    missing = [n for n in text if n not in ours]
    if strict and missing:
        raise KeyError(f"{len(missing)} language-model parameters missing from {path}: {missing[:5]}")
    with torch.no_grad():
        for n, t in ours.items():
            if n in params:
                if tuple(t.shape) != tuple(params[n].shape):
                    raise ValueError(f"{n}: checkpoint shape {tuple(t.shape)} != {tuple(params[n].shape)}")
                params[n].copy_(t.to(params[n].dtype))
    return len(ours)


def save_thinker(named: dict, module, directory: str, layer_offset: int = 0) -> str:
    """Hub-layout ``model.safetensors`` of the language model (bf16) under ``directory``."""
    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    state = {k: v.detach().to(torch.bfloat16).cpu().contiguous()
             for k, v in thinker_to_hf(named, module, layer_offset).items()}
    f = os.path.join(directory, "model.safetensors")
    save_file(state, f)
    return f
