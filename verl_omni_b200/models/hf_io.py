"""Diffusers-format weight import / export for the DiT families.

The modules here fuse what diffusers keeps apart (one ``to_qkv`` [3D, D] instead of ``attn.to_q`` /
``to_k`` / ``to_v``; the patch-embedding convolution as a linear over (ph, pw, c)-ordered patches).  This
module maps between the two layouts, so a diffusers ``transformer/diffusion_pytorch_model.safetensors``
loads into the fused modules and a trained model exports back to a directory diffusers can load
(reference: ``verl_omni/workers/engine/fsdp/diffusers_impl.py:203-304`` loads through
``SD3Transformer2DModel.from_pretrained``; ``verl_omni/utils/fsdp_utils.py`` writes the HF layout).

Supported: the SD3 / SD3.5 MMDiT (``SD3Transformer2DModel`` parameter names, including the SD3.5
"MMDiT-X" ``attn2`` branch and the context-pre-only last block).
"""

from __future__ import annotations

import json
import os
from typing import Callable

import torch


def _split_rows(t: torch.Tensor, n: int) -> list[torch.Tensor]:
    return list(t.chunk(n, 0))


def _sd3_pairs(module) -> list[tuple[str, list[str], str]]:
    """(our name, diffusers names, kind): kind ``same`` (1:1), ``cat`` (rows concatenated in order),
    ``conv`` (patch-embedding convolution <-> linear over (ph, pw, c) patches)."""
    out = [("pos_embed_proj.weight", ["pos_embed.proj.weight"], "conv"),
           ("pos_embed_proj.bias", ["pos_embed.proj.bias"], "same")]
    for ours, theirs in (("time_embed", "time_text_embed.timestep_embedder"),
                         ("text_embed", "time_text_embed.text_embedder")):
        for lin in ("linear_1", "linear_2"):
            for p in ("weight", "bias"):
                out.append((f"{ours}.{lin}.{p}", [f"{theirs}.{lin}.{p}"], "same"))
    for p in ("weight", "bias"):
        out.append((f"context_embedder.{p}", [f"context_embedder.{p}"], "same"))
        out.append((f"norm_out_linear.{p}", [f"norm_out.linear.{p}"], "same"))
        out.append((f"proj_out.{p}", [f"proj_out.{p}"], "same"))
    for i, blk in enumerate(module.transformer_blocks):
        b, a = f"transformer_blocks.{i}", f"transformer_blocks.{i}.attn"
        lin = [("norm1_linear", f"{b}.norm1.linear"), ("norm1_context_linear", f"{b}.norm1_context.linear"),
               ("to_out", f"{a}.to_out.0"), ("ff_1", f"{b}.ff.net.0.proj"), ("ff_2", f"{b}.ff.net.2")]
        if not blk.cpo:
            lin += [("to_add_out", f"{a}.to_add_out"), ("ff_context_1", f"{b}.ff_context.net.0.proj"),
                    ("ff_context_2", f"{b}.ff_context.net.2")]
        if blk.dual:
            lin += [("attn2_out", f"{b}.attn2.to_out.0")]
        for ours, theirs in lin:
            for p in ("weight", "bias"):
                out.append((f"{b}.{ours}.{p}", [f"{theirs}.{p}"], "same"))
        fused = [("to_qkv", [f"{a}.to_q", f"{a}.to_k", f"{a}.to_v"]),
                 ("add_qkv", [f"{a}.add_q_proj", f"{a}.add_k_proj", f"{a}.add_v_proj"])]
        if blk.dual:
            fused.append(("attn2_qkv", [f"{b}.attn2.to_q", f"{b}.attn2.to_k", f"{b}.attn2.to_v"]))
        for ours, theirs in fused:
            for p in ("weight", "bias"):
                out.append((f"{b}.{ours}.{p}", [f"{t}.{p}" for t in theirs], "cat"))
        norms = [("norm_q", f"{a}.norm_q"), ("norm_k", f"{a}.norm_k"), ("norm_added_q", f"{a}.norm_added_q"),
                 ("norm_added_k", f"{a}.norm_added_k")]
        if blk.dual:
            norms += [("norm2_q", f"{b}.attn2.norm_q"), ("norm2_k", f"{b}.attn2.norm_k")]
        for ours, theirs in norms:
            out.append((f"{b}.{ours}.weight", [f"{theirs}.weight"], "same"))
    return out


def _sd3_config(module) -> dict:
    c = module.cfg
    return {"_class_name": "SD3Transformer2DModel", "sample_size": c.sample_size, "patch_size": c.patch_size,
            "in_channels": c.in_channels, "num_layers": c.depth, "attention_head_dim": c.hidden // c.heads,
            "num_attention_heads": c.heads, "joint_attention_dim": c.joint_attention_dim,
            "caption_projection_dim": c.hidden, "pooled_projection_dim": c.pooled_projection_dim,
            "out_channels": c.out_channels, "pos_embed_max_size": c.pos_embed_max_size,
            "dual_attention_layers": list(range(c.dual_attention_layers)),
            "qk_norm": "rms_norm" if c.qk_norm else None}


_FAMILIES: dict[str, tuple[Callable, Callable]] = {"sd3": (_sd3_pairs, _sd3_config)}


def supported(module) -> bool:
    return getattr(module, "family", None) in _FAMILIES


def to_diffusers_state(named: dict, module) -> dict:
    """Our parameter tensors (by our names) -> a diffusers state dict for ``module``'s family."""
    pairs, _ = _FAMILIES[module.family]
    out = {}
    p = module.cfg.patch_size
    C = module.cfg.in_channels
    for ours, theirs, kind in pairs(module):
        if ours not in named:
            continue
        t = named[ours]
        if kind == "same":
            out[theirs[0]] = t
        elif kind == "cat":
            for name, part in zip(theirs, _split_rows(t, len(theirs))):
                out[name] = part
        else:  # linear [D, (ph, pw, c)] -> conv [D, c, ph, pw]
            out[theirs[0]] = t.reshape(t.shape[0], p, p, C).permute(0, 3, 1, 2)
    return {k: v.contiguous() for k, v in out.items()}


def from_diffusers_state(state: dict, module) -> dict:
    """A diffusers state dict -> our parameter tensors by our names (missing entries are skipped)."""
    pairs, _ = _FAMILIES[module.family]
    out = {}
    for ours, theirs, kind in pairs(module):
        if not all(t in state for t in theirs):
            continue
        if kind == "same":
            out[ours] = state[theirs[0]]
        elif kind == "cat":
            out[ours] = torch.cat([state[t] for t in theirs], 0)
        else:
            w = state[theirs[0]]
            out[ours] = w.permute(0, 2, 3, 1).reshape(w.shape[0], -1)
    return out


def save_diffusers(named: dict, module, directory: str) -> None:
    """``directory/config.json`` + ``directory/diffusion_pytorch_model.safetensors`` in bf16."""
    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    state = {k: v.detach().to(torch.bfloat16).cpu() for k, v in to_diffusers_state(named, module).items()}
    save_file(state, os.path.join(directory, "diffusion_pytorch_model.safetensors"))
    _, cfg_fn = _FAMILIES[module.family]
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(cfg_fn(module), f, indent=2)


def load_diffusers(module, path: str, strict: bool = True) -> int:
    """Load a diffusers transformer directory (or its ``transformer/`` subfolder, or one safetensors file)
    into ``module``; returns the number of tensors loaded."""
    from safetensors.torch import load_file

    if os.path.isdir(os.path.join(path, "transformer")):
        path = os.path.join(path, "transformer")
    files = [path] if path.endswith(".safetensors") else sorted(
        os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
    state = {}
    for f in files:
        state.update(load_file(f))
    ours = from_diffusers_state(state, module)
    params = dict(module.named_parameters())
    missing = [n for n in params if n not in ours]
    if strict and missing:
        raise KeyError(f"{len(missing)} parameters missing from {path}: {missing[:5]}")
    with torch.no_grad():
        for n, t in ours.items():
            if n in params:
                params[n].copy_(t.to(params[n].dtype).view_as(params[n]))
    return len(ours)
