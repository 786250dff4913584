"""Architecture presets: name -> (module factory, adapter arch, latent shape, conditioning spec)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional

import torch

from verl_omni_b200.models.dit import DiT, DiTConfig, TextEncoder
from verl_omni_b200.models.mmdit import MMDiT, MMDiTConfig


@dataclass
class ArchSpec:
    name: str
    adapter: str
    build: Callable[[], torch.nn.Module]
    latent_shape: tuple
    cond_shapes: dict  # key -> per-sample shape of random conditioning (embeddings)
    text_encoder: Optional[Callable[[], torch.nn.Module]] = None  # token-id prompts
    prompt_len: int = 16
    vocab: int = 1000
    reward: str = "vit"
    image_size: int = 512
    notes: str = ""
    sched_seq_len: Optional[int] = None  # token count that sets the dynamic shift (default: latent H x W / 4)
    # build straight on the training device (multi-billion-parameter presets): no fp32 host copy per rank
    init_on_device: bool = False


def _qwen_build(tiny: bool):
    from verl_omni_b200.models.qwen_image import QwenImageConfig, QwenImageDiT

    return QwenImageDiT(QwenImageConfig.tiny() if tiny else QwenImageConfig.qwen_image())


def _ltx2_build(tiny: bool):
    from verl_omni_b200.models.ltx2 import LTX2AVDiT, LTX2Config

    return LTX2AVDiT(LTX2Config.tiny() if tiny else LTX2Config.ltx2())


def _bagel_build(tiny: bool):
    from verl_omni_b200.models.bagel import BagelConfig, BagelMoT

    return BagelMoT(BagelConfig.tiny() if tiny else BagelConfig.bagel_7b_mot())


def _h3_build(tiny: bool):
    from verl_omni_b200.models.minimax_h3 import H3Config, MiniMaxH3DiT

    return MiniMaxH3DiT(H3Config.tiny() if tiny else H3Config.h3())


def _flux_build():
    from verl_omni_b200.models.flux import FluxConfig, FluxDiT

    return FluxDiT(FluxConfig.flux1_dev())


ARCHS: dict[str, ArchSpec] = {
    "tiny_dit": ArchSpec(
        "tiny_dit", "TinyDiT", lambda: DiT(DiTConfig.tiny_plumbing()), (4, 16, 16), {},
        text_encoder=lambda: TextEncoder(vocab=1000, dim=256, layers=2, heads=4), prompt_len=16, vocab=1000,
        reward="mlp", notes="4 blocks, hidden 256, 4 heads, patch 2; 2-layer text encoder (vocab 1000, hidden 256)"),
    "sd35_medium": ArchSpec(
        "sd35_medium", "SD3MMDiT", lambda: MMDiT(MMDiTConfig.sd35_medium()), (16, 64, 64),
        {"prompt_embeds": (333, 4096), "pooled_prompt_embeds": (2048,)}, reward="vit", image_size=512,
        notes="24 joint blocks, hidden 1536, 24 heads, patch 2, 16-ch latents; 256 T5 + 77 CLIP tokens"),
    "sd35_small": ArchSpec(
        "sd35_small", "SD3MMDiT", lambda: MMDiT(MMDiTConfig.small()), (16, 32, 32),
        {"prompt_embeds": (77, 256), "pooled_prompt_embeds": (128,)}, reward="mlp", image_size=64,
        notes="2 joint blocks, hidden 256, 4 heads of 64, 256 image + 77 text tokens"),
    "sd35_tiny": ArchSpec(
        "sd35_tiny", "SD3MMDiT", lambda: MMDiT(MMDiTConfig.tiny()), (4, 8, 8),
        {"prompt_embeds": (12, 48), "pooled_prompt_embeds": (32,)}, reward="mlp", image_size=64),
    "flux1_dev": ArchSpec(
        "flux1_dev", "FluxDiT", _flux_build, (16, 128, 128),
        {"prompt_embeds": (512, 4096), "pooled_prompt_embeds": (768,)}, reward="vit", image_size=1024,
        init_on_device=True),
    "flux_tiny": ArchSpec(
        "flux_tiny", "FluxDiT", lambda: __import__("verl_omni_b200.models.flux", fromlist=["x"]).FluxDiT(
            __import__("verl_omni_b200.models.flux", fromlist=["x"]).FluxConfig.tiny()), (4, 8, 8),
        {"prompt_embeds": (12, 48), "pooled_prompt_embeds": (32,)}, reward="mlp", image_size=64),
    "qwen_image": ArchSpec(
        "qwen_image", "QwenImage", lambda: _qwen_build(False), (16, 128, 128),
        {"prompt_embeds": (512, 3584), "prompt_embeds_mask": (512,)}, reward="vit", image_size=1024,
        notes="60 joint blocks, hidden 3072, 24 heads x 128, 2x2-packed 16-ch latents, Qwen2.5-VL 3584-d text",
        init_on_device=True),
    "qwen_image_tiny": ArchSpec(
        "qwen_image_tiny", "QwenImage", lambda: _qwen_build(True), (4, 8, 8),
        {"prompt_embeds": (12, 48), "prompt_embeds_mask": (12,)}, reward="mlp", image_size=64),
    "qwen_image_edit": ArchSpec(
        "qwen_image_edit", "QwenImageEdit", lambda: _qwen_build(False), (16, 128, 128),
        {"prompt_embeds": (512, 3584), "prompt_embeds_mask": (512,), "image_latents": (16, 128, 128)},
        reward="vit", image_size=1024, notes="Qwen-Image-Edit: reference-image latents appended to the image tokens",
        init_on_device=True),
    "qwen_image_edit_tiny": ArchSpec(
        "qwen_image_edit_tiny", "QwenImageEdit", lambda: _qwen_build(True), (4, 8, 8),
        {"prompt_embeds": (12, 48), "prompt_embeds_mask": (12,), "image_latents": (4, 8, 8)}, reward="mlp",
        image_size=64),
    "ltx2": ArchSpec(
        "ltx2", "LTX2", lambda: _ltx2_build(False), (16 * 16 * 24 + 126, 128),
        {"prompt_embeds": (256, 3840), "audio_prompt_embeds": (256, 3840)}, reward="mlp", image_size=512,
        sched_seq_len=16 * 16 * 24,
        notes="joint audio-video: 48 layers, video 4096 / 32 heads, audio 2048 / 32 heads, 6144 video + 126 audio "
              "tokens of 128 channels (121 frames at 512 x 768)", init_on_device=True),
    "ltx2_tiny": ArchSpec(
        "ltx2_tiny", "LTX2", lambda: _ltx2_build(True), (2 * 4 * 4 + 16, 16),
        {"prompt_embeds": (12, 48), "audio_prompt_embeds": (12, 48)}, reward="mlp", image_size=64, sched_seq_len=32),
    "bagel_7b_mot": ArchSpec(
        "bagel_7b_mot", "Bagel", lambda: _bagel_build(False), (16, 64, 64), {"prompt_ids": (64,)}, vocab=152064,
        reward="vit", image_size=512,
        notes="Mixture-of-Transformers: Qwen2.5-7B-shaped layers with understanding / generation weight sets, "
              "1024 latent tokens (16-ch VAE latents, 2x2 packed) after a 64-token prompt", init_on_device=True),
    "bagel_tiny": ArchSpec(
        "bagel_tiny", "Bagel", lambda: _bagel_build(True), (4, 8, 8), {"prompt_ids": (12,)}, vocab=512, reward="mlp",
        image_size=64),
    "minimax_h3": ArchSpec(
        "minimax_h3", "MiniMaxH3", lambda: _h3_build(False), (32, (8 * 30 * 52 * 96 + 256 * 32) // 32),
        {"prompt_embeds": (256, 4096)}, reward="mlp", image_size=480, sched_seq_len=8 * 30 * 52,
        notes="single-stream text/audio/video DiT: 40 layers, hidden 3072, 24 heads; 12480 video rows of 96 + "
              "256 audio rows of 32 packed into one flat latent (stored as [32, n/32])", init_on_device=True),
    "minimax_h3_tiny": ArchSpec(
        "minimax_h3_tiny", "MiniMaxH3", lambda: _h3_build(True), (32, (32 * 96 + 8 * 32) // 32),
        {"prompt_embeds": (12, 48)}, reward="mlp", image_size=64, sched_seq_len=32),
    "wan_tiny": ArchSpec(
        "wan_tiny", "WanDiT", lambda: DiT(DiTConfig(in_channels=4, out_channels=4, hidden=128, heads=2, depth=2,
                                                    ffn=256, text_dim=48)), (4, 3, 8, 8),
        {"prompt_embeds": (12, 48)}, reward="mlp", image_size=64),
    "wan21_14b": ArchSpec(
        "wan21_14b", "WanDiT", lambda: DiT(DiTConfig.wan21_14b()), (16, 21, 60, 104),
        {"prompt_embeds": (512, 4096)}, reward="vit_video", image_size=480, init_on_device=True),
}


def get_arch(name: str) -> ArchSpec:
    if name not in ARCHS:
        raise KeyError(f"unknown architecture {name!r}; known: {sorted(ARCHS)}")
    return ARCHS[name]


def count_params(m: torch.nn.Module) -> int:
    return sum(p.numel() for p in m.parameters())
