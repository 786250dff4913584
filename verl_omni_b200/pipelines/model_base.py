"""Model adapters: (architecture, algorithm) -> how a DiT is called and stepped.

Mirrors the registry/dispatch contract of ``verl_omni/pipelines/model_base.py:28-257``
(``DiffusionModelBase.register(arch, algorithm)``, ``build_scheduler``,
``prepare_model_inputs``, ``forward_and_sample_previous_step``, ``forward``) for the model
families implemented in ``verl_omni_b200.models``:

* ``TinyDiT``  : cross-attention DiT + 2-layer text encoder (token-id prompts)
* ``SD3MMDiT`` : SD3.5-shaped MMDiT, prompt = (joint CLIP+T5 embeds, pooled CLIP embed)
* ``FluxDiT``  : FLUX.1-shaped double/single-stream DiT with 2D RoPE and guidance embedding
* ``WanDiT``   : Wan2.1-shaped video DiT with 3D RoPE

The same adapter serves the rollout loop and the trainer's log-prob recompute, so both run
identical kernels on identical inputs (bit-identical log-probs for bypass mode).
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from verl_omni_b200.pipelines.schedulers.flow_match_sde import FlowMatchSDEDiscreteScheduler, build_scheduler

_REGISTRY: dict[tuple[str, str], type] = {}

# the reference keys its adapters by the diffusers / transformers pipeline class (``model_index.json``
# ``_class_name``); those names select the same adapters here (reference ``pipelines/*/__init__.py``
# registrations: ``("StableDiffusion3Pipeline", "flow_grpo")`` and so on)
PIPELINE_CLASS_ALIASES = {
    "StableDiffusion3Pipeline": "SD3MMDiT",
    "FluxPipeline": "FluxDiT",
    "QwenImagePipeline": "QwenImage",
    "QwenImageEditPlusPipeline": "QwenImageEdit",
    "QwenImageEditPipeline": "QwenImageEdit",
    "WanPipeline": "WanDiT",
    "LTX2Pipeline": "LTX2",
    "MiniMaxH3Pipeline": "MiniMaxH3",
    "OmniBagelForConditionalGeneration": "Bagel",
}


class DiffusionModelBase:
    """Adapter base; subclasses are stateless (classmethods), selected by (architecture, algorithm)."""

    scheduler_kind = "sd3"
    latent_key = "latents"

    @classmethod
    def register(cls, arch: str, algorithm: str | tuple = "flow_grpo"):
        algos = (algorithm,) if isinstance(algorithm, str) else tuple(algorithm)

        def deco(sub):
            for a in algos:
                _REGISTRY[(arch, a)] = sub
            return sub

        return deco

    @classmethod
    def get(cls, arch: str, algorithm: str) -> type:
        arch = PIPELINE_CLASS_ALIASES.get(arch, arch)
        if (arch, algorithm) in _REGISTRY:
            return _REGISTRY[(arch, algorithm)]
        if (arch, "flow_grpo") in _REGISTRY and algorithm in ("dance_grpo", "mix_grpo", "flow_dppo", "grpo_guard",
                                                             "diffusion_nft", "dpo", "distill_kl"):
            return _REGISTRY[(arch, "flow_grpo")]
        raise KeyError(f"no adapter registered for ({arch!r}, {algorithm!r}); known: {sorted(_REGISTRY)}")

    # -------------------------------------------------------------- schedule
    @classmethod
    def build_scheduler(cls, num_inference_steps: int, image_seq_len: Optional[int] = None,
                        device=None) -> FlowMatchSDEDiscreteScheduler:
        return build_scheduler(cls.scheduler_kind, num_inference_steps, image_seq_len=image_seq_len, device=device)

    # -------------------------------------------------------------- model call
    @classmethod
    def cond_keys(cls) -> tuple:
        """Per-sample conditioning tensors carried from rollout to training."""
        raise NotImplementedError

    @classmethod
    def forward(cls, module, latents: torch.Tensor, timesteps: torch.Tensor, cond: dict) -> torch.Tensor:
        raise NotImplementedError

    # Qwen-Image-style "true CFG": rescale the guided prediction to the conditional one's norm
    true_cfg_renorm = False

    @classmethod
    def predict(cls, module, latents, timesteps, cond: dict, neg_cond: Optional[dict] = None,
                guidance_scale: Optional[float] = None) -> torch.Tensor:
        """Velocity prediction with optional classifier-free guidance (cond+uncond batched in one forward)."""
        if guidance_scale is not None and guidance_scale > 1.0 and neg_cond is not None:
            both = {k: torch.cat([cond[k], neg_cond[k]], 0) for k in cond}
            out = cls.forward(module, torch.cat([latents, latents], 0), torch.cat([timesteps, timesteps], 0), both)
            pos, neg = out.chunk(2, 0)
            from verl_omni_b200.ops.cfg import cfg_combine

            return cfg_combine(pos, neg, guidance_scale, renorm=cls.true_cfg_renorm)
        return cls.forward(module, latents, timesteps, cond)

    @classmethod
    def forward_and_sample_previous_step(cls, module, scheduler: FlowMatchSDEDiscreteScheduler, *,
                                         latents: torch.Tensor, prev_latents: torch.Tensor, step_index: torch.Tensor,
                                         cond: dict, neg_cond: Optional[dict], guidance_scale: Optional[float],
                                         noise_level: float, sde_type: str) -> dict:
        t = scheduler.timesteps.to(latents.device)[step_index.to(latents.device)]
        v = cls.predict(module, latents, t, cond, neg_cond, guidance_scale)
        out = scheduler.sample_previous_step(latents.float(), v.float(), step_index=step_index, noise_level=noise_level,
                                             prev_sample=prev_latents.float(), sde_type=sde_type, return_sqrt_dt=True)
        return {"log_probs": out.log_prob, "prev_sample_mean": out.prev_sample_mean, "std_dev_t": out.std_dev_t,
                "sqrt_dt": out.sqrt_dt, "noise_pred": v}


@DiffusionModelBase.register("TinyDiT", ("flow_grpo",))
class TinyDiTFlowGRPO(DiffusionModelBase):
    scheduler_kind = "tiny"

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds",)

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"])


@DiffusionModelBase.register("SD3MMDiT", ("flow_grpo",))
class SD3FlowGRPO(DiffusionModelBase):
    scheduler_kind = "sd3"

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds", "pooled_prompt_embeds")

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"], cond["pooled_prompt_embeds"])


@DiffusionModelBase.register("WanDiT", ("flow_grpo", "dance_grpo"))
class WanFlowGRPO(DiffusionModelBase):
    scheduler_kind = "wan"

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds",)

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"])


@DiffusionModelBase.register("FluxDiT", ("flow_grpo",))
class FluxFlowGRPO(DiffusionModelBase):
    scheduler_kind = "flux"

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds", "pooled_prompt_embeds")

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"], cond["pooled_prompt_embeds"])


@DiffusionModelBase.register("QwenImage", ("flow_grpo", "mix_grpo", "diffusion_nft", "dpo"))
class QwenImageFlowGRPO(DiffusionModelBase):
    """Qwen-Image (``verl_omni/pipelines/qwen_image_flow_grpo/diffusers_training_adapter.py:66``): dynamic
    shift from the image sequence length, true CFG with the guided prediction rescaled to the conditional
    one's norm (``qwen_image_flow_grpo/common.py:32-40``), right-padded prompts with a mask."""

    scheduler_kind = "qwen_image"
    true_cfg_renorm = True

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds", "prompt_embeds_mask")

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"], cond.get("prompt_embeds_mask"))


@DiffusionModelBase.register("QwenImageEdit", ("flow_grpo",))
class QwenImageEditFlowGRPO(QwenImageFlowGRPO):
    """Qwen-Image-Edit image-to-image (``verl_omni/pipelines/qwen_image_edit_flow_grpo/diffusers_training_adapter.py:31``):
    the reference image's latents ride along as conditioning and are appended to the image tokens."""

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds", "prompt_embeds_mask", "image_latents")

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"], cond.get("prompt_embeds_mask"),
                      image_latents=cond["image_latents"])


@DiffusionModelBase.register("LTX2", ("flow_grpo",))
class LTX2FlowGRPO(DiffusionModelBase):
    """LTX-2 joint audio-video (``verl_omni/pipelines/ltx2_flow_grpo/diffusers_training_adapter.py:33``): one
    packed latent sequence (video tokens, then audio tokens), separate video / audio prompt embeddings, the SDE
    step and log-probability over the concatenation.  The reference's clean-sample-space guidance
    (``ltx2_flow_grpo/common.py:69-80``) equals velocity-space CFG for a shared sample and sigma, so the
    common combine is used."""

    scheduler_kind = "ltx2"

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds", "audio_prompt_embeds")

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"], cond["audio_prompt_embeds"])


def bagel_combine_cfg(v: torch.Tensor, v_text: torch.Tensor, v_img: Optional[torch.Tensor], text_scale: float,
                      img_scale: float, renorm_type: str = "global", renorm_min: float = 0.0) -> torch.Tensor:
    """BAGEL's 3-branch guidance (``verl_omni/pipelines/bagel_flow_grpo/diffusers_training_adapter.py:216-270``):
    text guidance, then optional image guidance, then a norm rescale clamped to [renorm_min, 1] -- per sample
    over all positions ("global"), per token over channels ("channel"), or on the text-guided prediction only
    ("text_channel")."""
    if renorm_type == "text_channel":
        vt = v_text + text_scale * (v - v_text)
        scale = (v.norm(dim=1, keepdim=True) / (vt.norm(dim=1, keepdim=True) + 1e-8)).clamp(min=renorm_min, max=1.0)
        vt = vt * scale
        return v_img + img_scale * (vt - v_img) if (img_scale > 1.0 and v_img is not None) else vt
    vt = v_text + text_scale * (v - v_text)
    out = v_img + img_scale * (vt - v_img) if (img_scale > 1.0 and v_img is not None) else vt
    if renorm_type == "global":
        dims = tuple(range(1, v.ndim))
        n, n_ = torch.linalg.vector_norm(v, dim=dims, keepdim=True), torch.linalg.vector_norm(out, dim=dims, keepdim=True)
    elif renorm_type == "channel":
        n, n_ = v.norm(dim=1, keepdim=True), out.norm(dim=1, keepdim=True)
    else:
        raise NotImplementedError(f"cfg_renorm_type={renorm_type!r}")
    return out * (n / (n_ + 1e-8)).clamp(min=renorm_min, max=1.0)


@DiffusionModelBase.register("Bagel", ("flow_grpo",))
class BagelFlowGRPO(DiffusionModelBase):
    """BAGEL-7B-MoT text-to-image (``verl_omni/pipelines/bagel_flow_grpo/diffusers_training_adapter.py:44``):
    prompt token ids embedded by the model itself; guidance combines the conditional and text-unconditional
    branches with BAGEL's global renorm (the image-unconditional branch only matters for editing)."""

    scheduler_kind = "sd3"
    cfg_renorm_type = "global"
    cfg_renorm_min = 0.0

    @classmethod
    def cond_keys(cls):
        return ("prompt_ids",)

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_ids"])

    @classmethod
    def predict(cls, module, latents, timesteps, cond: dict, neg_cond: Optional[dict] = None,
                guidance_scale: Optional[float] = None) -> torch.Tensor:
        if guidance_scale is not None and guidance_scale > 1.0 and neg_cond is not None:
            both = {k: torch.cat([cond[k], neg_cond[k]], 0) for k in cond}
            out = cls.forward(module, torch.cat([latents, latents], 0), torch.cat([timesteps, timesteps], 0), both)
            v, v_text = out.chunk(2, 0)
            return bagel_combine_cfg(v, v_text, None, guidance_scale, 1.0, cls.cfg_renorm_type, cls.cfg_renorm_min)
        return cls.forward(module, latents, timesteps, cond)


@DiffusionModelBase.register("MiniMaxH3", ("diffusion_nft", "flow_grpo"))
class MiniMaxH3Adapter(DiffusionModelBase):
    """MiniMax-H3 audio-video (``verl_omni/pipelines/minimax_h3_diffusion_nft/diffusers_training_adapter.py:38``):
    packed flat video / audio rows, text prompt embeddings; DiffusionNFT is its objective in the reference
    (the reverse-SDE path is available here as well since the model returns flow-matching velocities)."""

    scheduler_kind = "flux"

    @classmethod
    def cond_keys(cls):
        return ("prompt_embeds",)

    @classmethod
    def forward(cls, module, latents, timesteps, cond):
        return module(latents, timesteps, cond["prompt_embeds"])
