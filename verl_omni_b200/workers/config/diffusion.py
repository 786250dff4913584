"""Worker-side configs for diffusion actor / rollout / model.

Field names and defaults follow ``verl_omni/workers/config/diffusion/actor.py:38-181``,
``rollout.py:37-225`` and ``model.py:38-211`` so that override paths written for the reference
(``actor_rollout_ref.actor.diffusion_loss.clip_ratio=...``) keep working.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from verl_omni_b200.trainer.config.algorithm import RolloutCorrectionConfig
from verl_omni_b200.utils.base_config import BaseConfig

VALID_LOSS_MODES = ("flow_grpo", "dance_grpo", "flow_dppo", "grpo_guard", "dpo", "diffusion_nft", "kl",
                    "distill_kl", "distill_fm_mse", "mix_grpo")


@dataclass
class DiffusionLossConfig(BaseConfig):
    loss_mode: str = "flow_grpo"
    clip_ratio: float = 1e-4
    adv_clip_max: float = 5.0
    mix_beta: float = 0.5
    ref_kl_coef: float = 0.0
    adaptive_weight_min: float = 1e-5
    dpo_beta: float = 2000.0
    kl_mask_threshold: float = 1e-5
    add_kl_coefficient: bool = True

    def __post_init__(self):
        if self.loss_mode not in VALID_LOSS_MODES:
            raise ValueError(f"Invalid diffusion loss_mode: {self.loss_mode}. Must be one of {VALID_LOSS_MODES}")


@dataclass
class OptimConfig(BaseConfig):
    optimizer: str = "AdamW"
    lr: float = 1e-6
    lr_warmup_steps_ratio: float = 0.0
    total_training_steps: int = -1
    weight_decay: float = 0.01
    lr_warmup_steps: int = -1
    betas: list = field(default_factory=lambda: [0.9, 0.999])
    eps: float = 1e-8
    clip_grad: float = 1.0
    min_lr_ratio: float = 0.0
    num_cycles: float = 0.5
    lr_scheduler_type: str = "constant"

    def __post_init__(self):
        if self.lr_scheduler_type not in ("constant", "cosine"):
            raise ValueError(f"lr_scheduler_type must be constant or cosine, got {self.lr_scheduler_type}")


@dataclass
class FSDPEngineConfig(BaseConfig):
    """Sharded-engine knobs.

    ``reshard_after_forward=False`` keeps the gathered bf16 weights resident between the
    forward and backward (and through rollout), sharding only fp32 master weights, grads and
    AdamW state: with 180 GB per GPU the replicated bf16 copy of even a 14B model (28 GB) fits,
    and it removes the per-block all-gather from the hot loop.
    """

    param_offload: bool = False
    optimizer_offload: bool = False
    reshard_after_forward: bool = False
    fsdp_size: int = -1
    model_dtype: str = "bfloat16"
    dtype: str = "bfloat16"
    seed: int = 42
    ulysses_sequence_parallel_size: int = 1
    forward_only: bool = False
    strategy: str = "fsdp2"
    fused_collectives: str = "auto"


@dataclass
class VeOmniEngineConfig(BaseConfig):
    """The VeOmni engine's layout knobs (reference ``VeOmniDiffusionEngineConfig``,
    ``trainer/config/diffusion/engine/diffusion_veomni.yaml``), read by the sharded engine when
    ``strategy == "veomni"``: ``fsdp_size`` ranks per dp_shard group, replicated across the rest."""

    fsdp_size: int = -1
    ulysses_parallel_size: int = 1
    expert_parallel_size: int = 1
    init_device: str = "cuda"
    reshard_after_forward: bool = False
    model_dtype: str = "bfloat16"
    mixed_precision: bool = True
    mixed_precision_param_dtype: str = "bfloat16"
    mixed_precision_reduce_dtype: str = "float32"


@dataclass
class CheckpointConfig(BaseConfig):
    save_contents: list = field(default_factory=lambda: ["model", "optimizer", "extra"])
    load_contents: list = field(default_factory=lambda: ["model", "optimizer", "extra"])
    async_save: bool = False


@dataclass
class DiffusionActorConfig(BaseConfig):
    strategy: str = "fsdp2"
    ppo_mini_batch_size: int = 256
    ppo_micro_batch_size_per_gpu: int = 8
    diffusion_loss: DiffusionLossConfig = field(default_factory=DiffusionLossConfig)
    loss_scale_factor: Optional[float] = None
    use_kl_loss: bool = False
    kl_loss_coef: float = 0.001
    use_distill_loss: bool = False
    distill_loss_mode: str = "distill_kl"
    distill_loss_coef: float = 1.0
    ppo_epochs: int = 1
    shuffle: bool = False
    data_loader_seed: int = 42
    grad_clip: float = 1.0
    rollout_n: int = 1
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    optim: OptimConfig = field(default_factory=OptimConfig)
    fsdp_config: FSDPEngineConfig = field(default_factory=FSDPEngineConfig)
    veomni_config: VeOmniEngineConfig = field(default_factory=VeOmniEngineConfig)
    rollout_correction: RolloutCorrectionConfig = field(default_factory=RolloutCorrectionConfig)
    global_batch_info: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.strategy not in ("fsdp", "fsdp2", "veomni", "b200"):
            raise ValueError(f"Unknown actor strategy: {self.strategy!r}")
        if self.distill_loss_mode not in ("distill_kl", "distill_fm_mse"):
            raise ValueError(f"Invalid distill_loss_mode: {self.distill_loss_mode}")
        if self.ppo_epochs < 1:
            raise ValueError("ppo_epochs must be >= 1")


@dataclass
class DiffusionRolloutAlgoConfig(BaseConfig):
    noise_level: float = 1.0
    sde_type: str = "sde"
    sde_window_size: Optional[int] = None
    sde_window_range: Optional[list] = None
    sde_contiguous: bool = True
    sample_strategy: str = "random"
    iters_per_group: int = 1
    sde_window_seed: int = 0

    def __post_init__(self):
        if self.sde_type not in ("sde", "cps", "dance_sde"):
            raise ValueError(f"Unknown sde_type {self.sde_type!r}")
        if self.sample_strategy not in ("random", "progressive"):
            raise ValueError(f"Unknown sample_strategy: {self.sample_strategy!r}")
        if self.sample_strategy == "progressive" and self.iters_per_group <= 0:
            raise ValueError(f"iters_per_group must be positive, got {self.iters_per_group}.")


@dataclass
class DiffusionPipelineConfig(BaseConfig):
    height: int = 512
    width: int = 512
    num_inference_steps: int = 10
    output_type: str = "image"
    true_cfg_scale: float = 1.0
    max_sequence_length: int = 512
    guidance_scale: Optional[float] = None
    num_frames: int = 1
    frame_rate: float = 24.0
    aspect_ratio: Optional[str] = None
    video_flow_shift: float = 12.0


@dataclass
class DiffusionRolloutConfig(BaseConfig):
    name: str = "b200"
    mode: str = "async"
    nnodes: int = 0
    n_gpus_per_node: int = 8
    n: int = 1
    seed: Optional[int] = None
    prompt_length: int = 512
    max_prompt_embed_length: Optional[int] = None
    dtype: str = "bfloat16"
    tensor_model_parallel_size: int = 1
    data_parallel_size: int = 1
    expert_parallel_size: int = 1
    pipeline_model_parallel_size: int = 1
    max_num_seqs: int = 1024
    step_execution: bool = False
    free_cache_engine: bool = True
    calculate_log_probs: bool = True
    log_prob_micro_batch_size_per_gpu: Optional[int] = None
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    max_new_tokens: int = 256
    pipeline: DiffusionPipelineConfig = field(default_factory=DiffusionPipelineConfig)
    algo: DiffusionRolloutAlgoConfig = field(default_factory=DiffusionRolloutAlgoConfig)

    def __post_init__(self):
        if self.pipeline_model_parallel_size > 1:
            raise NotImplementedError("rollout pipeline parallelism is not supported (same as the reference)")
        if self.n < 1:
            raise ValueError("rollout.n must be >= 1")


@dataclass
class DiffusionModelConfig(BaseConfig):
    path: str = "random-init"
    algorithm: str = "flow_grpo"
    architecture: Optional[str] = None
    enable_gradient_checkpointing: bool = False
    attn_backend: str = "b200_fmha"
    lora_rank: int = 0
    lora_alpha: int = 64
    lora_init_weights: str = "gaussian"
    target_modules: object = "all-linear"
    exclude_modules: object = None
    lora_adapter_path: Optional[str] = None
    policy_state_adapters: list = field(default_factory=lambda: ["default"])
    fsdp_layer_prefixes: list = field(default_factory=lambda: ["transformer_blocks."])
    model_kwargs: dict = field(default_factory=dict)
    pipeline: DiffusionPipelineConfig = field(default_factory=DiffusionPipelineConfig)
    algo: DiffusionRolloutAlgoConfig = field(default_factory=DiffusionRolloutAlgoConfig)
