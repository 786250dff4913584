"""Omni RL entry point: ``python -m verl_omni_b200.trainer.main_omni key=value ...``.

Counterpart of ``verl_omni/trainer/main_omni.py:57-360`` (Hydra config ``omni_trainer``): the config tree
``trainer/config/omni_trainer.yaml`` with the same override syntax; one process per GPU under ``torchrun``
instead of Ray workers.  ``actor_rollout_ref.actor.megatron.{tensor,expert,pipeline}_model_parallel_size`` set the
TP (attention heads + sequence, consecutive ranks), EP (experts sharded, consecutive ranks) and PP (layer
stages; stage s on ranks [s W / pp, (s + 1) W / pp)) sizes, ``actor_rollout_ref.rollout.tensor_model_parallel_size``
the rollout's (heads and KV caches split over groups of consecutive ranks);
checkpoints use the diffusion trainers' layout (``global_step_{N}/actor`` + expert slices) and resume with
``trainer.resume_mode=auto``.
"""

from __future__ import annotations

import json
import logging
import sys

import torch

from verl_omni_b200.parallel import dist as D
from verl_omni_b200.utils.config import load_config

ARCHS = {"qwen3_omni_30b_a3b": "qwen3_omni_30b_a3b", "qwen3_omni_tiny": "tiny"}


def build_omni_trainer(config):
    from verl_omni_b200.models.moe_llm import MoEConfig
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer
    from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig

    arc = config.actor_rollout_ref
    arch = str(arc.model.architecture)
    if arch not in ARCHS:
        raise KeyError(f"unknown omni architecture {arch!r}; known: {sorted(ARCHS)}")
    mcfg = getattr(MoEConfig, ARCHS[arch])()
    # optional depth override (full width, fewer layers): smoke runs of the full-width model on few GPUs
    nl = arc.model.get("num_layers", None) if hasattr(arc.model, "get") else None
    if nl:
        mcfg.layers = int(nl)
    act = arc.actor
    ac = DiffusionActorConfig()
    ac.grad_clip = float(act.grad_clip)
    for k in ("lr", "weight_decay", "eps", "clip_grad", "lr_warmup_steps", "lr_warmup_steps_ratio",
              "lr_scheduler_type"):
        setattr(ac.optim, k, act.optim[k])
    ac.optim.betas = list(act.optim.betas)
    ac.fsdp_config.dtype = str(act.fsdp_config.dtype)
    ac.fsdp_config.fused_collectives = str(act.fsdp_config.fused_collectives)
    ac.checkpoint.save_contents = list(act.checkpoint.save_contents)
    ac.checkpoint.load_contents = list(act.checkpoint.load_contents)
    W = D.world_size()
    tp = int(act.megatron.tensor_model_parallel_size)
    ep = int(act.megatron.expert_model_parallel_size)
    pp = int(act.megatron.pipeline_model_parallel_size)
    for name, n in (("tensor", tp), ("expert", ep), ("pipeline", pp)):
        if n < 1 or W % n:
            raise ValueError(f"{name}_model_parallel_size={n} must divide the world size {W}")
    tp_group = D.make_hsdp_groups(tp)[0] if tp > 1 else None
    rtp = int(arc.rollout.tensor_model_parallel_size)
    if rtp < 1 or W % rtp:
        raise ValueError(f"rollout.tensor_model_parallel_size={rtp} must divide the world size {W}")
    rollout_tp_group = D.make_hsdp_groups(rtp)[0] if rtp > 1 else None
    ep_group = D.make_hsdp_groups(ep)[0] if ep > 1 else None
    dp = W // tp // pp
    gbs = int(config.data.train_batch_size)
    if gbs % dp:
        raise ValueError(f"data.train_batch_size={gbs} must be divisible by the data-parallel size {dp}")
    device = torch.device("cuda", torch.cuda.current_device()) if config.trainer.device == "cuda" else \
        torch.device("cpu")
    ro = arc.rollout
    trainer = OmniGRPOTrainer(
        mcfg, ac, device=device, n=int(ro.n), prompt_text=int(config.data.prompt_text_tokens),
        audio_tokens=int(config.data.prompt_audio_tokens), image_tokens=int(config.data.prompt_image_tokens),
        response_len=int(ro.response_length), loss_mode=str(act.policy_loss.loss_mode), ep_group=ep_group,
        tp_group=tp_group, seed=int(config.data.seed), micro_batch_size=int(act.ppo_micro_batch_size_per_gpu),
        temperature=float(ro.temperature), kv_block_size=int(ro.kv_block_size),
        total_steps=int(config.trainer.total_training_steps), pp_size=pp, rollout_tp_group=rollout_tp_group,
        model_path=arc.model.get("path", None))
    trainer.prompts_per_rank = gbs // dp
    files = config.data.get("train_files", None)
    if files:
        from verl_omni_b200.utils.datasets_parquet import ParquetOmniRLDataset

        trainer.dataset = ParquetOmniRLDataset(files, vocab=mcfg.vocab,
                                               max_prompt_length=int(config.data.get("max_prompt_length", 512)),
                                               max_samples=int(config.data.get("train_max_samples", -1) or -1))
    return trainer


def run_omni(config) -> list[dict]:
    D.init_distributed(device=config.trainer.device, timeout_s=int(config.actor_rollout_ref.nccl_timeout))
    if config.algorithm.trainer_type not in ("policy_gradient", "direct_preference"):
        raise ValueError(f"unknown algorithm.trainer_type {config.algorithm.trainer_type!r}: policy_gradient "
                         "(online GRPO / GSPO) or direct_preference (offline DPO on parquet pairs)")
    trainer = build_omni_trainer(config)
    if config.algorithm.trainer_type == "direct_preference":
        return _run_dpo(config, trainer)
    ckpt = str(config.trainer.default_local_dir)
    if config.trainer.resume_mode == "auto":
        trainer.load_checkpoint(ckpt)
    save_freq = int(config.trainer.save_freq)
    total = int(config.trainer.total_training_steps)
    log = "console" in list(config.trainer.logger)
    hist = []
    while trainer.step_count < total:
        m = trainer.step(trainer.prompts_per_rank)
        hist.append(m)
        if log and D.rank() == 0:
            print(json.dumps({k: (round(v, 6) if isinstance(v, float) else v) for k, v in m.items()}), flush=True)
        if save_freq > 0 and (trainer.step_count % save_freq == 0 or trainer.step_count >= total):
            trainer.save_checkpoint(ckpt)
    return hist


def _run_dpo(config, trainer) -> list[dict]:
    """Offline omni DPO (reference ``OmniDirectPreferenceRayTrainer``, ``trainer/omni/ray_omni_trainer.py``):
    (chosen, rejected) response pairs from ``data.train_files`` (``prompt_ids`` / ``chosen_ids`` /
    ``rejected_ids``, optional prompt features) against a frozen reference copy of the initial policy;
    ``algorithm.dpo_beta``; checkpoints and resume as in the online trainer."""
    from verl_omni_b200.models.moe_llm import MoELLM
    from verl_omni_b200.utils.datasets_parquet import ParquetMLLMDPODataset

    files = config.data.get("train_files", None)
    if not files:
        raise ValueError("direct_preference needs data.train_files with prompt_ids / chosen_ids / rejected_ids")
    if trainer.pp is not None:
        raise ValueError("offline omni DPO runs without pipeline stages")
    trainer.dataset = None
    ds = ParquetMLLMDPODataset(files, max_samples=int(config.data.get("train_max_samples", -1) or -1))
    # the reference: an independent frozen copy of the initial policy (the same expert shard per rank), taken
    # before a resumed run loads its trained weights
    with torch.device(trainer.device):
        ref = MoELLM(trainer.cfg, trainer.model.ep)
    ref.load_state_dict({k: v.detach() for k, v in trainer.model.state_dict().items()})
    ref.to(next(trainer.model.parameters()).dtype).eval().requires_grad_(False)
    ckpt = str(config.trainer.default_local_dir)
    if config.trainer.resume_mode == "auto":
        trainer.load_checkpoint(ckpt)
    beta = float(config.algorithm.get("dpo_beta", 0.1))
    bs = trainer.prompts_per_rank
    save_freq, total = int(config.trainer.save_freq), int(config.trainer.total_training_steps)
    log = "console" in list(config.trainer.logger)
    hist = []
    while trainer.step_count < total:
        trainer.step_count += 1
        start = ((trainer.step_count - 1) * trainer.dp + trainer.dp_rank) * bs
        chosen, rejected = ds.get_pairs([(start + j) % len(ds) for j in range(bs)])
        m = trainer.dpo_step(chosen, rejected, ref, beta=beta)
        m.update({"training/global_step": trainer.step_count, "actor/lr": trainer.engine.lr(),
                  "actor/grad_norm": float(trainer.engine.last_grad_norm.reshape(()))})
        hist.append(m)
        if log and D.rank() == 0:
            print(json.dumps({k: (round(v, 6) if isinstance(v, float) else v) for k, v in m.items()}), flush=True)
        if save_freq > 0 and (trainer.step_count % save_freq == 0 or trainer.step_count >= total):
            trainer.save_checkpoint(ckpt)
    return hist


def main(argv=None) -> None:
    logging.basicConfig(level=logging.INFO)
    argv = list(sys.argv[1:] if argv is None else argv)
    cfg = load_config("omni_trainer", argv)
    run_omni(cfg)
    D.destroy()


if __name__ == "__main__":
    main()
