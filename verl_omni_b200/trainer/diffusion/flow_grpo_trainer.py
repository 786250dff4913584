"""Synchronous on-policy diffusion RL trainer (FlowGRPO / DanceGRPO / MixGRPO / GRPO-Guard / Flow-DPPO).

One step, as in ``PolicyGradientRayTrainer.fit`` (``verl_omni/trainer/diffusion/ray_diffusion_trainer.py:1067-1361``):

  prompts -> repeat n (uid per prompt) -> rollout (SDE trajectories + log-probs) -> decode -> reward
  -> old log-probs (skipped in bypass mode) -> rollout correction -> reference means (KL)
  -> group advantage -> actor update (micro-batches x SDE steps) -> checkpoint -> weight sync -> metrics

Differences by design: ranks are plain processes (torchrun) instead of Ray actors; rollout runs
in-process on the same weights (the hybrid engine is the default and weight sync is zero-copy
when colocated); every rank owns whole prompt groups so advantages need only one all-gather of the
scalar rewards.
"""

from __future__ import annotations

import copy
import logging
import os
import time
import zlib
from typing import Optional

import numpy as np
import torch

from verl_omni_b200.models.registry import ArchSpec, get_arch
from verl_omni_b200.models.reward import LatentMLPReward, VAEDecoder, ViTScorer
from verl_omni_b200.parallel import dist as D
from verl_omni_b200.pipelines.model_base import DiffusionModelBase
from verl_omni_b200.trainer.config.algorithm import DiffusionAlgoConfig
from verl_omni_b200.trainer.diffusion import diffusion_algos as algos
from verl_omni_b200.trainer.diffusion.rollout_correction import (
    apply_bypass_mode_to_diffusion_batch, apply_rollout_correction_to_diffusion_batch,
    compute_rollout_corr_metrics_from_batch, rollout_correction_enabled)
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.utils.dataset import ResumableSampler, SyntheticPromptDataset
from verl_omni_b200.utils import metrics as M
from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig, DiffusionModelConfig, DiffusionRolloutConfig
from verl_omni_b200.workers.engine.diffusion_engine import PPODiffusionEngine
from verl_omni_b200.workers.reward.reward_manager import ModelScorer, VisualRewardManager
from verl_omni_b200.workers.rollout.dit_rollout import DiTRolloutEngine
from verl_omni_b200.workers.utils_losses import diffusion_loss

_log = logging.getLogger(__name__)


def build_multi_reward(subs: list, device, dtype, default=None):
    """``reward.sub_rewards`` -> a weighted multi-reward manager (reference ``reward_manager/multi.py``)."""
    from verl_omni_b200.workers.reward.reward_manager import (SCORERS, MultiVisualRewardManager,
                                                              build_model_scorer)

    model_kinds = ("pickscore", "hpsv3", "ocr", "unified_reward", "clap", "imagebind")
    entries = []
    for sub in subs:
        sub = dict(sub)
        kind = str(sub.get("scorer", sub.get("name")))
        name = str(sub.get("name", kind))
        if kind == "default" and default is not None:
            mgr = default[0]
        elif kind in model_kinds:
            mgr = VisualRewardManager(build_model_scorer(kind, device, dtype, **dict(sub.get("sizes", {}) or {})),
                                      name=name)
        elif kind in SCORERS:
            mgr = VisualRewardManager(SCORERS[kind], name=name, **dict(sub.get("kwargs", {}) or {}))
        else:
            raise KeyError(f"unknown reward scorer {kind!r}")
        entries.append((name, mgr, float(sub.get("weight", 1.0)), bool(sub.get("required", True))))
    return MultiVisualRewardManager(entries)


def load_pretrained(module, path) -> int:
    """``actor_rollout_ref.model.path``: ``random-init`` (or empty) keeps the random weights; a diffusers
    pipeline / transformer directory (or a safetensors file) loads through the diffusers name mapping."""
    if not path or str(path) in ("random-init", "null", "None"):
        return 0
    from verl_omni_b200.models import hf_io

    if not hf_io.supported(module):
        raise NotImplementedError(f"loading pretrained weights for the {getattr(module, 'family', '?')!r} family")
    return hf_io.load_diffusers(module, str(path))


class PolicyGradientTrainer:
    def __init__(self, config, *, arch: Optional[str] = None, device: Optional[torch.device] = None,
                 rollout_only: bool = False, dp_override: Optional[int] = None):
        """``rollout_only`` (a standalone rollout rank): the policy module, rollout engine, reward and prompt
        stream without optimizer state or collectives; ``dp_override`` sets the data-parallel size whose
        prompt shares this rank produces (the trainer ranks' count)."""
        self.config = config
        self.rollout_only = rollout_only
        di = D.info()
        self.device = device or di.device
        self.rank, self.world = D.rank(), D.world_size()
        arc = config.actor_rollout_ref
        self.actor_cfg = DiffusionActorConfig.from_cfg(arc.actor)
        self.rollout_cfg = DiffusionRolloutConfig.from_cfg(arc.rollout)
        self.model_cfg = DiffusionModelConfig.from_cfg(arc.model)
        self.algo_cfg = DiffusionAlgoConfig.from_cfg(config.algorithm)
        self.spec: ArchSpec = get_arch(arch or self.model_cfg.architecture or "tiny_dit")
        self.adapter = DiffusionModelBase.get(self.spec.adapter, self.model_cfg.algorithm)
        self.n = self.rollout_cfg.n
        # Ulysses sequence parallelism: groups of `sp` consecutive ranks share their samples (each rank
        # runs 1/sp of every sequence); data parallelism runs over the dp = world / sp groups
        self.sp = int(getattr(self.actor_cfg.fsdp_config, "ulysses_sequence_parallel_size", 1) or 1)
        if self.world % self.sp:
            raise ValueError(f"world size {self.world} not divisible by ulysses_sequence_parallel_size={self.sp}")
        self.dp, self.dp_rank = self.world // self.sp, self.rank // self.sp
        if dp_override is not None:
            self.dp, self.dp_rank = int(dp_override), 0
        self.sp_group = None
        if self.sp > 1:
            from verl_omni_b200.parallel.ulysses import make_sp_groups

            self.sp_group, self.dp_group = make_sp_groups(self.sp)
        gbs = int(config.data.train_batch_size)
        if gbs % self.dp:
            raise ValueError(f"data.train_batch_size={gbs} must be divisible by the data-parallel size {self.dp}")
        self.prompts_per_rank = gbs // self.dp
        self.global_step = 0
        self.total_steps = int(config.trainer.total_training_steps or 1)
        seed = int(self.actor_cfg.fsdp_config.seed)
        torch.manual_seed(seed)
        cuda = self.device.type == "cuda"
        # ---------------------------------------------------------------- models
        if cuda and self.spec.init_on_device:
            # multi-billion-parameter presets: built (and randomly initialised) on the device, no fp32 host copy
            # per rank; the engine then moves each parameter into its flat buffers and frees it one by one
            with torch.device(self.device):
                module = self.spec.build()
        else:
            module = self.spec.build()
        load_pretrained(module, self.model_cfg.path)
        if self.model_cfg.enable_gradient_checkpointing and hasattr(module, "gradient_checkpointing"):
            module.gradient_checkpointing = True
        module.to(self.device)
        self.lora = self.model_cfg.lora_rank > 0
        if self.lora:
            from verl_omni_b200.models.lora import inject_lora

            inject_lora(module, self.model_cfg.lora_rank, self.model_cfg.lora_alpha, self.model_cfg.target_modules,
                        self.model_cfg.exclude_modules, adapters=tuple(self.model_cfg.policy_state_adapters),
                        init=self.model_cfg.lora_init_weights)
        # with LoRA the reference policy is the base model (adapters disabled): no second copy
        ref_module = (copy.deepcopy(module) if (self.actor_cfg.use_kl_loss and not self.lora and not rollout_only)
                      else None)
        # the trainer's flat-buffer parameter set (a standalone rollout rank lays its push buffer out the same way)
        self.trainable_names = [n for n, p in module.named_parameters() if p.requires_grad]
        if self.sp_group is not None:
            module.sp_group = self.sp_group
            if ref_module is not None:
                ref_module.sp_group = self.sp_group
        T = self.rollout_cfg.pipeline.num_inference_steps
        seq = self.spec.sched_seq_len or int(np.prod(self.spec.latent_shape[-2:])) // 4
        self.scheduler = self.adapter.build_scheduler(T, image_seq_len=seq, device=self.device)
        self.actor = PPODiffusionEngine(module, self.adapter, self.scheduler, self.actor_cfg, self.model_cfg,
                                        device=self.device, total_steps=self.total_steps,
                                        trainable=not rollout_only)
        # on-policy distillation: a frozen teacher of the same family scores the rollout trajectories
        self.teacher = None
        dist_cfg = config.get("distillation", {}) or {}
        if bool(dist_cfg.get("enabled", dist_cfg.get("enable", False))) and not rollout_only:
            tcfg = (dist_cfg.get("teacher_models", {}) or {}).get("teacher_model", {}) or {}
            torch.manual_seed(int(tcfg.get("seed", 1234)))
            teacher_module = self.spec.build()
            load_pretrained(teacher_module, tcfg.get("model_path"))
            teacher_module.to(self.device)
            if self.sp_group is not None:
                teacher_module.sp_group = self.sp_group
            self.teacher = PPODiffusionEngine(teacher_module, self.adapter, self.scheduler, self.actor_cfg,
                                              self.model_cfg, device=self.device, trainable=False)
            torch.manual_seed(seed)
        self.ref = None
        if ref_module is not None:
            # ref.fsdp_config.param_offload (or the actor's): the frozen reference waits on the host between uses
            rfc = ((config.actor_rollout_ref.get("ref", {}) or {}).get("fsdp_config", {}) or {})
            ref_off = bool(rfc.get("param_offload", False)) or bool(self.actor_cfg.fsdp_config.param_offload)
            self.ref = PPODiffusionEngine(ref_module, self.adapter, self.scheduler, self.actor_cfg, self.model_cfg,
                                          device=self.device, trainable=False, param_offload=ref_off)
        dt = self.actor.engine.dtype
        self.text_encoder = None
        if self.spec.text_encoder is not None:
            torch.manual_seed(seed + 1)
            self.text_encoder = self.spec.text_encoder().to(self.device, dt).eval()
            for p in self.text_encoder.parameters():
                p.requires_grad_(False)
        # ---------------------------------------------------------------- reward + decoder
        torch.manual_seed(seed + 2)
        decoder = None
        if self.spec.reward == "mlp":
            scorer = ModelScorer(LatentMLPReward(self.spec.latent_shape[0]).to(self.device, dt), "final_latents",
                                 self.device)
        else:
            vae = VAEDecoder(self.spec.latent_shape[0]).to(self.device, dt)
            if cuda:
                vae = vae.to(memory_format=torch.channels_last)
            decoder = vae.decode_video if self.spec.reward == "vit_video" else vae
            scorer = ModelScorer(ViTScorer(image_size=self.spec.image_size).to(self.device, dt), "images", self.device)
        self.reward_fn = VisualRewardManager(scorer, name="score")
        subs = list(config.get("reward", {}).get("sub_rewards", []) or [])
        if subs:
            self.reward_fn = build_multi_reward(subs, self.device, dt, default=(self.reward_fn, "score"))
        self.rollout = DiTRolloutEngine(module, self.adapter, self.rollout_cfg, self.model_cfg, device=self.device,
                                        latent_shape=self.spec.latent_shape, decoder=decoder,
                                        sched_seq_len=self.spec.sched_seq_len)
        # optional agent-loop path: per-sample coroutines over a request-packing rollout server
        agent_cfg = config.actor_rollout_ref.rollout.get("agent", {}) or {}
        self.agent_manager = None
        if bool(agent_cfg.get("enable", False)):
            if self.sp > 1:
                raise NotImplementedError("agent-loop rollout with Ulysses sequence parallelism: every rank of a "
                                          "sequence-parallel group must run the same engine batches")
            from verl_omni_b200.workers.agent_loop import DiffusionAgentLoopManager
            from verl_omni_b200.workers.rollout.server import DiffusionRolloutServer

            self.rollout_server = DiffusionRolloutServer(self.rollout)
            self.agent_manager = DiffusionAgentLoopManager(
                self.rollout_server, config.actor_rollout_ref.rollout, self.reward_fn,
                cond_keys=tuple(self.adapter.cond_keys()), num_workers=int(agent_cfg.get("num_workers", 8)),
                default_agent_loop=str(agent_cfg.get("default_agent_loop", "diffusion_single_turn_agent")))
        # ---------------------------------------------------------------- data
        train_files = config.data.get("train_files", "synthetic")
        if train_files and str(train_files) != "synthetic":
            # parquet prompts (verl RLHF layout): precomputed conditioning columns, or text for the text encoder
            from verl_omni_b200.utils.datasets_parquet import ParquetPromptDataset

            self.dataset = ParquetPromptDataset(
                train_files, cond_keys=tuple(self.spec.cond_shapes),
                token_len=self.spec.prompt_len if self.spec.text_encoder else 0, vocab=self.spec.vocab,
                prompt_key=str(config.data.get("prompt_key", "prompt")),
                max_samples=int(config.data.get("train_max_samples", -1) or -1))
            n_prompts = len(self.dataset)
        else:
            n_prompts = int(config.data.get("synthetic", {}).get("num_prompts", 1024))
            self.dataset = SyntheticPromptDataset(n_prompts, seed=int(config.data.get("seed", 0) or 0),
                                                  token_len=self.spec.prompt_len if self.spec.text_encoder else 0,
                                                  vocab=self.spec.vocab, cond_shapes=self.spec.cond_shapes)
        self.sampler = ResumableSampler(n_prompts, gbs, seed=int(config.data.get("seed", 0) or 0),
                                        shuffle=bool(config.data.get("shuffle", True)))
        self.loss_fn = lambda model_output, data: diffusion_loss(self.actor_cfg, model_output, data)
        self.ckpt_dir = config.trainer.default_local_dir
        from verl_omni_b200.utils.mfu import DiffusionFlopsCounter

        self.flops_counter = DiffusionFlopsCounter(module, getattr(module, "family", ""))

    # ------------------------------------------------------------------ pieces
    @torch.no_grad()
    def encode_prompts(self, batch: DataProto) -> DataProto:
        dt = self.actor.engine.dtype
        t = {}
        if self.text_encoder is not None:
            t["prompt_embeds"] = self.text_encoder(batch.batch["input_ids"].to(self.device, non_blocking=True))
        for k in self.spec.cond_shapes:
            v = batch.batch[k].to(self.device, non_blocking=True)
            t[k] = v.to(dt) if v.is_floating_point() else v
        return DataProto(t, dict(batch.non_tensor_batch))

    def local_prompt_ids(self, global_ids: list[int]) -> list[int]:
        p = self.prompts_per_rank
        return global_ids[self.dp_rank * p:(self.dp_rank + 1) * p]

    def compute_advantage(self, scores: torch.Tensor, uid: np.ndarray, T: int) -> torch.Tensor:
        """Group-normalised advantage; global std needs every rank's scores (one small all-gather).  Ranks
        of one sequence-parallel group hold the same samples: one copy per data-parallel rank is kept."""
        all_scores = D.all_gather_object(scores.detach().float().cpu())[::self.sp]
        all_uid = D.all_gather_object(list(uid))[::self.sp]
        g_scores = torch.cat(all_scores)
        g_uid = np.concatenate([np.asarray(u, dtype=object) for u in all_uid])
        est = algos.get_diffusion_adv_estimator_fn(self.algo_cfg.adv_estimator)
        adv, _ = est(g_scores[:, None].expand(-1, T), g_uid, norm_adv_by_std_in_grpo=self.algo_cfg.norm_adv_by_std_in_grpo,
                     global_std=self.algo_cfg.global_std)
        B = scores.shape[0]
        return adv[self.dp_rank * B:(self.dp_rank + 1) * B]

    # ------------------------------------------------------------------ one step
    def generate(self, ids: list[int], *, rollout=None, seed_step: Optional[int] = None,
                 uid_prefix: Optional[str] = None) -> tuple[DataProto, torch.Tensor, dict]:
        """Rollout + decode + reward for this rank's prompt ids (``n`` samples each)."""
        rollout = rollout or self.rollout
        step = self.global_step if seed_step is None else seed_step
        prompts = self.dataset.get_batch(ids)
        cond = self.encode_prompts(prompts)
        pre = uid_prefix if uid_prefix is not None else str(step)
        cond.non_tensor_batch["uid"] = np.array([f"{pre}-{i}" for i in ids], dtype=object)
        gen = cond.repeat(self.n, interleave=True)
        base_seed = int(self.rollout_cfg.seed if self.rollout_cfg.seed is not None else 12345)
        seed = (base_seed + step - 1) * 9973 + self.dp_rank * 7 + (zlib.crc32(pre.encode()) & 0xFFFF) * 131
        if self.agent_manager is not None and rollout is self.rollout:
            # per-row seeds from the step seed and each row's global index (prompt id x n + sample)
            gen.meta_info.update({"global_steps": step, "rollout_seed": seed})
            gen.non_tensor_batch["_rollout_seed_global_idx"] = np.array(
                [int(i) * self.n + j for i in ids for j in range(self.n)], dtype=np.int64)
            out = self.agent_manager.generate_sequences(gen)
            scores = out.batch.pop("rm_scores")[:, 0]
            return out, scores.to(self.device), {"reward/score_mean": float(scores.mean())}
        out = rollout.generate(gen, seed=seed, global_step=step)
        out.non_tensor_batch.update({k: v[: len(out)] for k, v in gen.non_tensor_batch.items()})
        scores, rmetrics = self.reward_fn(out)
        return out, scores.to(self.device), rmetrics

    def train_on(self, out: DataProto, scores: torch.Tensor, timer: "M.PhaseTimer") -> dict:
        """old log-probs -> rollout correction -> reference means -> advantage -> actor update."""
        T = out.batch["step_index"].shape[1]
        with timer("old_log_prob"):
            if self.algo_cfg.rollout_correction.bypass_mode or self.actor_cfg.rollout_correction.bypass_mode:
                apply_bypass_mode_to_diffusion_batch(out)
            else:
                old = self.actor.infer_batch(out, keys=("log_probs",))
                out.batch["old_log_probs"] = old.batch["log_probs"]
        corr_metrics = compute_rollout_corr_metrics_from_batch(out, bypass_mode=self.algo_cfg.rollout_correction.bypass_mode)
        if rollout_correction_enabled(self.algo_cfg.rollout_correction) and not self.algo_cfg.rollout_correction.bypass_mode:
            out, m2 = apply_rollout_correction_to_diffusion_batch(out, self.algo_cfg.rollout_correction)
            corr_metrics.update(m2)
        if self.actor_cfg.use_kl_loss:
            with timer("ref"):
                if self.ref is not None:
                    r = self.ref.infer_batch(out, keys=("prev_sample_mean",))
                else:
                    from verl_omni_b200.models.lora import use_adapter

                    with use_adapter(self.actor.module, None):
                        r = self.actor.infer_batch(out, keys=("prev_sample_mean",))
                out.batch["ref_prev_sample_mean"] = r.batch["prev_sample_mean"]
        if self.teacher is not None:
            with timer("teacher"):
                fm = self.actor_cfg.distill_loss_mode == "distill_fm_mse"
                tm = self.teacher.infer_batch(out, keys=("prev_sample_mean", "noise_pred") if fm else
                                              ("prev_sample_mean",))
                out.batch["teacher_prev_sample_mean"] = tm.batch["prev_sample_mean"]
                if fm:
                    out.batch["teacher_noise_pred"] = tm.batch["noise_pred"]
        if self.actor_cfg.diffusion_loss.loss_mode in ("flow_dppo", "grpo_guard"):
            with timer("old_mean"):
                om = self.actor.infer_batch(out, keys=("prev_sample_mean",))
                out.batch["old_prev_sample_mean"] = om.batch["prev_sample_mean"]
        with timer("adv"):
            adv = self.compute_advantage(scores, out.non_tensor_batch["uid"], T).to(self.device)
            out.batch["advantages"] = adv
        train_metrics = {}
        with timer("update_actor"):
            for _ in range(self.actor_cfg.ppo_epochs):
                mini = max(1, int(self.actor_cfg.ppo_mini_batch_size) * self.n // self.dp)
                for s in range(0, len(out), mini):
                    train_metrics = self.actor.train_batch(out.select_idxs(slice(s, min(len(out), s + mini))),
                                                           self.loss_fn)
        metrics = dict(train_metrics)
        metrics.update(corr_metrics)
        metrics.update(M.compute_data_metrics_diffusion(scores, adv[:, 0], out.non_tensor_batch["uid"]))
        return metrics

    # ------------------------------------------------------------------ validation
    @torch.no_grad()
    def validate(self) -> dict:
        """Validation generations (reference ``_validate``, ``ray_diffusion_trainer.py:508-641``): a fixed
        prompt set (``data.val_num_prompts``, seeded apart from the training prompts), ``val_kwargs.n``
        samples each with the ``val_kwargs`` sampling settings (steps, noise level, seed), scored by the
        reward manager.  Returns ``val-core/<data_source>/reward/mean@n`` plus ``val-aux`` spread metrics, all
        reduced over the data-parallel ranks."""
        vk = self.config.actor_rollout_ref.rollout.get("val_kwargs", {}) or {}
        n = int(vk.get("n", 1))
        nval = int(self.config.data.get("val_num_prompts", 0) or 0) or max(self.dp, self.prompts_per_rank)
        if not hasattr(self, "_val_dataset"):
            self._val_dataset = SyntheticPromptDataset(
                nval, seed=int(self.config.data.get("seed", 0) or 0) + 7919,
                token_len=self.spec.prompt_len if self.spec.text_encoder else 0, vocab=self.spec.vocab,
                cond_shapes=self.spec.cond_shapes)
        per = -(-nval // self.dp)
        ids = list(range(self.dp_rank * per, min(nval, (self.dp_rank + 1) * per)))
        scores = torch.zeros(0, device=self.device)
        if ids:
            cond = self.encode_prompts(self._val_dataset.get_batch(ids))
            cond.non_tensor_batch["uid"] = np.array([f"val-{i}" for i in ids], dtype=object)
            gen = cond.repeat(n, interleave=True)
            algo = vk.get("algo", {}) or {}
            steps = (vk.get("pipeline", {}) or {}).get("num_inference_steps")
            out = self.rollout.generate(gen, seed=int(vk.get("seed", 42)), global_step=0, record_logprobs=False,
                                        window=(0, int(steps or self.rollout_cfg.pipeline.num_inference_steps)),
                                        noise_level=float(algo.get("noise_level", 0.0)),
                                        sde_type=algo.get("sde_type"), num_inference_steps=steps)
            out.non_tensor_batch.update({k: v[:len(out)] for k, v in gen.non_tensor_batch.items()})
            scores, _ = self.reward_fn(out)
            scores = scores.to(self.device).float()
        # mean / std / best-of-n over every rank's samples
        stats = torch.tensor([float(scores.sum()), float((scores ** 2).sum()), float(scores.numel()),
                              float(scores.view(-1, n).max(-1).values.sum()) if scores.numel() else 0.0],
                             dtype=torch.float64, device=self.device)
        if self.world > 1:
            D.all_reduce(stats)
        if self.sp > 1:
            stats /= self.sp  # the ranks of a sequence-parallel group score the same samples
        cnt = max(1.0, float(stats[2]))
        mean = float(stats[0]) / cnt
        var = max(0.0, float(stats[1]) / cnt - mean * mean)
        src = str(self.config.data.get("data_source", "synthetic"))
        return {f"val-core/{src}/reward/mean@{n}": mean, f"val-aux/{src}/reward/std@{n}": var ** 0.5,
                f"val-core/{src}/reward/best@{n}/mean": float(stats[3]) / max(1.0, cnt / n)}

    # ------------------------------------------------------------------ one step
    def step(self, global_ids: Optional[list[int]] = None) -> dict:
        self._check_ranks_alive()
        self.global_step += 1
        if getattr(self, "_profiler", None) is None:
            from verl_omni_b200.utils.profiler import StepProfiler

            self._profiler = StepProfiler(self.config.get("global_profiler"), self.rank)
        self._profiler.start(self.global_step)
        try:
            return self._step_body(global_ids)
        finally:
            self._profiler.stop(self.global_step)

    def _step_body(self, global_ids: Optional[list[int]] = None) -> dict:
        timer = M.PhaseTimer(self.device)
        t_start = time.perf_counter()
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        ids = self.local_prompt_ids(global_ids if global_ids is not None else self.sampler.next_batch())
        with timer("gen"):
            out, scores, rmetrics = self.generate(ids)
        metrics = {"training/global_step": self.global_step}
        metrics.update(self.train_on(out, scores, timer))
        with timer("update_weights"):
            self.rollout.update_weights(self.actor.engine.get_per_tensor_param())
        save_freq = int(self.config.trainer.save_freq)
        if save_freq > 0:
            esi = self._esi_close_to_expiration()
            if esi or self.global_step >= self.total_steps or self.global_step % save_freq == 0:
                if esi and self.rank == 0:
                    print("Force saving checkpoint: ESI instance expiration approaching.")
                with timer("save_checkpoint"):
                    self.save_checkpoint()
        step_time = time.perf_counter() - t_start
        self.max_steps_duration = max(getattr(self, "max_steps_duration", 0.0), step_time)
        metrics.update(rmetrics)
        metrics.update(M.compute_timing_metrics_diffusion(timer.timing, len(out)))
        metrics.update(M.compute_throughput_metrics_diffusion(step_time, len(out) * self.dp, self.world))
        metrics.update(self._mfu_metrics(out, timer.timing, step_time))
        return metrics

    def _mfu_metrics(self, out: DataProto, timing: dict, step_time: float) -> dict:
        """``perf/mfu/*`` from the architecture's FLOPs formula and the phase timings."""
        from verl_omni_b200.utils.mfu import step_mfu_metrics

        from verl_omni_b200.utils.mfu import token_counts

        image_tokens, text_tokens = token_counts(self.spec)
        gs = self.model_cfg.pipeline.guidance_scale
        cfg_passes = 2 if (gs is not None and gs > 1.0 and "negative_prompt_embeds" in out.batch) else 1
        bypass = self.algo_cfg.rollout_correction.bypass_mode or self.actor_cfg.rollout_correction.bypass_mode
        ref_passes = 1 if self.actor_cfg.use_kl_loss else 0
        try:
            return step_mfu_metrics(self.flops_counter, samples=len(out),
                                    rollout_steps=int(self.rollout_cfg.pipeline.num_inference_steps),
                                    train_steps=int(out.batch["step_index"].shape[1]), image_tokens=image_tokens,
                                    text_tokens=text_tokens, cfg_passes=cfg_passes, timing=timing,
                                    step_time=step_time, recompute_old=not bypass, ref_passes=ref_passes, sp=self.sp)
        except Exception:  # noqa: BLE001 - a missing config field must not break a training step
            return {}

    def _esi_close_to_expiration(self) -> bool:
        """Capacity-block expiration rule, agreed by every rank (one flag all-reduce, MAX)."""
        from verl_omni_b200.utils.failure import should_save_ckpt_esi

        flag = should_save_ckpt_esi(getattr(self, "max_steps_duration", 0.0),
                                    float(self.config.trainer.get("esi_redundant_time", 0) or 0))
        if self.world > 1:
            flag = D.all_reduce_max(1.0 if flag else 0.0, device=self.device) > 0
        return flag

    def _check_ranks_alive(self) -> None:
        """Host-side liveness check between steps (``trainer.heartbeat_timeout_s`` > 0 turns it on)."""
        timeout = float(self.config.trainer.get("heartbeat_timeout_s", 0) or 0)
        if timeout <= 0 or self.world <= 1:
            return
        if getattr(self, "_heartbeat", None) is None:
            from verl_omni_b200.utils.failure import HeartbeatMonitor

            port = int(os.environ.get("VERL_OMNI_HEARTBEAT_PORT", int(os.environ.get("MASTER_PORT", 29500)) + 17))
            self._heartbeat = HeartbeatMonitor(self.rank, self.world, os.environ.get("MASTER_ADDR", "127.0.0.1"),
                                               port, interval_s=min(1.0, timeout / 4), timeout_s=timeout)
        self._heartbeat.check()

    def fit(self, steps: Optional[int] = None, log_fn=None) -> list[dict]:
        steps = steps or self.total_steps
        if self.config.trainer.resume_mode == "auto":
            self.maybe_resume()
        hist = []
        test_freq = int(self.config.trainer.get("test_freq", -1) or -1)
        if self.config.trainer.get("val_before_train", False):
            v = self.validate()
            hist.append(dict(v, **{"training/global_step": self.global_step}))
            if log_fn is not None and self.rank == 0:
                log_fn(hist[-1])
        while self.global_step < steps:
            m = self.step()
            if test_freq > 0 and (self.global_step % test_freq == 0 or self.global_step >= steps):
                t0 = time.perf_counter()
                m.update(self.validate())
                m["timing_s/testing"] = time.perf_counter() - t0
            hist.append(m)
            if log_fn is not None and self.rank == 0:
                log_fn(m)
        return hist

    # ------------------------------------------------------------------ checkpoint / resume
    def save_checkpoint(self) -> str:
        """``{default_local_dir}/global_step_{N}/actor`` + ``data.pt`` + ``latest_checkpointed_iteration.txt``."""
        root = os.path.join(self.ckpt_dir, f"global_step_{self.global_step}")
        self.actor.engine.save_checkpoint(os.path.join(root, "actor"), self.global_step,
                                          tuple(self.actor_cfg.checkpoint.save_contents))
        if self.rank == 0:
            torch.save({"sampler": self.sampler.state_dict(), "global_step": self.global_step},
                       os.path.join(root, "data.pt"))
            with open(os.path.join(self.ckpt_dir, "latest_checkpointed_iteration.txt"), "w") as f:
                f.write(str(self.global_step))
            self._prune_checkpoints()
        D.barrier()
        return root

    def _prune_checkpoints(self) -> None:
        """``trainer.max_actor_ckpt_to_keep``: keep the newest K ``global_step_*`` directories."""
        keep = self.config.trainer.get("max_actor_ckpt_to_keep")
        if not keep or int(keep) <= 0:
            return
        import shutil

        steps = sorted(int(d.split("_")[-1]) for d in os.listdir(self.ckpt_dir)
                       if d.startswith("global_step_") and d.split("_")[-1].isdigit())
        for st in steps[:-int(keep)]:
            shutil.rmtree(os.path.join(self.ckpt_dir, f"global_step_{st}"), ignore_errors=True)

    def maybe_resume(self) -> bool:
        mode = self.config.trainer.resume_mode
        if mode == "disable":
            return False
        if mode == "resume_path" and self.config.trainer.resume_from_path:
            root = self.config.trainer.resume_from_path
        else:
            marker = os.path.join(self.ckpt_dir, "latest_checkpointed_iteration.txt")
            if not os.path.exists(marker):
                return False
            with open(marker) as f:
                root = os.path.join(self.ckpt_dir, f"global_step_{int(f.read().strip())}")
        self.actor.engine.load_checkpoint(os.path.join(root, "actor"),
                                          tuple(self.actor_cfg.checkpoint.load_contents))
        d = torch.load(os.path.join(root, "data.pt"), weights_only=False)
        self.sampler.load_state_dict(d["sampler"])
        self.global_step = int(d["global_step"])
        return True
