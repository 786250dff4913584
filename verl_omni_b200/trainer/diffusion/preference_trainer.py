"""Direct-preference diffusion trainers: DiffusionNFT and Diffusion-DPO (online / offline).

Counterpart of ``DirectPreferenceRayTrainer`` (``verl_omni/trainer/diffusion/ray_diffusion_trainer.py:1364-1772``)
with the NFT and DPO engines (``verl_omni/workers/engine/fsdp/diffusers_impl.py:946-1256``):

* **DiffusionNFT** (forward process): rollout clean latents, group advantages -> ``reward_prob``
  (``DiffusionNFTLoss.prepare_actor_batch``); for every selected timestep ``t``:
  ``x_t = (1 - t) x_0 + t eps``; three predictions -- the old policy (``old`` LoRA adapter, or an EMA copy
  for full fine-tuning; no grad), the current policy (grad), the reference (adapters disabled / frozen
  copy; no grad) -- into ``DiffusionNFTLoss``.  The old policy is refreshed every
  ``old_policy_update_interval`` optimizer steps with the configured EMA decay schedule.
* **Diffusion-DPO**: online -- rollout ``n`` samples per prompt, score, keep the best/worst pair per
  prompt; offline -- (chosen, rejected) latent pairs from a dataset.  Pairs share a logit-normal
  timestep and noise; reference noise predictions are computed before the update; ``DPOLoss``.
"""

from __future__ import annotations

import copy
import math
import time
from typing import Optional

import numpy as np
import torch

from verl_omni_b200.models import lora as LR
from verl_omni_b200.pipelines.schedulers.flow_match_sde import FlowMatchSDEDiscreteScheduler
from verl_omni_b200.trainer.config.algorithm import old_policy_decay_at
from verl_omni_b200.trainer.diffusion import diffusion_algos as algos
from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
from verl_omni_b200.utils import metrics as M
from verl_omni_b200.utils.dataproto import DataProto


def logit_normal_timesteps(n: int, scheduler_timesteps: torch.Tensor, generator=None, mean: float = 0.0,
                           std: float = 1.0) -> torch.Tensor:
    """``u = sigmoid(N(mean, std))``, index ``u * len(timesteps)`` into the (shifted) training schedule."""
    u = torch.sigmoid(torch.randn(n, generator=generator) * std + mean)
    idx = (u * scheduler_timesteps.numel()).long().clamp_(0, scheduler_timesteps.numel() - 1)
    return scheduler_timesteps.cpu()[idx]


class DirectPreferenceTrainer(PolicyGradientTrainer):
    def __init__(self, config, **kw):
        super().__init__(config, **kw)
        self.mode = self.actor_cfg.diffusion_loss.loss_mode
        if self.mode not in ("diffusion_nft", "dpo"):
            raise ValueError(f"DirectPreferenceTrainer handles diffusion_nft / dpo, got {self.mode!r}")
        self.loss_obj = algos.get_diffusion_loss_fn(self.mode)
        self.old_module = None
        self.ref_module = None
        if self.mode == "diffusion_nft":
            if self.lora:
                LR.copy_adapter(self.actor.module, "default", "old")
            else:
                self.old_module = self._frozen_copy()
        if not self.lora:
            self.ref_module = self._frozen_copy()
        self.train_sched = FlowMatchSDEDiscreteScheduler(shift=self.scheduler.shift)
        self.opt_steps = 0

    def _frozen_copy(self):
        m = copy.deepcopy(self.actor.module)
        for p in m.parameters():
            p.requires_grad_(False)
        return m

    # ------------------------------------------------------------------ predictions
    def _predict(self, which: str, x, t, cond):
        module = self.actor.module
        if which == "current":
            return self.adapter.forward(module, x, t, cond)
        with torch.no_grad():
            if which == "old":
                if self.old_module is not None:
                    return self.adapter.forward(self.old_module, x, t, cond)
                with LR.use_adapter(module, "old"):
                    return self.adapter.forward(module, x, t, cond)
            if self.ref_module is not None:
                return self.adapter.forward(self.ref_module, x, t, cond)
            with LR.use_adapter(module, None):
                return self.adapter.forward(module, x, t, cond)

    def _cond(self, mb: DataProto):
        return {k: mb.batch[k].to(self.device) for k in self.adapter.cond_keys()}

    # ------------------------------------------------------------------ NFT
    def _nft_update(self, batch: DataProto) -> dict:
        eng = self.actor.engine
        eng.train_mode()
        eng.zero_grad()
        T = batch.batch["train_timesteps"].shape[1]
        mbs = self.actor._micro_batches(batch, self.actor_cfg.ppo_micro_batch_size_per_gpu)
        gas = len(mbs) * T
        ms = []
        for mb in mbs:
            x0 = mb.batch["latents_clean"].to(self.device).float()
            cond = self._cond(mb)
            for j in range(T):
                tt = mb.batch["train_timesteps"][:, j].to(self.device).float()
                t = (tt / 1000.0).view(-1, *([1] * (x0.ndim - 1)))
                xt = (1.0 - t) * x0 + t * torch.randn_like(x0)
                out = {"old_prediction": self._predict("old", xt, tt, cond).float(),
                       "forward_prediction": self._predict("current", xt, tt, cond).float(),
                       "ref_forward_prediction": self._predict("ref", xt, tt, cond).float(),
                       "x0": x0, "xt": xt, "t_expanded": t}
                res = self.loss_obj(config=self.actor_cfg, model_output=out,
                                    data={"reward_prob": mb.batch["reward_prob"][:, j].to(self.device)})
                (res.loss / gas).backward()
                ms.append(res.metrics)
        norm = eng.optimizer_step()
        self.opt_steps += 1
        if self.opt_steps % self.algo_cfg.old_policy_update_interval == 0:
            decay = old_policy_decay_at(self.algo_cfg.old_policy_decay_schedule, self.opt_steps,
                                        self.algo_cfg.old_policy_decay)
            self.update_old_policy(decay)
        out = {k: float(np.mean([float(m[k]) for m in ms])) for k in ms[0]}
        out["actor/grad_norm"] = float(norm.reshape(()))
        return out

    @torch.no_grad()
    def update_old_policy(self, decay: float) -> None:
        """``old <- decay * old + (1 - decay) * current`` (hard copy at decay 0)."""
        if self.old_module is None:
            LR.ema_update_adapter(self.actor.module, "default", "old", decay)
            return
        for po, pc in zip(self.old_module.parameters(), self.actor.module.parameters()):
            po.lerp_(pc.to(po.dtype), 1.0 - decay)

    # ------------------------------------------------------------------ DPO
    def _dpo_update(self, batch: DataProto) -> dict:
        """``batch`` rows are adjacent (chosen, rejected) pairs with ``latents_clean`` and conditioning."""
        eng = self.actor.engine
        x0 = batch.batch["latents_clean"].to(self.device).float()
        B = x0.shape[0]
        g = torch.Generator().manual_seed(self.global_step)
        pair_noise = torch.randn((B // 2,) + tuple(x0.shape[1:]), generator=g).to(self.device)
        noise = pair_noise.repeat_interleave(2, 0)
        tt = logit_normal_timesteps(B // 2, self.train_sched.timesteps, g).repeat_interleave(2).to(self.device)
        t = (tt / 1000.0).view(-1, *([1] * (x0.ndim - 1)))
        xt = (1.0 - t) * x0 + t * noise
        cond = self._cond(batch)
        with torch.no_grad():
            ref_pred = self._predict("ref", xt, tt, cond).float()
        eng.train_mode()
        eng.zero_grad()
        pred = self._predict("current", xt, tt, cond).float()
        res = self.loss_obj(config=self.actor_cfg,
                            model_output={"noise": noise, "latent": x0, "noise_pred": pred},
                            data={"ref_noise_pred": ref_pred, "sample_level_rewards": batch.batch["rm_scores"],
                                  "uid": batch.non_tensor_batch.get("uid")})
        res.loss.backward()
        norm = eng.optimizer_step()
        out = {k: float(v) for k, v in res.metrics.items()}
        out["actor/grad_norm"] = float(norm.reshape(()))
        return out

    # ------------------------------------------------------------------ step
    def step(self, global_ids: Optional[list[int]] = None, offline_batch: Optional[DataProto] = None) -> dict:
        self.global_step += 1
        timer = M.PhaseTimer(self.device)
        t0 = time.perf_counter()
        metrics = {"training/global_step": self.global_step}
        if offline_batch is not None:
            batch = offline_batch
        else:
            ids = self.local_prompt_ids(global_ids if global_ids is not None else self.sampler.next_batch())
            with timer("gen"):
                out, scores, rm = self.generate(ids)
            metrics.update(rm)
            out.batch["rm_scores"] = scores
            out.batch["latents_clean"] = out.batch["final_latents"].float()
            out.batch["train_timesteps"] = out.batch["timesteps"]
            cfg = _TrainerView(self)
            with timer("prepare"):
                batch = self.loss_obj.prepare_actor_batch(out, scores.float().cpu(), cfg)
        with timer("update_actor"):
            metrics.update(self._nft_update(batch) if self.mode == "diffusion_nft" else self._dpo_update(batch))
        with timer("update_weights"):
            self.rollout.update_weights(self.actor.engine.get_per_tensor_param())
        metrics.update(M.compute_timing_metrics_diffusion(timer.timing, len(batch)))
        metrics.update(M.compute_throughput_metrics_diffusion(time.perf_counter() - t0, len(batch) * self.world,
                                                              self.world))
        return metrics


class _TrainerView:
    """Exposes ``config.algorithm`` / ``config.actor_rollout_ref.actor`` as validated dataclasses."""

    def __init__(self, t: DirectPreferenceTrainer):
        self.algorithm = t.algo_cfg

        class _ARR:
            actor = t.actor_cfg

        self.actor_rollout_ref = _ARR


class OfflineDPODataset:
    """Synthetic offline preference pairs: ``(chosen, rejected)`` latents + conditioning per prompt.

    Stands in for ``OfflineDPODataset`` (``verl_omni/utils/dataset/offline_dpo_dataset.py:170-315``), which
    reads chosen/rejected latents and prompt embeddings from parquet; rows come out interleaved
    ``[chosen0, rejected0, chosen1, ...]`` with ``rm_scores`` 1 / 0.
    """

    def __init__(self, trainer: PolicyGradientTrainer, num_pairs: int = 64, seed: int = 0):
        self.t = trainer
        self.n = num_pairs
        self.seed = seed

    def get_batch(self, ids: list[int]) -> DataProto:
        t = self.t
        prompts = t.encode_prompts(t.dataset.get_batch(ids))
        g = torch.Generator().manual_seed(self.seed + sum(ids))
        lat = torch.randn((2 * len(ids),) + tuple(t.spec.latent_shape), generator=g)
        b = prompts.repeat(2, interleave=True)
        b.batch["latents_clean"] = lat.to(t.device)
        b.batch["rm_scores"] = torch.tensor([1.0, 0.0] * len(ids), device=t.device)
        b.non_tensor_batch["uid"] = np.repeat(np.array([f"p{i}" for i in ids], dtype=object), 2)
        return b
