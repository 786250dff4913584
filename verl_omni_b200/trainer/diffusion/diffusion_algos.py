"""Advantage estimators and worker-side diffusion losses (registries + implementations).

Public surface and semantics follow ``verl_omni/trainer/diffusion/diffusion_algos.py``:

* ``register_diffusion_adv_est`` / ``get_diffusion_adv_estimator_fn`` (``:155-187``) and the
  GRPO group-normalised outcome advantage (``:190-265``) -- here vectorised with segment
  reductions instead of a per-sample Python loop;
* ``register_diffusion_loss`` / ``get_diffusion_loss_fn`` (``:129-145``) with the losses
  ``flow_grpo``/``dance_grpo`` (``:268-358``), ``flow_dppo`` (``:361-463``), ``grpo_guard``
  (``:466-587``), ``dpo`` (``:590-778``), ``diffusion_nft`` (``:781-1010``), ``kl``
  (``:1013-1051``), ``distill_kl`` (``:1054-1094``) and ``distill_fm_mse`` (``:1097-1132``).

``data`` passed to a loss is a plain ``dict`` (tensor and non-tensor entries) instead of a
TensorDict.  Per-sample policy-gradient terms are computed by ``ops.losses`` (one fused kernel on
CUDA for the ratio / clip / mask / reductions).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections import defaultdict
from dataclasses import dataclass
from enum import Enum
from typing import Any, Callable, Optional

import numpy as np
import torch
import torch.nn.functional as F

from verl_omni_b200.ops import losses as loss_ops
from verl_omni_b200.utils.dataproto import DataProto


@dataclass
class DiffusionLossResult:
    loss: torch.Tensor
    metrics: dict
    add_loss_metric: bool = False


def _keys_of(mapping: Any) -> str:
    try:
        return "[" + ", ".join(sorted(str(k) for k in mapping.keys())) + "]"
    except AttributeError:
        return f"<{type(mapping).__name__} has no keys()>"


class DiffusionLossFn(ABC):
    required_model_output_keys: tuple = ()
    required_data_keys: tuple = ()

    def validate_inputs(self, *, loss_name: str, model_output: dict, data: dict) -> None:
        mo = [k for k in self.required_model_output_keys if k not in model_output]
        dd = [k for k in self.required_data_keys if k not in data]
        if not mo and not dd:
            return
        msg = [f"Diffusion loss `{loss_name}` is missing required inputs."]
        if mo:
            msg.append(f"Missing model_output keys: {mo}. Available model_output keys: {_keys_of(model_output)}.")
        if dd:
            msg.append(f"Missing data keys: {dd}. Available data keys: {_keys_of(data)}.")
        raise KeyError(" ".join(msg))

    @classmethod
    @abstractmethod
    def compute_loss(cls, **kwargs) -> tuple[torch.Tensor, dict]:
        raise NotImplementedError

    @abstractmethod
    def __call__(self, *, config, model_output: dict, data: dict) -> DiffusionLossResult:
        raise NotImplementedError

    @staticmethod
    def prepare_actor_batch(batch: DataProto, reward_tensor: torch.Tensor, config: Any) -> DataProto:
        """Hook for losses that reshape rollouts into actor inputs (NFT, online DPO)."""
        return batch


DIFFUSION_LOSS_REGISTRY: dict[str, DiffusionLossFn] = {}


def register_diffusion_loss(name: str) -> Callable:
    def deco(cls):
        DIFFUSION_LOSS_REGISTRY[name] = cls()
        return cls

    return deco


def get_diffusion_loss_fn(name: str) -> DiffusionLossFn:
    if name not in DIFFUSION_LOSS_REGISTRY:
        raise ValueError(f"Unsupported diffusion loss mode: {name}. Supported modes are: "
                         f"{list(DIFFUSION_LOSS_REGISTRY.keys())}")
    return DIFFUSION_LOSS_REGISTRY[name]


class DiffusionAdvantageEstimator(str, Enum):
    FLOW_GRPO = "flow_grpo"
    DANCE_GRPO = "dance_grpo"
    MIX_GRPO = "mix_grpo"


DIFFUSION_ADV_ESTIMATOR_REGISTRY: dict[str, Callable] = {}


def register_diffusion_adv_est(name_or_enum) -> Callable:
    def deco(fn):
        name = name_or_enum.value if isinstance(name_or_enum, Enum) else name_or_enum
        prev = DIFFUSION_ADV_ESTIMATOR_REGISTRY.get(name)
        if prev is not None and prev is not fn:
            raise ValueError(f"Diffusion adv estimator {name} has already been registered: {prev} vs {fn}")
        DIFFUSION_ADV_ESTIMATOR_REGISTRY[name] = fn
        return fn

    return deco


def get_diffusion_adv_estimator_fn(name_or_enum) -> Callable:
    name = name_or_enum.value if isinstance(name_or_enum, Enum) else name_or_enum
    if name not in DIFFUSION_ADV_ESTIMATOR_REGISTRY:
        raise ValueError(f"Unknown diffusion advantage estimator: {name}. "
                         f"Supported: {list(DIFFUSION_ADV_ESTIMATOR_REGISTRY.keys())}")
    return DIFFUSION_ADV_ESTIMATOR_REGISTRY[name]


def _group_ids(index) -> tuple[torch.Tensor, int]:
    """Map arbitrary uid objects to dense group ids (first-appearance order)."""
    seen: dict = {}
    ids = []
    for u in list(index):
        key = u.item() if isinstance(u, torch.Tensor) else u
        if key not in seen:
            seen[key] = len(seen)
        ids.append(seen[key])
    return torch.tensor(ids, dtype=torch.long), len(seen)


def group_normalize(scores: torch.Tensor, index, *, epsilon: float = 1e-4, norm_by_std: bool = True,
                    global_std: bool = True) -> torch.Tensor:
    """GRPO normalisation of 1-D ``scores`` by prompt group.

    mean: per group (a singleton is its own mean); std: the whole batch's (unbiased) std when
    ``global_std`` else the group's unbiased std, with 1.0 for singletons.
    """
    x = scores.detach().float()
    gid, g = _group_ids(index)
    gid = gid.to(x.device)
    cnt = torch.zeros(g, device=x.device).index_add_(0, gid, torch.ones_like(x))
    s1 = torch.zeros(g, device=x.device).index_add_(0, gid, x)
    mean = s1 / cnt
    centered = x - mean[gid]
    if global_std:
        std = torch.std(x) if x.numel() > 1 else torch.tensor(float("nan"), device=x.device)
        std_per = std.expand_as(x)
    else:
        ss = torch.zeros(g, device=x.device).index_add_(0, gid, centered ** 2)
        gstd = torch.where(cnt > 1, torch.sqrt(ss / (cnt - 1).clamp_min(1)), torch.ones_like(cnt))
        std_per = gstd[gid]
    if norm_by_std:
        return centered / (std_per + epsilon)
    return centered


@register_diffusion_adv_est(DiffusionAdvantageEstimator.FLOW_GRPO)
@register_diffusion_adv_est(DiffusionAdvantageEstimator.DANCE_GRPO)
@register_diffusion_adv_est(DiffusionAdvantageEstimator.MIX_GRPO)
def compute_flow_grpo_outcome_advantage(sample_level_rewards: torch.Tensor, index, epsilon: float = 1e-4,
                                        norm_adv_by_std_in_grpo: bool = True, global_std: bool = True,
                                        config: Any = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Outcome advantage for every SDE step.

    Rows of ``sample_level_rewards`` [B, T] are grouped by prompt uid.  A group's mean and
    (unbiased) std run over all of its B_g x T entries; a single-row group is its own mean
    (advantage 0) with std 1 (or the batch std when ``global_std``).
    """
    scores = sample_level_rewards.detach().float()
    assert scores.ndim == 2
    b, t = scores.shape
    gid, g = _group_ids(index)
    gid = gid.to(scores.device)
    rows = torch.zeros(g, device=scores.device).index_add_(0, gid, torch.ones(b, device=scores.device))
    cnt = rows * t
    s1 = torch.zeros(g, device=scores.device).index_add_(0, gid, scores.sum(1))
    gmean = s1 / cnt
    single = (rows == 1)[gid]
    mean = torch.where(single[:, None], scores, gmean[gid][:, None].expand(b, t))
    centered = scores - mean
    if global_std:
        std = torch.std(scores).expand(b)
    else:
        ss = torch.zeros(g, device=scores.device).index_add_(0, gid, ((scores - gmean[gid][:, None]) ** 2).sum(1))
        gstd = torch.sqrt(ss / (cnt - 1).clamp_min(1))
        std = torch.where(single, torch.ones_like(gstd[gid]), gstd[gid])
    adv = centered / (std[:, None] + epsilon) if norm_adv_by_std_in_grpo else centered
    adv = adv.to(sample_level_rewards.dtype)
    return adv, adv


# ----------------------------------------------------------------------------- losses
def _clamp_adv(adv: torch.Tensor, cfg) -> torch.Tensor:
    return torch.clamp(adv, -cfg.adv_clip_max, cfg.adv_clip_max)


@register_diffusion_loss("flow_grpo")
@register_diffusion_loss("dance_grpo")
@register_diffusion_loss("mix_grpo")
class FlowGRPOLoss(DiffusionLossFn):
    required_model_output_keys = ("log_probs",)
    required_data_keys = ("old_log_probs", "advantages")

    @classmethod
    def compute_loss(cls, *, old_log_prob, log_prob, advantages, config, rollout_is_weights=None):
        lc = config.diffusion_loss
        adv = _clamp_adv(advantages, lc)
        loss, stats = loss_ops.ppo_clip_loss(log_prob, old_log_prob, adv, lc.clip_ratio, rollout_is_weights)
        return loss, {
            "actor/ppo_kl": stats["ppo_kl"],
            "actor/pg_clipfrac": stats["clipfrac"],
            "actor/pg_clipfrac_higher": stats["clipfrac_higher"],
            "actor/pg_clipfrac_lower": stats["clipfrac_lower"],
            "actor/ratio_mean": stats["ratio_mean"],
            "actor/ratio_std": stats["ratio_std"],
        }

    def __call__(self, *, config, model_output, data):
        loss, m = self.compute_loss(old_log_prob=data["old_log_probs"], log_prob=model_output["log_probs"],
                                    advantages=data["advantages"], config=config,
                                    rollout_is_weights=data.get("rollout_is_weights"))
        return DiffusionLossResult(loss, m)


def _bcast_like(v: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    if v.ndim == 0:
        return v.reshape(*([1] * target.ndim))
    return v.reshape(v.shape[0], *([1] * (target.ndim - 1)))


def _per_sample(v: torch.Tensor, batch: int):
    """``v`` as a ``[B]`` (or 0-d) tensor when it is constant over every non-batch dim, else None."""
    if v.numel() == 1:
        return v.reshape(())
    if v.numel() == batch and v.shape[0] == batch:
        return v.reshape(batch)
    return None


def _mean_nonbatch(x: torch.Tensor) -> torch.Tensor:
    return x.mean(dim=tuple(range(1, x.ndim))) if x.ndim > 1 else x


@register_diffusion_loss("flow_dppo")
class FlowDPPOLoss(DiffusionLossFn):
    required_model_output_keys = ("log_probs", "prev_sample_mean", "std_dev_t", "sqrt_dt")
    required_data_keys = ("old_log_probs", "advantages", "old_prev_sample_mean")

    @classmethod
    def compute_loss(cls, *, old_log_prob, log_prob, advantages, config, old_prev_sample_mean, prev_sample_mean,
                     std_dev_t, sqrt_dt, rollout_is_weights=None):
        lc = config.diffusion_loss
        adv = advantages.detach()
        log_ratio = log_prob - old_log_prob
        ratio = torch.exp(log_ratio)
        unclipped = -adv * ratio
        if getattr(lc, "add_kl_coefficient", True):
            sig = std_dev_t * _bcast_like(sqrt_dt, std_dev_t)
        else:
            sig = torch.ones((), device=prev_sample_mean.device)
        sig_b = _per_sample(sig, prev_sample_mean.shape[0])
        if sig_b is not None:
            kl = loss_ops.sq_dist(prev_sample_mean, old_prev_sample_mean) / (2 * sig_b.pow(2))
        else:
            kl = _mean_nonbatch((prev_sample_mean - old_prev_sample_mean).pow(2) / (2 * sig.pow(2)))
        high = kl >= lc.kl_mask_threshold
        pos = high & (ratio > 1.0) & (adv > 0)
        neg = high & (ratio < 1.0) & (adv < 0)
        rm = pos | neg
        keep = (~rm).detach()
        per = torch.where(keep, unclipped, torch.zeros((), dtype=unclipped.dtype, device=unclipped.device))
        if rollout_is_weights is not None:
            per = per * rollout_is_weights.detach()
        loss = per.mean()
        with torch.no_grad():
            m = {
                "actor/ppo_kl": torch.mean(-log_ratio).detach(),
                "actor/approx_kl": (0.5 * log_ratio.pow(2)).mean().detach(),
                "actor/ratio_mean": ratio.mean().detach(),
                "actor/ratio_std": ratio.std(unbiased=False).detach(),
                "actor/ratio_min": ratio.min().detach(),
                "actor/ratio_max": ratio.max().detach(),
                "actor/kl_new_old_mean": kl.mean().detach(),
                "actor/kl_new_old_max": kl.max().detach(),
                "actor/kl_mask_fraction": high.float().mean().detach(),
                "actor/pos_rm_fraction": pos.float().mean().detach(),
                "actor/neg_rm_fraction": neg.float().mean().detach(),
                "actor/masked_fraction": rm.float().mean().detach(),
                "actor/unmasked_fraction": keep.float().mean().detach(),
            }
        return loss, m

    def __call__(self, *, config, model_output, data):
        loss, m = self.compute_loss(old_log_prob=data["old_log_probs"], log_prob=model_output["log_probs"],
                                    advantages=data["advantages"], old_prev_sample_mean=data["old_prev_sample_mean"],
                                    prev_sample_mean=model_output["prev_sample_mean"],
                                    std_dev_t=model_output["std_dev_t"], sqrt_dt=model_output["sqrt_dt"],
                                    config=config, rollout_is_weights=data.get("rollout_is_weights"))
        return DiffusionLossResult(loss, m)


@register_diffusion_loss("grpo_guard")
class GRPOGuardLoss(DiffusionLossFn):
    required_model_output_keys = ("log_probs", "prev_sample_mean", "std_dev_t", "sqrt_dt")
    required_data_keys = ("old_log_probs", "advantages", "old_prev_sample_mean")

    @classmethod
    def compute_loss(cls, *, old_log_prob, log_prob, advantages, config, old_prev_sample_mean, prev_sample_mean,
                     std_dev_t, sqrt_dt, rollout_is_weights=None):
        lc = config.diffusion_loss
        adv = _clamp_adv(advantages, lc)
        sigma_t = std_dev_t.mean()
        sqrt_dt_mean = sqrt_dt.mean()
        scale = sqrt_dt_mean * sigma_t
        bias = loss_ops.sq_dist(prev_sample_mean, old_prev_sample_mean) / (2 * scale ** 2)
        log_ratio = log_prob - old_log_prob
        ratio = torch.exp((log_ratio + bias) * scale)
        unc = -adv * ratio
        clp = -adv * torch.clamp(ratio, 1.0 - lc.clip_ratio, 1.0 + lc.clip_ratio)
        per = torch.maximum(unc, clp)
        if rollout_is_weights is not None:
            per = per * rollout_is_weights.detach()
        loss = per.mean() / (sqrt_dt_mean ** 2)
        with torch.no_grad():
            m = {
                "actor/ppo_kl": torch.mean(-log_ratio).detach(),
                "actor/pg_clipfrac": torch.mean((torch.abs(ratio - 1.0) > lc.clip_ratio).float()).detach(),
                "actor/pg_clipfrac_higher": torch.mean((ratio - 1.0 > lc.clip_ratio).float()).detach(),
                "actor/pg_clipfrac_lower": torch.mean((1.0 - ratio > lc.clip_ratio).float()).detach(),
                "actor/ratio_mean": ratio.mean().detach(),
                "actor/ratio_std": ratio.std() if ratio.numel() > 1 else torch.zeros((), device=ratio.device),
            }
        return loss, m

    def __call__(self, *, config, model_output, data):
        loss, m = self.compute_loss(old_log_prob=data["old_log_probs"], log_prob=model_output["log_probs"],
                                    advantages=data["advantages"], old_prev_sample_mean=data["old_prev_sample_mean"],
                                    prev_sample_mean=model_output["prev_sample_mean"],
                                    std_dev_t=model_output["std_dev_t"], sqrt_dt=model_output["sqrt_dt"],
                                    config=config, rollout_is_weights=data.get("rollout_is_weights"))
        return DiffusionLossResult(loss, m)


@register_diffusion_loss("dpo")
class DPOLoss(DiffusionLossFn):
    required_model_output_keys = ("noise", "latent", "noise_pred")
    required_data_keys = ("ref_noise_pred", "sample_level_rewards")

    @staticmethod
    def build_online_dpo_pair_indices(*, uids, scores: torch.Tensor) -> list[int]:
        """One (best, worst) adjacent pair per prompt uid with at least two samples."""
        flat = (scores.squeeze(-1) if scores.ndim > 1 else scores).detach().cpu().float().tolist()
        uids = np.asarray(uids, dtype=object).reshape(-1)
        if len(uids) != len(flat):
            raise ValueError(f"Online DPO pairing expects one uid per score, got {len(uids)} vs {len(flat)}.")
        groups: dict = defaultdict(list)
        for i, u in enumerate(uids):
            groups[u].append(i)
        out: list[int] = []
        for idxs in groups.values():
            if len(idxs) < 2:
                continue
            order = sorted(idxs, key=lambda i: flat[i], reverse=True)
            out += [order[0], order[-1]]
        return out

    @staticmethod
    def prepare_actor_batch(batch: DataProto, reward_tensor: torch.Tensor, config: Any) -> DataProto:
        if config.algorithm.sample_source == "offline":
            return batch
        if "uid" not in batch.non_tensor_batch:
            raise KeyError("Online DPO pairing requires `uid` in non_tensor_batch.")
        rewards = reward_tensor.squeeze(-1).float() if reward_tensor.ndim > 1 else reward_tensor.float()
        sel = DPOLoss.build_online_dpo_pair_indices(uids=batch.non_tensor_batch["uid"], scores=rewards)
        if not sel:
            raise RuntimeError("Online DPO could not build preference pairs; increase actor_rollout_ref.rollout.n.")
        out = batch.select_idxs(sel)
        out.meta_info["prepare_actor_batch_selected_indices"] = sel
        return out

    @staticmethod
    def _pairs_share_uid(index, n: int) -> bool:
        if isinstance(index, torch.Tensor):
            f = index.reshape(-1)[:n]
            return bool(torch.all(f[0::2] == f[1::2]).item())
        f = np.asarray(list(index), dtype=object).reshape(-1)[:n]
        return bool(np.all(f[0::2] == f[1::2]))

    @classmethod
    def compute_loss(cls, noise, latent, model_noise_pred, ref_noise_pred, sample_level_rewards, config=None, *,
                     index=None):
        scores = sample_level_rewards.squeeze(-1) if sample_level_rewards.ndim > 1 else sample_level_rewards
        if scores.shape[0] < 2 or scores.shape[0] % 2:
            raise ValueError("DPO loss expects an even batch of adjacent chosen/rejected pairs.")
        if index is not None and not cls._pairs_share_uid(index, int(scores.shape[0])):
            raise ValueError("DPO loss expects each adjacent chosen/rejected pair to share the same prompt uid.")
        if torch.any(scores[0::2] < scores[1::2]).item():
            raise ValueError("DPO loss expects each chosen sample reward to be >= its rejected pair reward.")
        beta = config.diffusion_loss.dpo_beta
        target = noise.float() - latent.float()
        model_err = loss_ops.sq_dist(model_noise_pred.float().contiguous(), target.contiguous())
        with torch.no_grad():
            ref_err = loss_ops.sq_dist(ref_noise_pred.float().contiguous(), target.contiguous())
        w_diff = model_err[0::2] - ref_err[0::2]
        l_diff = model_err[1::2] - ref_err[1::2]
        inside = -0.5 * beta * (w_diff - l_diff)
        loss = -F.logsigmoid(inside).mean()
        with torch.no_grad():
            rc, rr = -0.5 * beta * w_diff, -0.5 * beta * l_diff
            m = {
                "actor/dpo_loss": loss.detach(),
                "actor/implicit_acc": ((inside > 0).sum().float() / inside.numel()).detach(),
                "rewards/chosen": rc.mean().detach(),
                "rewards/rejected": rr.mean().detach(),
                "rewards/margins": (rc - rr).mean().detach(),
            }
        return loss, m

    def __call__(self, *, config, model_output, data):
        loss, m = self.compute_loss(noise=model_output["noise"], latent=model_output["latent"],
                                    model_noise_pred=model_output["noise_pred"], ref_noise_pred=data["ref_noise_pred"],
                                    sample_level_rewards=data["sample_level_rewards"], config=config,
                                    index=data.get("uid"))
        return DiffusionLossResult(loss, m)


@register_diffusion_loss("diffusion_nft")
class DiffusionNFTLoss(DiffusionLossFn):
    required_model_output_keys = ("forward_prediction", "old_prediction", "ref_forward_prediction", "x0", "xt",
                                  "t_expanded")
    required_data_keys = ("reward_prob",)

    @classmethod
    def compute_loss(cls, *, forward_prediction, old_prediction, ref_forward_prediction, x0, xt, t_expanded,
                     reward_prob, config):
        lc = config.diffusion_loss
        beta = lc.mix_beta
        old = old_prediction.detach()
        ref = ref_forward_prediction.detach()
        w = reward_prob.flatten(1).mean(1) if reward_prob.ndim > 1 else reward_prob
        w = w.to(device=x0.device, dtype=x0.dtype)
        dims = tuple(range(1, x0.ndim))
        pos_pred = beta * forward_prediction + (1.0 - beta) * old
        neg_pred = (1.0 + beta) * old - beta * forward_prediction
        x0_pos = xt - t_expanded * pos_pred
        x0_neg = xt - t_expanded * neg_pred
        with torch.no_grad():
            pw = torch.abs(x0_pos.double() - x0.double()).mean(dim=dims, keepdim=True).clip(
                min=lc.adaptive_weight_min).to(x0_pos.dtype)
            nw = torch.abs(x0_neg.double() - x0.double()).mean(dim=dims, keepdim=True).clip(
                min=lc.adaptive_weight_min).to(x0_neg.dtype)
        # per-sample squared distances (one fused pass each on CUDA fp32), divided by the per-sample weights
        x0c = x0.contiguous()
        pos_loss = loss_ops.sq_dist(x0_pos.contiguous(), x0c) / pw.reshape(-1).float()
        neg_loss = loss_ops.sq_dist(x0_neg.contiguous(), x0c) / nw.reshape(-1).float()
        per = w * pos_loss / beta + (1.0 - w) * neg_loss / beta
        policy_loss = (per * lc.adv_clip_max).mean()
        ref_kl = loss_ops.sq_dist(forward_prediction.contiguous(), ref.contiguous()).mean()
        loss = policy_loss + lc.ref_kl_coef * ref_kl
        with torch.no_grad():
            m = {
                "actor/policy_loss": policy_loss.detach(),
                "actor/positive_loss": pos_loss.mean().detach(),
                "actor/negative_loss": neg_loss.mean().detach(),
                "actor/ref_kl_loss": ref_kl.detach(),
                "actor/old_deviate": loss_ops.sq_dist(forward_prediction.detach().contiguous(), old.contiguous()).mean(),
                "actor/reward_prob_mean": w.mean().detach(),
                "actor/total_loss": loss.detach(),
            }
        return loss, m

    def __call__(self, *, config, model_output, data):
        loss, m = self.compute_loss(**{k: model_output[k] for k in self.required_model_output_keys},
                                    reward_prob=data["reward_prob"], config=config)
        return DiffusionLossResult(loss, m)

    @staticmethod
    def _compute_group_advantages(rewards, uid, norm_by_std: bool, global_std: bool, epsilon: float = 1e-4):
        return group_normalize(rewards.detach().float(), uid, epsilon=epsilon, norm_by_std=norm_by_std,
                               global_std=global_std)

    @staticmethod
    def _advantage_to_reward_prob(advantages, adv_clip_max: float, adv_mode: str):
        a = torch.clamp(advantages, -adv_clip_max, adv_clip_max)
        if adv_mode == "positive_only":
            a = torch.clamp(a, 0, adv_clip_max)
        elif adv_mode == "negative_only":
            a = torch.clamp(a, -adv_clip_max, 0)
        elif adv_mode == "one_only":
            a = (a > 0).to(a.dtype)
        elif adv_mode == "binary":
            a = torch.sign(a)
        return torch.clamp((a / adv_clip_max) / 2.0 + 0.5, 0, 1)

    @staticmethod
    def _select_train_timesteps(train_timesteps: torch.Tensor, timestep_fraction: float, seed: Optional[int] = None):
        if train_timesteps.ndim != 2:
            raise ValueError(f"`train_timesteps` must have shape [B, T], got {tuple(train_timesteps.shape)}.")
        t = train_timesteps.shape[1]
        k = max(1, int(t * timestep_fraction))
        gen = None
        if seed is not None:
            gen = torch.Generator(device=train_timesteps.device)
            gen.manual_seed(int(seed))
        rows = [row[torch.randperm(t, device=train_timesteps.device, generator=gen)[:k]] for row in train_timesteps]
        return torch.stack(rows, 0).long()

    @staticmethod
    def prepare_actor_batch(batch: DataProto, reward_tensor: torch.Tensor, config: Any) -> DataProto:
        algo = config.algorithm
        actor = config.actor_rollout_ref.actor
        if "uid" not in batch.non_tensor_batch:
            raise ValueError("DiffusionNFT actor batch requires `uid` in non_tensor_batch.")
        for key in ("latents_clean", "train_timesteps"):
            if key not in batch.batch:
                raise ValueError(f"DiffusionNFT actor batch requires `{key}` from rollout.")
        adv = DiffusionNFTLoss._compute_group_advantages(reward_tensor, batch.non_tensor_batch["uid"],
                                                         algo.norm_adv_by_std_in_grpo, algo.global_std)
        rp = DiffusionNFTLoss._advantage_to_reward_prob(adv, actor.diffusion_loss.adv_clip_max, algo.adv_mode)
        tt = DiffusionNFTLoss._select_train_timesteps(batch.batch["train_timesteps"], algo.timestep_fraction,
                                                      seed=actor.data_loader_seed)
        k = tt.shape[1]
        batch.batch["train_timesteps"] = tt
        batch.batch["advantages"] = adv[:, None].expand(-1, k).contiguous()
        batch.batch["reward_prob"] = rp[:, None].expand(-1, k).contiguous()
        batch.batch["returns"] = batch.batch["advantages"]
        batch.batch["sample_level_rewards"] = reward_tensor[:, None].expand(-1, k).contiguous()
        return batch


class _MeanKL(DiffusionLossFn):
    """Gaussian KL between two reverse-SDE means sharing the std: mean((m1-m2)^2) / (2 std^2)."""

    target_key = ""
    metric = ""
    required_model_output_keys = ("prev_sample_mean", "std_dev_t")

    @classmethod
    def _kl(cls, prev_sample_mean, other, std_dev_t):
        if prev_sample_mean.ndim > 1:
            std_b = _per_sample(std_dev_t, prev_sample_mean.shape[0])
            if std_b is not None:
                d2 = loss_ops.sq_dist(prev_sample_mean, other)
                return (d2 / (2 * std_b ** 2)).reshape(-1, *([1] * (prev_sample_mean.ndim - 1)))
        d2 = ((prev_sample_mean - other) ** 2)
        d2 = d2.mean(dim=tuple(range(1, d2.ndim)), keepdim=True)
        std = std_dev_t.reshape(std_dev_t.shape[0], *([1] * (d2.ndim - 1))) if std_dev_t.ndim else std_dev_t
        return d2 / (2 * std ** 2)

    def __call__(self, *, config, model_output, data):
        kl = self._kl(model_output["prev_sample_mean"], data[self.target_key], model_output["std_dev_t"])
        return DiffusionLossResult(kl.mean(), {self.metric: kl.mean().detach()})


@register_diffusion_loss("kl")
class KLLoss(_MeanKL):
    required_data_keys = ("ref_prev_sample_mean",)
    target_key = "ref_prev_sample_mean"
    metric = "actor/kl_loss"

    @classmethod
    def compute_loss(cls, *, prev_sample_mean, ref_prev_sample_mean, std_dev_t):
        kl = cls._kl(prev_sample_mean, ref_prev_sample_mean, std_dev_t)
        return kl.mean(), {cls.metric: kl.mean().detach()}


@register_diffusion_loss("distill_kl")
class DistillKLLoss(_MeanKL):
    required_data_keys = ("teacher_prev_sample_mean",)
    target_key = "teacher_prev_sample_mean"
    metric = "actor/distill_kl_loss"

    @classmethod
    def compute_loss(cls, *, prev_sample_mean, teacher_prev_sample_mean, std_dev_t):
        kl = cls._kl(prev_sample_mean, teacher_prev_sample_mean, std_dev_t)
        return kl.mean(), {cls.metric: kl.mean().detach()}


@register_diffusion_loss("distill_fm_mse")
class DistillFlowMatchingMSELoss(DiffusionLossFn):
    required_model_output_keys = ("noise_pred",)
    required_data_keys = ("teacher_noise_pred",)

    @classmethod
    def compute_loss(cls, *, noise_pred, teacher_noise_pred):
        mse = ((noise_pred - teacher_noise_pred) ** 2).mean()
        return mse, {"actor/distill_fm_mse_loss": mse.detach()}

    def __call__(self, *, config, model_output, data):
        loss, m = self.compute_loss(noise_pred=model_output["noise_pred"], teacher_noise_pred=data["teacher_noise_pred"])
        return DiffusionLossResult(loss, m)
