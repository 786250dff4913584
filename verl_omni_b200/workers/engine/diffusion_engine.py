"""Diffusion policy engines: per-micro-batch x per-SDE-step forward/backward on the sharded engine.

The hot loop of ``verl_omni/workers/engine/fsdp/diffusers_impl.py:784-943``: the batch is split
into micro-batches; for every micro-batch and every trained timestep the adapter runs the DiT and
the fused SDE log-prob, the loss is computed and back-propagated immediately (gradient
accumulation over ``n_micro * T`` passes into the fp32 main grads).  ``infer_batch`` is the
forward-only variant used for old-policy / reference log-probs and reverse-SDE means.

Metrics stay on the device as tensors and are reduced once per call.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Callable, Optional

import torch

from verl_omni_b200.pipelines.model_base import DiffusionModelBase
from verl_omni_b200.utils.dataproto import DataProto
from verl_omni_b200.workers.engine.base import ShardedEngine

_ENGINE_REGISTRY: dict[tuple[str, str], type] = {}


def register_engine(model_type: str, backend: tuple = ("fsdp", "fsdp2")):
    def deco(cls):
        for b in backend:
            _ENGINE_REGISTRY[(model_type, b)] = cls
        return cls

    return deco


def new_engine(model_type: str, backend: str, *args, **kwargs):
    """``EngineRegistry.new`` equivalent."""
    if (model_type, backend) not in _ENGINE_REGISTRY:
        raise KeyError(f"no engine for model_type={model_type!r} backend={backend!r}")
    return _ENGINE_REGISTRY[(model_type, backend)](*args, **kwargs)


def _mean_metrics(ms: list[dict]) -> dict:
    """Means of per-micro-step metrics.  Device tensors are stacked on the device and read back with one
    copy; host floats are averaged on the host."""
    acc: dict = defaultdict(list)
    for m in ms:
        for k, v in m.items():
            acc[k].append(v)
    out, dev_keys, dev_vals = {}, [], []
    for k, vs in acc.items():
        if all(isinstance(v, torch.Tensor) for v in vs):
            dev_keys.append(k)
            dev_vals.append(torch.stack([v.detach().float().reshape(()) for v in vs]).mean())
        else:
            out[k] = float(sum(float(v) for v in vs) / len(vs))
    if dev_keys:
        by_dev: dict = defaultdict(list)
        for k, v in zip(dev_keys, dev_vals):
            by_dev[v.device].append((k, v))
        for items in by_dev.values():
            vals = torch.stack([v for _, v in items]).cpu().tolist()
            out.update({k: x for (k, _), x in zip(items, vals)})
    return out


@register_engine("diffusion_model", ("fsdp", "fsdp2", "veomni", "b200"))
class PPODiffusionEngine:
    """Actor (or frozen ref) DiT with the PPO-style per-timestep training loop."""

    def __init__(self, module, adapter: type[DiffusionModelBase], scheduler, actor_cfg, model_cfg, *, device,
                 group=None, total_steps: int = 1, trainable: bool = True, param_offload: Optional[bool] = None):
        self.engine = ShardedEngine(module, actor_cfg, device=device, group=group, total_steps=total_steps,
                                    trainable=trainable, param_offload=param_offload)
        self.module = module
        self.adapter = adapter
        self.scheduler = scheduler
        self.cfg = actor_cfg
        self.model_cfg = model_cfg
        self.device = device
        # sequence-parallel ranks each back-propagate their own tokens' share: the loss is scaled by sp so the
        # world-averaged gradient equals the data-parallel average
        self.sp = int(getattr(actor_cfg.fsdp_config, "ulysses_sequence_parallel_size", 1) or 1)
        self.engine.offload_params()  # frozen engine with param_offload: on the host until its phase runs

    # ------------------------------------------------------------------ helpers
    def _micro_batches(self, data: DataProto, mbs: Optional[int]) -> list[DataProto]:
        n = len(data)
        mbs = mbs or n
        return [data.select_idxs(slice(i, min(i + mbs, n))) for i in range(0, n, mbs)]

    def _cond(self, mb: DataProto, neg: bool = False):
        keys = self.adapter.cond_keys()
        pre = "negative_" if neg else ""
        if neg and (pre + keys[0]) not in mb.batch:
            return None
        return {k: mb.batch[pre + k].to(self.device, non_blocking=True) for k in keys}

    def _step_out(self, mb: DataProto, t: int) -> dict:
        lat = mb.batch["latents"]
        algo = self.model_cfg.algo
        return self.adapter.forward_and_sample_previous_step(
            self.module, self.scheduler,
            latents=lat[:, t].to(self.device, non_blocking=True),
            prev_latents=lat[:, t + 1].to(self.device, non_blocking=True),
            step_index=mb.batch["step_index"][:, t].to(self.device),
            cond=self._cond(mb), neg_cond=self._cond(mb, True),
            guidance_scale=self.model_cfg.pipeline.guidance_scale, noise_level=algo.noise_level,
            sde_type=algo.sde_type)

    # ------------------------------------------------------------------ infer
    @torch.no_grad()
    def infer_batch(self, data: DataProto, keys=("log_probs",), micro_batch_size: Optional[int] = None) -> DataProto:
        """Per-step outputs for every trajectory: ``log_probs`` [B, T] and optionally
        ``prev_sample_mean`` [B, T, ...] (reference/old means for KL, DPPO, GRPO-Guard)."""
        self.engine.eval_mode()
        self.engine.load_params()
        try:
            return self._infer(data, keys, micro_batch_size)
        finally:
            self.engine.offload_params()

    def _infer(self, data: DataProto, keys, micro_batch_size: Optional[int]) -> DataProto:
        T = data.batch["step_index"].shape[1]
        outs = defaultdict(list)
        for mb in self._micro_batches(data, micro_batch_size or self.cfg.ppo_micro_batch_size_per_gpu):
            per = defaultdict(list)
            for t in range(T):
                o = self._step_out(mb, t)
                for k in keys:
                    per[k].append(o[k].detach())
            for k in keys:
                outs[k].append(torch.stack(per[k], 1))
        return DataProto({k: torch.cat(v, 0) for k, v in outs.items()})

    # ------------------------------------------------------------------ train
    def train_batch(self, data: DataProto, loss_fn: Callable) -> dict:
        """One optimizer step over ``data`` (zero_grad -> fwd/bwd over micro x T -> step)."""
        eng = self.engine
        eng.train_mode()
        eng.zero_grad()
        T = data.batch["step_index"].shape[1]
        mbs = self._micro_batches(data, self.cfg.ppo_micro_batch_size_per_gpu)
        gas = len(mbs) * T
        metrics, losses = [], []
        for mb in mbs:
            for t in range(T):
                out = self._step_out(mb, t)
                d = {"old_log_probs": mb.batch["old_log_probs"][:, t].to(self.device),
                     "advantages": mb.batch["advantages"][:, t].to(self.device),
                     "gradient_accumulation_steps": gas, "sp_size": self.sp}
                for k in ("ref_prev_sample_mean", "old_prev_sample_mean", "teacher_prev_sample_mean",
                          "teacher_noise_pred", "rollout_is_weights"):
                    if k in mb.batch:
                        d[k] = mb.batch[k][:, t].to(self.device)
                if "uid" in mb.non_tensor_batch:
                    d["uid"] = mb.non_tensor_batch["uid"]
                loss, m = loss_fn(model_output=out, data=d)
                loss.backward()
                losses.append(loss.detach() * gas)
                metrics.append(m)
        grad_norm = eng.optimizer_step()
        metrics.append({"actor/pg_loss": torch.stack(losses).float().mean(), "actor/grad_norm": grad_norm.reshape(())})
        res = _mean_metrics(metrics)
        res["actor/lr"] = eng.lr()
        return res
