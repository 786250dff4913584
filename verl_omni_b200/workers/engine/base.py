"""Sharded training engine core: flat parameters, fp32 main grads, sharded AdamW, checkpoints.

Design for B200 (180 GB HBM per GPU):

* every trainable parameter lives in ONE flat compute-dtype buffer (bf16 on GPU); parameter
  tensors are views into it, so the rollout engine and the trainer share the same weights and
  the trainer->rollout "weight sync" within a process is free;
* gradients accumulate in a flat fp32 ``main_grad`` buffer (the GEMM weight-gradient epilogue
  adds into it directly) across all micro-batches and SDE timesteps of a step;
* the fp32 master weights and AdamW moments are sharded 1/world per rank; one optimizer step is
  reduce-scatter(main_grad) -> global-norm clip -> fused AdamW on the shard (writing the fp32
  master and the bf16 copy in one pass) -> all-gather of the bf16 shards;
* ``reshard_after_forward=False`` (default): the gathered bf16 weights stay resident (ZeRO-2
  style); this removes per-block all-gathers from the hot loop for every model in scope.

Engine contract and checkpoint layout follow the reference's FSDP engine
(``verl_omni/workers/engine/fsdp/diffusers_impl.py:405-724``): AdamW with constant/cosine
warm-up schedules, grad-clip with a skipped step on a non-finite norm, and per-rank files
``model_world_size_{W}_rank_{r}.pt`` / ``optim_world_size_{W}_rank_{r}.pt`` /
``extra_state_world_size_{W}_rank_{r}.pt`` + ``fsdp_config.json``.  Model files hold each
parameter's dim-0 shard (the FSDP2 ``Shard(0)`` placement, recorded in the file), so a checkpoint
can be re-loaded at a different world size.
"""

from __future__ import annotations

import json
import math
import os
from typing import Callable, Iterable, Optional

import torch
import torch.nn as nn

from verl_omni_b200.parallel import dist as D
from verl_omni_b200.ops._ext import ext

_ALIGN = 128
_PARAM_ALIGN = 16  # elements


def _dtype(name: str) -> torch.dtype:
    return {"bfloat16": torch.bfloat16, "bf16": torch.bfloat16, "float32": torch.float32, "fp32": torch.float32,
            "float16": torch.float16}[name]


class FlatParams:
    """Packs the trainable parameters of ``module`` into one flat buffer + fp32 grad buffer."""

    def __init__(self, module: nn.Module, dtype: torch.dtype, device: torch.device, world: int, rank: int,
                 group=None, symmetric: bool = False, select=None, owns_module: bool = True):
        self.module = module
        self.group = group
        self.world, self.rank = world, rank
        self.names, self.params = [], []
        for n, p in module.named_parameters():
            if p.requires_grad and (select is None or select(n, p)):
                self.names.append(n)
                self.params.append(p)
        self.shapes = [tuple(p.shape) for p in self.params]
        self.numels = [p.numel() for p in self.params]
        self.offsets = []
        off = 0
        for n in self.numels:
            self.offsets.append(off)
            # every parameter (and its main_grad slice) starts on a 64-byte boundary: TMA epilogues
            # and vector reductions address them directly
            off += (n + _PARAM_ALIGN - 1) // _PARAM_ALIGN * _PARAM_ALIGN
        self.numel = off
        unit = world * _ALIGN
        self.padded = max(unit, (off + unit - 1) // unit * unit)
        self.shard_size = self.padded // world
        self.shard_lo = rank * self.shard_size
        self.device, self.dtype = device, dtype
        self.symm_flat = self.symm_grad = None
        if symmetric:
            self._try_symmetric(dtype, device, group)
        if self.symm_flat is not None:
            self.flat, self.main_grad = self.symm_flat.tensor, self.symm_grad.tensor
        else:
            self.flat = torch.zeros(self.padded, dtype=dtype, device=device)
            self.main_grad = torch.zeros(self.padded, dtype=torch.float32, device=device)
        # parameter by parameter: the compute copy into the flat buffer, this rank's slice into the fp32
        # master, then the parameter is rebound to its flat view (its own storage is released at once), so
        # no full-size fp32 temporary exists and peak memory stays near one model copy
        self.flat.zero_()
        self.master = torch.zeros(self.shard_size, dtype=torch.float32, device=device)
        lo, hi = self.shard_lo, self.shard_lo + self.shard_size
        for p, o, n, s in zip(self.params, self.offsets, self.numels, self.shapes):
            src = p.detach().reshape(-1)
            self.flat[o:o + n].copy_(src)
            a, b = max(o, lo), min(o + n, hi)
            if a < b:
                self.master[a - lo:b - lo].copy_(src[a - o:b - o])
            p.data = self.flat[o:o + n].view(s)
            p.main_grad = self.main_grad[o:o + n].view(s)
            p.register_post_accumulate_grad_hook(self._accumulate)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.grad_shard = torch.zeros_like(self.master)
        if not owns_module:
            return
        # non-trainable parameters and buffers follow the compute dtype/device
        for m in module.modules():
            for k, p in list(m._parameters.items()):
                if p is not None and not p.requires_grad:
                    p.data = p.data.to(device=device, dtype=dtype if p.is_floating_point() else p.dtype)
            for k, b in list(m._buffers.items()):
                if b is not None:
                    m._buffers[k] = b.to(device=device)

    def _try_symmetric(self, dtype, device, group) -> None:
        """Peer-mapped flat buffers (the fused optimizer step reads peers' grads and writes peers'
        weights).  Every rank must succeed: the outcome is agreed collectively and, if any rank could not
        map its peers, all ranks fall back to ordinary buffers and NCCL collectives."""
        from verl_omni_b200.parallel.symm_mem import SymmetricBuffer

        bufs, err = [], None
        try:
            bufs.append(SymmetricBuffer(self.padded, dtype, device, group))
            bufs.append(SymmetricBuffer(self.padded, torch.float32, device, group))
        except Exception as e:  # noqa: BLE001 - agreed on below, reported by rank
            err = e
        ok = torch.tensor([0 if err is not None else 1], dtype=torch.int32, device=device)
        D.all_reduce(ok, op=torch.distributed.ReduceOp.MIN, group=group)
        if int(ok.item()) == 1:
            self.symm_flat, self.symm_grad = bufs
            return
        for b in bufs:
            b.close(collective=False)
        if err is not None:
            import warnings

            warnings.warn(f"symmetric memory unavailable, using NCCL collectives: {err}")

    @staticmethod
    def _accumulate(p: torch.Tensor) -> None:
        if p.grad is not None:
            if p.main_grad is None:
                raise RuntimeError("backward after the gradient buffer was released: call the engine's zero_grad "
                                   "before the update's first backward")
            p.main_grad.add_(p.grad.view_as(p.main_grad))
            p.grad = None

    def zero_grad(self) -> None:
        if self.main_grad is None:  # released by ``release_grads``: re-created zeroed and re-bound
            self.main_grad = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
            for p, o, n, s in zip(self.params, self.offsets, self.numels, self.shapes):
                p.main_grad = self.main_grad[o:o + n].view(s)
            return
        self.main_grad.zero_()

    # ------------------------------------------------------------------ host offload
    def release_grads(self) -> None:
        """Drops the full-size fp32 gradient buffer (between updates it holds nothing: every update starts
        with ``zero_grad``, which re-creates it).  Peer-mapped gradient buffers stay."""
        if self.symm_grad is not None or self.main_grad is None:
            return
        self.main_grad = None
        for p in self.params:
            p.main_grad = None

    _OPT_STATE = ("master", "exp_avg", "exp_avg_sq", "grad_shard")

    def offload_optimizer(self) -> None:
        """fp32 master shard, AdamW moments and the gradient shard to pinned host memory (the device copies
        are released); ``load_optimizer`` brings them back."""
        if self.device.type != "cuda" or not self.master.is_cuda:
            return
        for k in self._OPT_STATE:
            t = getattr(self, k)
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t, non_blocking=True)
            setattr(self, k, h)
        torch.cuda.current_stream(self.device).synchronize()  # host copies complete before anyone reads them

    def load_optimizer(self) -> None:
        if self.device.type != "cuda" or self.master.is_cuda:
            return
        for k in self._OPT_STATE:
            setattr(self, k, getattr(self, k).to(self.device, non_blocking=True))

    def shard_view(self) -> torch.Tensor:
        return self.flat[self.shard_lo:self.shard_lo + self.shard_size]

    def full_master(self) -> torch.Tensor:
        full = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        D.all_gather_into(full, self.master, self.group)
        return full

    def param_views(self, flat: torch.Tensor) -> Iterable[tuple[str, torch.Tensor]]:
        for n, o, k, s in zip(self.names, self.offsets, self.numels, self.shapes):
            yield n, flat[o:o + k].view(s)


class LRSchedule:
    """Constant or cosine schedule with linear warm-up (reference ``diffusers_impl.py:412-443``)."""

    def __init__(self, optim_cfg, total_steps: int):
        self.base = float(optim_cfg.lr)
        self.kind = optim_cfg.lr_scheduler_type
        total = optim_cfg.total_training_steps if optim_cfg.total_training_steps > 0 else total_steps
        self.total = max(1, int(total))
        warm = optim_cfg.lr_warmup_steps
        if warm is None or warm < 0:
            warm = int(optim_cfg.lr_warmup_steps_ratio * self.total)
        self.warmup = warm
        self.min_ratio = optim_cfg.min_lr_ratio
        self.cycles = optim_cfg.num_cycles
        self.step_count = 0

    def lr(self) -> float:
        s = self.step_count
        if self.warmup > 0 and s < self.warmup:
            return self.base * (s + 1) / self.warmup
        if self.kind == "constant":
            return self.base
        prog = (s - self.warmup) / max(1, self.total - self.warmup)
        cos = 0.5 * (1.0 + math.cos(math.pi * 2.0 * self.cycles * prog))
        return self.base * (self.min_ratio + (1 - self.min_ratio) * cos)

    def step(self) -> None:
        self.step_count += 1

    def state_dict(self) -> dict:
        return {"step_count": self.step_count}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step_count"])


class ShardedEngine:
    """Owns a module, its flat parameters and the sharded AdamW state."""

    def __init__(self, module: nn.Module, actor_cfg, *, device: torch.device, group=None, total_steps: int = 1,
                 trainable: bool = True, expert_group=None, pp_size: int = 1, param_offload: Optional[bool] = None):
        """``pp_size > 1``: ``module`` is one pipeline stage and ``group`` the ranks holding the same stage; the
        gradient norm for clipping is then reduced over every rank (all stages)."""
        self.cfg = actor_cfg
        self.pp_size = int(pp_size)
        self.group = group if group is not None else D.default_group()
        # expert-parallel parameters (marked ``_vo_expert``: each rank holds only its experts' slices) live in
        # a second flat set sharded over ``expert_group`` -- the ranks that hold the same experts
        self.expert_group = expert_group
        self.eflat = None
        self.replica_group = None
        self.n_replicas = 1
        fs = int(getattr(actor_cfg.fsdp_config, "fsdp_size", -1) or -1)
        vc = getattr(actor_cfg, "veomni_config", None) if getattr(actor_cfg, "strategy", "") == "veomni" else None
        if vc is not None and fs <= 0:
            # VeOmni layout (reference workers/engine/veomni/diffusion_impl.py:97-132): dp_shard groups of
            # veomni_config.fsdp_size ranks, replicated across dp_replicate = world / fsdp_size
            fs = int(getattr(vc, "fsdp_size", -1) or -1)
        if group is None and 0 < fs < D.world_size() and trainable:
            # HSDP: shard within groups of fsdp_size consecutive ranks (one node), replicate across them
            self.group, self.replica_group = D.make_hsdp_groups(fs)
            self.n_replicas = D.world_size() // fs
        self.world = D.world_size(self.group)
        self.rank = D.rank(self.group)
        self.device = device
        self.dtype = _dtype(actor_cfg.fsdp_config.dtype) if device.type == "cuda" else torch.float32
        self.module = module
        self.trainable = trainable
        if not trainable:
            for p in module.parameters():
                p.requires_grad_(False)
            module.to(device=device, dtype=self.dtype)
            self.flat = None
        else:
            has_experts = any(getattr(p, "_vo_expert", False) for p in module.parameters())
            if has_experts and self.replica_group is not None:
                raise ValueError("expert-parallel parameters with HSDP replicas are not supported")
            not_expert = (lambda n, p: not getattr(p, "_vo_expert", False)) if has_experts else None
            self.flat = FlatParams(module, self.dtype, device, self.world, self.rank, self.group,
                                   symmetric=(not has_experts and self.replica_group is None and self.pp_size == 1
                                              and self._want_symmetric(actor_cfg, device, self.group)),
                                   select=not_expert)
            if has_experts:
                eg = expert_group
                self.eflat = FlatParams(module, self.dtype, device, D.world_size(eg), D.rank(eg), eg,
                                        select=lambda n, p: getattr(p, "_vo_expert", False), owns_module=False)
        self.opt_step = 0
        self.sched = LRSchedule(actor_cfg.optim, total_steps) if trainable else None
        self.last_grad_norm = None
        fc = actor_cfg.fsdp_config
        if trainable and bool(getattr(fc, "reshard_after_forward", False)):
            import warnings

            warnings.warn("fsdp_config.reshard_after_forward=true: the bf16 weights stay whole on every rank (only "
                          "the fp32 master, moments and gradient shards are sharded); use param_offload / "
                          "optimizer_offload to reduce device memory")
        self.optimizer_offload = bool(getattr(fc, "optimizer_offload", False)) and device.type == "cuda"
        po = getattr(fc, "param_offload", False) if param_offload is None else param_offload
        self.param_offload = bool(po) and device.type == "cuda"
        self._host_params = None
        if trainable:
            self._after_update()

    def _flats(self) -> list:
        return [f for f in (self.flat, self.eflat) if f is not None]

    def _after_update(self) -> None:
        """Between updates: optimizer state to the host (``optimizer_offload``), gradient buffers released
        (``param_offload``; the bf16 weights stay, the colocated rollout reads them in place)."""
        for f in self._flats():
            if self.optimizer_offload:
                f.offload_optimizer()
            if self.param_offload:
                f.release_grads()

    def _before_update(self) -> None:
        for f in self._flats():
            f.load_optimizer()

    # frozen engines (reference policy, distillation teacher): weights on the host while idle
    def offload_params(self) -> None:
        """``param_offload`` on a frozen engine: its weights move to pinned host memory until ``load_params``
        (reference / teacher models are read in one phase of the step and idle in the others)."""
        if self.trainable or not self.param_offload or self._host_params is not None:
            return
        self._host_params = []
        for p in self.module.parameters():
            h = torch.empty(p.shape, dtype=p.dtype, pin_memory=True)
            h.copy_(p.data, non_blocking=True)
            self._host_params.append((p, h))
            p.data = h
        torch.cuda.current_stream(self.device).synchronize()

    def load_params(self) -> None:
        if self._host_params is None:
            return
        for p, h in self._host_params:
            p.data = h.to(self.device, non_blocking=True)
        self._host_params = None

    def _want_symmetric(self, actor_cfg, device, group) -> bool:
        """``fsdp_config.fused_collectives``: "auto" (on for NCCL ranks of one node), "on", "off"."""
        mode = str(getattr(actor_cfg.fsdp_config, "fused_collectives", "auto")).lower()
        if mode in ("off", "false", "none") or device.type != "cuda" or self.world < 2:
            return False
        from verl_omni_b200.parallel import symm_mem

        ok = symm_mem.available(group)
        if mode in ("on", "true") and not ok:
            raise RuntimeError("fused_collectives=on needs NCCL ranks on one node")
        return ok

    # ------------------------------------------------------------------ modes
    def train_mode(self):
        self.module.train()
        return self

    def eval_mode(self):
        self.module.eval()
        return self

    def zero_grad(self) -> None:
        for f in self._flats():
            f.zero_grad()

    # ------------------------------------------------------------------ optimizer
    def optimizer_step(self) -> torch.Tensor:
        """Reduce-scatter grads, clip by global norm, AdamW on the shard, all-gather bf16 weights.

        Returns the global grad norm as a device scalar (non-finite -> the update is skipped on device).
        """
        self._before_update()
        try:
            return self._optimizer_step()
        finally:
            self._after_update()

    def _optimizer_step(self) -> torch.Tensor:
        fp = self.flat
        oc = self.cfg.optim
        if fp.symm_grad is not None:
            from verl_omni_b200.parallel.symm_mem import fused_optimizer_step

            self.opt_step += 1
            norm = fused_optimizer_step(
                fp.symm_flat, fp.symm_grad, fp.shard_lo, fp.shard_size, fp.master, fp.grad_shard, fp.exp_avg,
                fp.exp_avg_sq, lr=self.sched.lr(), betas=(float(oc.betas[0]), float(oc.betas[1])),
                eps=float(oc.eps), weight_decay=float(oc.weight_decay), step=self.opt_step,
                max_norm=float(self.cfg.grad_clip if self.cfg.grad_clip is not None else oc.clip_grad),
                group=self.group)
            self.sched.step()
            fp.zero_grad()
            self.last_grad_norm = norm
            return norm
        D.reduce_scatter_into(fp.grad_shard, fp.main_grad, self.group)
        if self.replica_group is not None:  # HSDP: average the shard over the replicas
            D.all_reduce(fp.grad_shard, group=self.replica_group)
        if self.world * self.n_replicas > 1:
            fp.grad_shard.mul_(1.0 / (self.world * self.n_replicas))
        flats = [fp]
        ef = self.eflat
        if ef is not None:
            # an expert's gradient already sums the contributions of every rank of its EP group (the exchange
            # backward); summing over the ranks holding the same experts and dividing by the data-parallel size
            # (the world, or the ranks of one pipeline stage) gives the same mean as the dense parameters
            D.reduce_scatter_into(ef.grad_shard, ef.main_grad, ef.group)
            ef.grad_shard.mul_(1.0 / (D.world_size() // self.pp_size))
            flats.append(ef)
        self.opt_step += 1
        lr = self.sched.lr()
        b1, b2 = float(oc.betas[0]), float(oc.betas[1])
        max_norm = float(self.cfg.grad_clip if self.cfg.grad_clip is not None else oc.clip_grad)
        # the dense and expert shards partition the parameters over the world: one all-reduce of the local
        # squared norms gives the global norm
        norm_group = self.group if (ef is None and self.pp_size == 1) else None
        if fp.master.is_cuda:
            sq = ext().sq_norm(fp.grad_shard)
            if ef is not None:
                sq = sq + ext().sq_norm(ef.grad_shard)
            D.all_reduce(sq, group=norm_group)
            for f in flats:
                ext().adamw_flat(f.master, f.grad_shard, f.exp_avg, f.exp_avg_sq, f.shard_view(), lr, b1, b2,
                                 float(oc.eps), float(oc.weight_decay), self.opt_step, max_norm, sq, 1.0)
        else:
            sq = sum((f.grad_shard.double() ** 2).sum() for f in flats).float().reshape(1)
            D.all_reduce(sq, group=norm_group)
            norm = float(sq.sqrt())
            if math.isfinite(norm):
                coef = min(1.0, max_norm / (norm + 1e-6)) if max_norm > 0 else 1.0
                for f in flats:
                    _adamw_torch(f.master, f.grad_shard * coef, f.exp_avg, f.exp_avg_sq, lr, b1, b2, float(oc.eps),
                                 float(oc.weight_decay), self.opt_step)
                    f.shard_view().copy_(f.master.to(f.dtype))
        for f in flats:
            D.all_gather_into(f.flat, f.shard_view().clone() if f.world > 1 else f.shard_view(), f.group)
            f.zero_grad()
        self.sched.step()
        self.last_grad_norm = sq.sqrt()
        return self.last_grad_norm

    def lr(self) -> float:
        return self.sched.lr() if self.sched is not None else 0.0

    # ------------------------------------------------------------------ weights
    def get_per_tensor_param(self) -> Iterable[tuple[str, torch.Tensor]]:
        """(name, bf16 full tensor) pairs for the rollout engine (already replicated: no gather)."""
        return self.flat.param_views(self.flat.flat)

    def load_full_state(self, state: dict) -> None:
        """Load full fp32/bf16 tensors by name into master shards and the compute buffer."""
        fp = self.flat
        full = torch.zeros(fp.padded, dtype=torch.float32, device=self.device)
        for n, o, k in zip(fp.names, fp.offsets, fp.numels):
            if n in state:
                full[o:o + k].copy_(state[n].reshape(-1).to(full.device, torch.float32))
            else:
                full[o:o + k].copy_(fp.flat[o:o + k].float())
        fp.master.copy_(full[fp.shard_lo:fp.shard_lo + fp.shard_size])
        fp.flat.copy_(full.to(fp.dtype))

    # ------------------------------------------------------------------ checkpoints
    def save_checkpoint(self, local_path: str, global_step: int = 0, save_contents=("model", "optimizer", "extra"),
                        hf_export: bool = False) -> None:
        self._before_update()  # offloaded optimizer state back on the device for the collectives below
        try:
            self._save_checkpoint(local_path, global_step, save_contents, hf_export)
        finally:
            self._after_update()

    def load_checkpoint(self, local_path: str, load_contents=("model", "optimizer", "extra")) -> dict:
        self._before_update()
        try:
            return self._load_checkpoint(local_path, load_contents)
        finally:
            self._after_update()

    def _save_checkpoint(self, local_path: str, global_step: int, save_contents, hf_export: bool) -> None:
        os.makedirs(local_path, exist_ok=True)
        hf_export = hf_export or "hf_model" in save_contents  # verl's checkpoint-contents name for the HF export
        W, r = self.world, self.rank
        fp = self.flat
        # HSDP: every replica holds the same shards; replica 0 writes them
        writer = self.replica_group is None or D.rank() // self.world == 0
        if "model" in save_contents:
            # each rank writes its own slice of the flat fp32 master as it lies in memory (no gather); the
            # per-parameter layout travels with it so any world size can re-shard on load
            if writer:
                torch.save({"layout": "flat", "master": fp.master.detach().cpu(), "shard_lo": fp.shard_lo,
                            "numel": fp.numel, "padded": fp.padded, "names": list(fp.names),
                            "offsets": list(fp.offsets), "numels": list(fp.numels),
                            "shapes": [tuple(sh) for sh in fp.shapes], "world_size": W},
                           os.path.join(local_path, f"model_world_size_{W}_rank_{r}.pt"))
            if hf_export:
                full = fp.full_master()  # the only gather: the exported file holds every parameter
                if r == 0 and writer:
                    from safetensors.torch import save_file

                    from verl_omni_b200.models import hf_io

                    hf_dir = os.path.join(local_path, "huggingface")
                    named = dict(fp.param_views(full))
                    if hf_io.supported(self.module):  # diffusers parameter names and layouts
                        hf_io.save_diffusers(named, self.module, hf_dir)
                    else:
                        os.makedirs(hf_dir, exist_ok=True)
                        save_file({n: v.to(torch.bfloat16).contiguous().cpu() for n, v in named.items()},
                                  os.path.join(hf_dir, "diffusion_pytorch_model.safetensors"))
                del full
        if "optimizer" in save_contents and writer:
            torch.save({"exp_avg": fp.exp_avg.cpu(), "exp_avg_sq": fp.exp_avg_sq.cpu(), "step": self.opt_step,
                        "padded": fp.padded, "world_size": W},
                       os.path.join(local_path, f"optim_world_size_{W}_rank_{r}.pt"))
        if "extra" in save_contents and writer:
            torch.save({"lr_scheduler": self.sched.state_dict(), "global_step": global_step,
                        "rng": torch.get_rng_state(),
                        "cuda_rng": torch.cuda.get_rng_state() if torch.cuda.is_available() else None},
                       os.path.join(local_path, f"extra_state_world_size_{W}_rank_{r}.pt"))
        if self.eflat is not None:
            # expert-parallel slices: every rank writes its own experts' master shard and moments (reloaded at
            # the same world size and expert layout)
            ef = self.eflat
            torch.save({"names": ef.names, "shapes": ef.shapes, "master": ef.master.cpu(), "exp_avg": ef.exp_avg.cpu(),
                        "exp_avg_sq": ef.exp_avg_sq.cpu(), "group_world": ef.world, "group_rank": ef.rank},
                       os.path.join(local_path, f"expert_world_size_{D.world_size()}_rank_{D.rank()}.pt"))
        if r == 0 and writer:
            with open(os.path.join(local_path, "fsdp_config.json"), "w") as f:
                json.dump({"FSDP_version": 2, "world_size": W, "layout": "flat-shard-adamw",
                           "replicas": self.n_replicas}, f)
        D.barrier()

    def _load_checkpoint(self, local_path: str, load_contents) -> dict:
        with open(os.path.join(local_path, "fsdp_config.json")) as f:
            meta = json.load(f)
        Wsaved = int(meta["world_size"])
        fp = self.flat
        info: dict = {}
        if "model" in load_contents:
            own = torch.load(os.path.join(local_path, f"model_world_size_{Wsaved}_rank_{self.rank}.pt"),
                             map_location="cpu") if self.rank < Wsaved else None
            if (Wsaved == self.world and own is not None and own.get("layout") == "flat"
                    and own["names"] == list(fp.names) and own["padded"] == fp.padded):
                # same world size and layout: the shard goes straight back; compute weights are re-gathered
                fp.master.copy_(own["master"].to(self.device))
                D.all_gather_into(fp.flat, fp.master.to(fp.dtype), self.group)
            else:
                self.load_full_state(read_full_state(local_path, Wsaved))
        if "optimizer" in load_contents:
            if Wsaved == self.world:
                o = torch.load(os.path.join(local_path, f"optim_world_size_{Wsaved}_rank_{self.rank}.pt"),
                               map_location="cpu")
                fp.exp_avg.copy_(o["exp_avg"].to(self.device))
                fp.exp_avg_sq.copy_(o["exp_avg_sq"].to(self.device))
                self.opt_step = int(o["step"])
            else:  # re-shard the moments through the full flat layout
                full_m, full_v = [], []
                for i in range(Wsaved):
                    o = torch.load(os.path.join(local_path, f"optim_world_size_{Wsaved}_rank_{i}.pt"),
                                   map_location="cpu")
                    full_m.append(o["exp_avg"])
                    full_v.append(o["exp_avg_sq"])
                    self.opt_step = int(o["step"])
                m, v = torch.cat(full_m), torch.cat(full_v)
                lo, n = fp.shard_lo, fp.shard_size
                fp.exp_avg.zero_()
                fp.exp_avg_sq.zero_()
                k = max(0, min(n, fp.numel - lo, m.numel() - lo))
                if k > 0:
                    fp.exp_avg[:k].copy_(m[lo:lo + k].to(self.device))
                    fp.exp_avg_sq[:k].copy_(v[lo:lo + k].to(self.device))
        if self.eflat is not None:
            ef = self.eflat
            path = os.path.join(local_path, f"expert_world_size_{D.world_size()}_rank_{D.rank()}.pt")
            if not os.path.exists(path):
                raise FileNotFoundError(f"expert-parallel checkpoint {path} (expert slices reload at the same "
                                        "world size and expert layout)")
            e = torch.load(path, map_location="cpu")
            if list(e["names"]) != list(ef.names) or e["group_world"] != ef.world:
                raise ValueError("expert-parallel checkpoint layout differs from this run's")
            ef.master.copy_(e["master"].to(self.device))
            ef.exp_avg.copy_(e["exp_avg"].to(self.device))
            ef.exp_avg_sq.copy_(e["exp_avg_sq"].to(self.device))
            full = torch.empty(ef.padded, dtype=torch.float32, device=self.device)
            D.all_gather_into(full, ef.master, ef.group)
            ef.flat.copy_(full.to(ef.dtype))
        if "extra" in load_contents:
            r = self.rank if Wsaved == self.world else 0
            e = torch.load(os.path.join(local_path, f"extra_state_world_size_{Wsaved}_rank_{r}.pt"),
                           map_location="cpu", weights_only=False)
            self.sched.load_state_dict(e["lr_scheduler"])
            info["global_step"] = e.get("global_step", 0)
        D.barrier(self.group)
        return info


def read_full_state(ckpt_dir: str, world_size: Optional[int] = None) -> dict:
    """Every parameter of a sharded actor checkpoint as a full CPU tensor, by name.

    Reads ``model_world_size_{W}_rank_{r}.pt`` for all ``r``: the flat layout (each rank's slice of the
    flat fp32 master plus the name / offset / shape table) or per-parameter dim-0 shards.
    """
    import glob
    import re

    if world_size is None:
        files = glob.glob(os.path.join(ckpt_dir, "model_world_size_*_rank_*.pt"))
        if not files:
            raise FileNotFoundError(f"no model_world_size_*_rank_*.pt under {ckpt_dir}")
        world_size = int(re.search(r"model_world_size_(\d+)_rank_", os.path.basename(files[0])).group(1))
    parts = [torch.load(os.path.join(ckpt_dir, f"model_world_size_{world_size}_rank_{i}.pt"), map_location="cpu")
             for i in range(world_size)]
    if parts[0].get("layout") == "flat":
        flat = torch.cat([p["master"] for p in parts])
        meta = parts[0]
        return {n: flat[o:o + k].view(sh).clone()
                for n, o, k, sh in zip(meta["names"], meta["offsets"], meta["numels"], meta["shapes"])}
    out = {}
    for n in parts[0]["params"]:
        pieces = [p["params"][n] for p in parts]
        out[n] = torch.cat(pieces, 0) if pieces[0].ndim else pieces[0]
    return out


def _adamw_torch(p, g, m, v, lr, b1, b2, eps, wd, step):
    p.mul_(1 - lr * wd)
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    bc1 = 1 - b1 ** step
    bc2 = 1 - b2 ** step
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)
