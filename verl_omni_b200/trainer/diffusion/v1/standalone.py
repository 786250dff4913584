"""Standalone-rollout topology: trainer ranks and rollout ranks in one job, weights pushed across GPUs.

Counterpart of the reference's separate-async trainer with its own rollout pool
(``verl_omni/trainer/diffusion/v1/trainer_separate_async.py:104-160``) and checkpoint engine
(``verl_omni/workers/checkpoint_engine.py:25-68``).  With ``trainer.v1.standalone_rollout_ranks = R``
the last ``R`` ranks of the job are rollout ranks; the first ``W - R`` train (their collectives run on a
trainer-only group).  Trainer ``t`` is fed by rollout rank ``W - R + t % R``.

Schedule (one-step off-policy, no host polling): a rollout rank generates batch ``k`` for each of its
trainers and sends it; before generating batch ``k`` (``k > 2``) it joins the weight push that follows
trainer step ``k - 2`` when that step is a sync step (every ``trainer.v1.parameter_sync_step`` steps).
Trainers receive batch ``s``, train on it, and push after sync steps.  Rollout of batch ``s + 1`` overlaps
training on batch ``s``; every sample carries the weight version it was generated with and the replay
buffer reports the staleness.

The push: the rollout ranks keep their policy weights in one flat bf16 buffer with the trainer's layout.
On CUDA ranks of one node that buffer is a symmetric (peer-mapped) allocation over the push group
(trainer 0 + rollout ranks) and trainer 0 writes every rollout rank's buffer with one peer-store kernel
(``parallel/weight_sync.push``, ``csrc/symm.cu`` ``peer_push``); elsewhere the flat buffer is broadcast.
Batches travel rollout -> trainer as point-to-point sends (a pickled header, then the tensors).
"""

from __future__ import annotations

import pickle
import time
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from verl_omni_b200.parallel import dist as D
from verl_omni_b200.utils.dataproto import DataProto

_TOPO = None


class Topology:
    """Rank roles and process groups of a job with ``R`` standalone rollout ranks (created by every rank)."""

    def __init__(self, rollout_ranks: int):
        W = D.world_size()
        R = int(rollout_ranks)
        if not 0 < R < W:
            raise ValueError(f"standalone_rollout_ranks={R} must leave at least one trainer rank of {W}")
        self.W, self.R, self.T = W, R, W - R
        self.rank = D.rank()
        self.is_rollout = self.rank >= self.T
        # every rank creates every group, in the same order (new_group is collective over the world)
        self.trainer_group = dist.new_group(list(range(self.T)))
        self.push_ranks = [0] + list(range(self.T, W))
        self.push_group = dist.new_group(self.push_ranks)

    def rollout_of(self, trainer: int) -> int:
        return self.T + trainer % self.R

    def trainers_of(self, rollout: int) -> list[int]:
        return [t for t in range(self.T) if self.rollout_of(t) == rollout]


def topology(rollout_ranks: int) -> Topology:
    global _TOPO
    if _TOPO is None:
        _TOPO = Topology(rollout_ranks)
    return _TOPO


# ---------------------------------------------------------------------------------------- batch transport
def _p2p_device(dev: torch.device) -> torch.device:
    return dev if (dist.get_backend() == "nccl") else torch.device("cpu")


def send_batch(batch: DataProto, dst: int, version: int, device: torch.device) -> list:
    """Queues the batch's sends (non-blocking); returns ``(works, buffers)`` to wait on later.  The sender
    must not block here: its trainer may be inside a weight push that the sender joins next."""
    keys = sorted(batch.batch.keys())
    header = {"keys": keys, "shapes": [tuple(batch.batch[k].shape) for k in keys],
              "dtypes": [str(batch.batch[k].dtype).split(".")[-1] for k in keys],
              "non_tensor": {k: list(v) for k, v in batch.non_tensor_batch.items()}, "version": int(version)}
    raw = torch.frombuffer(bytearray(pickle.dumps(header)), dtype=torch.uint8)
    pd = _p2p_device(device)
    bufs = [torch.tensor([raw.numel()], dtype=torch.int64, device=pd), raw.to(pd)]
    bufs += [batch.batch[k].contiguous().to(pd) for k in keys]
    works = [dist.isend(b, dst) for b in bufs]
    return [works, bufs]


def wait_sends(pending: list) -> None:
    works, _ = pending
    for w in works:
        w.wait()


def recv_batch(src: int, device: torch.device) -> tuple[DataProto, int]:
    pd = _p2p_device(device)
    n = torch.zeros(1, dtype=torch.int64, device=pd)
    dist.recv(n, src)
    raw = torch.empty(int(n.item()), dtype=torch.uint8, device=pd)
    dist.recv(raw, src)
    header = pickle.loads(raw.cpu().numpy().tobytes())
    tensors = {}
    for k, shp, dt in zip(header["keys"], header["shapes"], header["dtypes"]):
        t = torch.empty(shp, dtype=getattr(torch, dt), device=pd)
        dist.recv(t, src)
        tensors[k] = t.to(device)
    nt = {k: np.array(v, dtype=object) for k, v in header["non_tensor"].items()}
    return DataProto(tensors, nt), int(header["version"])


# ---------------------------------------------------------------------------------------- weight push
def flat_layout(module: torch.nn.Module, trainable: list[str]) -> tuple[list[str], list[int], list[tuple], int]:
    """Names, element offsets, shapes and size of the trainer's flat buffer for the parameters named in
    ``trainable`` (the ``FlatParams`` layout: module order, every parameter on a 16-element boundary)."""
    keep = set(trainable)
    names, offs, shapes, off = [], [], [], 0
    for n, p in module.named_parameters():
        if n in keep:
            names.append(n)
            offs.append(off)
            shapes.append(tuple(p.shape))
            off += (p.numel() + 15) // 16 * 16
    return names, offs, shapes, off


class PushChannel:
    """Trainer 0 -> rollout ranks weight transfer over the push group.  Every member calls ``push`` at the
    same points; trainer 0 passes its flat bf16 buffer, rollout ranks receive into ``self.buf``."""

    def __init__(self, topo: Topology, numel: int, dtype, device: torch.device):
        self.topo, self.numel, self.device = topo, int(numel), device
        self.symm = None
        self.buf = None
        if device.type == "cuda":
            try:
                from verl_omni_b200.parallel.symm_mem import SymmetricBuffer, available

                if available(topo.push_group):
                    self.symm = SymmetricBuffer(self.numel, dtype, device, topo.push_group)
            except Exception:  # noqa: BLE001 - fall back to broadcast, agreed below
                self.symm = None
        ok = torch.tensor([1 if (self.symm is not None or device.type != "cuda") else 0], dtype=torch.int32,
                          device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=topo.push_group)
        if device.type == "cuda" and int(ok.item()) == 0 and self.symm is not None:
            self.symm.close(collective=False)
            self.symm = None
        if self.symm is not None:
            self.buf = self.symm.tensor
            from verl_omni_b200.parallel import weight_sync

            slots = list(range(1, len(topo.push_ranks)))  # push-group ranks of the rollout ranks
            self.plan = weight_sync.plan_replicate(self.numel * self.buf.element_size(), slots)
        elif topo.is_rollout:
            self.buf = torch.zeros(self.numel, dtype=dtype, device=device)
        self.bytes_pushed = 0

    def push(self, src: Optional[torch.Tensor] = None) -> float:
        """Returns the seconds the push took on this rank."""
        t0 = time.perf_counter()
        if self.symm is not None:
            from verl_omni_b200.parallel import weight_sync
            from verl_omni_b200.parallel.symm_mem import stream_barrier

            # every rollout rank has finished the work that reads its weights before the peer stores land
            stream_barrier(self.topo.push_group, self.device)
            if self.topo.rank == 0:
                weight_sync.push(src[:self.numel].contiguous(), self.symm.peer_ptrs, self.plan, self.topo.push_group)
            else:
                stream_barrier(self.topo.push_group, self.device)  # ... and they start after the stores
        else:
            t = src[:self.numel] if self.topo.rank == 0 else self.buf
            if self.device.type == "cuda" or dist.get_backend() == "gloo":
                t = t.contiguous()
                dist.broadcast(t, 0, group=self.topo.push_group)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.bytes_pushed += self.numel * 2 * (len(self.topo.push_ranks) - 1)
        return time.perf_counter() - t0


# ---------------------------------------------------------------------------------------- rollout rank
class RolloutRank:
    """The rollout side: the trainer's model / rollout engine / reward / prompt stream, with the policy
    weights living in the push buffer."""

    def __init__(self, config, topo: Topology):
        from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer

        self.config, self.topo = config, topo
        # the trainer object in rollout-only mode gives the identical model (same seed), the rollout engine, the
        # reward and the prompt stream (sharded over the trainer ranks), with no optimizer state or collectives
        self.core = PolicyGradientTrainer(config, rollout_only=True, dp_override=topo.T)
        self.device = self.core.device
        module = self.core.actor.module
        names, offs, shapes, numel = flat_layout(module, self.core.trainable_names)
        self.channel = PushChannel(topo, numel, self.core.actor.engine.dtype, self.device)
        params = dict(module.named_parameters())
        for n, o, s in zip(names, offs, shapes):  # the module's weights alias the push buffer
            k = int(torch.Size(s).numel())
            params[n].data = self.channel.buf[o:o + k].view(s)
        v1 = config.trainer.v1
        self.P = int(v1.get("parameter_sync_step", 1))
        self.steps = int(config.trainer.total_training_steps or 1)
        self.version = 0

    def serve(self) -> list[dict]:
        core, topo = self.core, self.topo
        self.channel.push()  # initial weights from trainer 0
        mine = topo.trainers_of(topo.rank)
        hist = []
        inflight: list = []  # queued sends of the previous batches (at most two batches outstanding)
        for k in range(1, self.steps + 1):
            s = k - 2
            if s >= 1 and s % self.P == 0:
                dt = self.channel.push()  # the trainers consume batch k - 1 after this push
                self.version = s
                hist.append({"rollout/push_s": dt})
            ids_all = core.sampler.next_batch()  # the global prompt batch of step k (same stream as the trainers)
            p = core.prompts_per_rank
            for t in mine:
                out = self._generate_for(ids_all[t * p:(t + 1) * p], t, k)
                inflight.append(send_batch(out, t, self.version, self.device))
            while len(inflight) > len(mine):  # batch k - 1 was received before the trainers reached push(k - 1)
                wait_sends(inflight.pop(0))
        for pend in inflight:
            wait_sends(pend)
        return hist

    @torch.no_grad()
    def _generate_for(self, ids: list[int], trainer: int, k: int) -> DataProto:
        core = self.core
        out, scores, _ = core.generate(ids, seed_step=k, uid_prefix=f"{k}-t{trainer}")
        out.batch["rm_scores"] = scores.to(out.batch["latents"].device)
        out.batch.pop("images", None)  # scored here: the trainer needs trajectories, not pixels
        return out


# ---------------------------------------------------------------------------------------- trainer rank
class StandaloneTrainerRank:
    """A trainer rank of the standalone topology: receives its batches from its rollout rank, trains on the
    trainer-only group, and (trainer 0) pushes the weights after every ``parameter_sync_step`` steps."""

    def __init__(self, config, topo: Topology):
        from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer

        self.config, self.topo = config, topo
        D.set_default_group(topo.trainer_group)  # the trainer, its engine and helpers run on the trainer ranks
        self.core = PolicyGradientTrainer(config)
        v1 = config.trainer.v1
        self.P = int(v1.get("parameter_sync_step", 1))
        self.steps = int(config.trainer.total_training_steps or 1)
        self.channel = None
        if topo.rank == 0:
            fp = self.core.actor.engine.flat
            self.channel = PushChannel(topo, fp.numel, fp.dtype, self.core.device)
        self.global_steps = 0
        self.weight_version = 0

    def _push(self) -> float:
        if self.channel is not None:
            src = self.core.actor.engine.flat.flat
            self.last_pushed = src[:self.channel.numel].detach().clone()
            return self.channel.push(src)
        return 0.0

    def fit(self, log_fn=None) -> list[dict]:
        from verl_omni_b200.utils import metrics as M

        core, topo = self.core, self.topo
        self._push()  # initial weights
        src = topo.rollout_of(topo.rank)
        hist = []
        for s in range(1, self.steps + 1):
            timer = M.PhaseTimer(core.device)
            t0 = time.perf_counter()
            core.sampler.next_batch()  # keep the sampler state in step with the rollout ranks (resume)
            with timer("wait_rollout"):
                data, version = recv_batch(src, core.device)  # complete prompt groups of this rank's share
            self.global_steps = s
            core.global_step = s
            m = core.train_on(data, data.batch["rm_scores"], timer)
            # the policy being trained is version s - 1; the batch came from version `version`
            m["training/staleness/mean"] = m["training/staleness/max"] = float(s - 1 - version)
            if s % self.P == 0 and s <= self.steps - 2:
                with timer("update_weights"):
                    m["rollout/push_s"] = self._push()
                self.weight_version = s
            m.update(M.compute_timing_metrics_diffusion(timer.timing, len(data)))
            m.update(M.compute_throughput_metrics_diffusion(time.perf_counter() - t0, len(data) * core.dp,
                                                             topo.T))
            m["training/global_step"] = s
            m["training/weight_version"] = self.weight_version
            m["training/sample_version"] = version
            hist.append(m)
            if log_fn is not None and topo.rank == 0:
                log_fn(m)
        return hist


def build_standalone(config):
    """The role object of this rank: a trainer rank or a rollout rank (``fit()`` runs either loop)."""
    topo = topology(int(config.trainer.v1.get("standalone_rollout_ranks", 0)))
    if topo.is_rollout:
        r = RolloutRank(config, topo)
        r.fit = lambda log_fn=None: r.serve()
        return r
    return StandaloneTrainerRank(config, topo)
