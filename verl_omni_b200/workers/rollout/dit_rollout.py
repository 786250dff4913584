"""In-process DiT rollout engine (replaces the vLLM-Omni diffusion server of the reference).

For a batch of requests it runs the reverse-SDE denoising loop on the current policy weights
(shared with the trainer when colocated), recording the fp32 trajectory inside the SDE window,
per-step log-probs and timesteps -- the ``DiffusionOutput`` contract of
``verl_omni/workers/rollout/replica.py:20`` / ``vllm_omni_async_server.py:638-778``:

* request batching: requests are packed into forward batches of at most ``max_num_seqs``
  (cond+uncond counted twice under CFG);
* per-request seeds: the Gaussian draw of row ``i`` at step ``t`` comes from Philox keyed by
  ``(seed, i, t)`` inside the fused SDE kernel, so a rollout is reproducible from its seed;
* SDE window: steps outside ``[w0, w0+W)`` take the deterministic ODE update (noise 0) and are not
  recorded (FlowGRPO fast / MixGRPO windows, ``verl_omni/pipelines/request_batch.py:32-56``);
* sleep / wake: activations and cached buffers are dropped between rollouts (``free_cache_engine``);
* abort: ``abort()`` makes the running ``generate`` return the finished requests plus synthesized
  aborted outputs (``vllm_omni_async_server.py:790-941``).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Callable, Optional

import numpy as np
import torch

from verl_omni_b200.ops.sde import normal_rows
from verl_omni_b200.pipelines.model_base import DiffusionModelBase
from verl_omni_b200.utils.dataproto import DataProto


# Philox counter offset of the initial latent noise (SDE step t uses offset t)
_INIT_NOISE_OFFSET = 0x7FFFFFFF


def select_sde_window(algo_cfg, T: int, global_step: int, seed: int = 0) -> tuple[int, int]:
    """(start, size) of the SDE window; whole schedule when ``sde_window_size`` is unset.

    ``random``: start drawn uniformly from ``sde_window_range`` (default ``[0, T-W]``) with a seeded
    generator; ``progressive`` (MixGRPO): the window slides by one step every ``iters_per_group``
    optimizer steps and wraps around.
    """
    W = algo_cfg.sde_window_size
    if not W:
        return 0, T
    W = min(int(W), T)
    lo, hi = 0, T - W
    if algo_cfg.sde_window_range:
        lo, hi = int(algo_cfg.sde_window_range[0]), min(int(algo_cfg.sde_window_range[1]), T - W)
    if algo_cfg.sample_strategy == "progressive":
        span = hi - lo + 1
        return lo + (global_step // max(1, algo_cfg.iters_per_group)) % span, W
    g = np.random.default_rng(int(algo_cfg.sde_window_seed) * 1_000_003 + int(seed) * 7919 + global_step)
    return int(g.integers(lo, hi + 1)), W


@dataclass
class RolloutRequest:
    cond: dict
    neg_cond: Optional[dict] = None
    seed: int = 0


class DiTRolloutEngine:
    def __init__(self, module, adapter: type[DiffusionModelBase], rollout_cfg, model_cfg, *, device,
                 latent_shape: tuple, decoder: Optional[Callable] = None, sched_seq_len: Optional[int] = None):
        self.module = module
        self.adapter = adapter
        self.cfg = rollout_cfg
        self.model_cfg = model_cfg
        self.device = device
        self.latent_shape = tuple(latent_shape)
        self.decoder = decoder
        T = rollout_cfg.pipeline.num_inference_steps
        seq = sched_seq_len or int(np.prod(self.latent_shape[-2:])) // 4
        self._sched_seq = seq
        self.scheduler = adapter.build_scheduler(T, image_seq_len=seq, device=device)
        self._schedulers = {T: self.scheduler}
        self._abort = threading.Event()
        self.sleeping = False

    # ------------------------------------------------------------------ lifecycle
    def sleep(self) -> None:
        self.sleeping = True
        if self.cfg.free_cache_engine and torch.cuda.is_available():
            torch.cuda.empty_cache()

    def wake_up(self) -> None:
        self.sleeping = False

    def abort(self) -> None:
        self._abort.set()

    def update_weights(self, named_tensors) -> int:
        """Load (name, tensor) pairs into the rollout module; returns bytes copied.

        Colocated engines share parameter storage with the trainer, so tensors that already alias
        the module's parameters are skipped (zero-copy)."""
        params = dict(self.module.named_parameters())
        n = 0
        with torch.no_grad():
            for name, t in named_tensors:
                p = params.get(name)
                if p is None or p.data_ptr() == t.data_ptr():
                    continue
                p.copy_(t)
                n += t.numel() * t.element_size()
        return n

    # ------------------------------------------------------------------ generate
    @torch.no_grad()
    def generate(self, batch: DataProto, *, seed: int = 0, global_step: int = 0, record_logprobs: bool = True,
                 decode: bool = True, row_seeds: Optional[torch.Tensor] = None,
                 window: Optional[tuple[int, int]] = None, noise_level: Optional[float] = None,
                 sde_type: Optional[str] = None, guidance_scale: Optional[float] = None,
                 num_inference_steps: Optional[int] = None) -> DataProto:
        """``batch`` holds the conditioning tensors (adapter ``cond_keys``, optional ``negative_*``).

        ``row_seeds`` (int64 [B]) keys each sample's initial noise and SDE noise by its own seed, so
        a sample's trajectory does not depend on how requests were packed into device batches.
        ``window`` / ``noise_level`` / ``sde_type`` / ``guidance_scale`` override the configured
        values for this call (validation sampling, request-level parameters); ``num_inference_steps``
        samples with a schedule of that many steps (built once per length).
        """
        if self.sleeping:
            self.wake_up()
        self._abort.clear()
        cfg, algo = self.cfg, self.cfg.algo
        T = int(num_inference_steps or cfg.pipeline.num_inference_steps)
        sched_T = self._scheduler_for(T)
        w0, W = window if window is not None else select_sde_window(algo, T, global_step, seed)
        B = len(batch)
        guidance = cfg.pipeline.guidance_scale if guidance_scale is None else guidance_scale
        nl = algo.noise_level if noise_level is None else float(noise_level)
        st = algo.sde_type if sde_type is None else sde_type
        cfg_mult = 2 if (guidance is not None and guidance > 1.0) else 1
        mbs = max(1, min(B, cfg.max_num_seqs // cfg_mult))
        sched = self.scheduler
        sig = sched.sigmas
        chunks = []
        for s in range(0, B, mbs):
            if self._abort.is_set():
                break
            mb = batch.select_idxs(slice(s, min(B, s + mbs)))
            rs = row_seeds[s:min(B, s + mbs)] if row_seeds is not None else None
            chunks.append(self._run_chunk(mb, T, w0, W, seed * 1_000_003 + s, guidance, record_logprobs, rs, nl, st,
                                          sched_T))
        done = sum(len(c) for c in chunks)
        out = DataProto.concat(chunks) if chunks else DataProto()
        if done < B:  # aborted: synthesize aborted outputs for the unfinished requests
            rest = B - done
            abort = {k: torch.zeros((rest,) + v.shape[1:], dtype=v.dtype, device=v.device)
                     for k, v in (out.batch.items() if chunks else [])}
            out = DataProto.concat([out, DataProto(abort)]) if chunks else DataProto()
            out.meta_info["aborted"] = np.array([False] * done + [True] * rest)
        if decode and self.decoder is not None and len(out):
            out.batch["images"] = self.decode(out.batch["final_latents"])
        out.meta_info.update({"sde_window": (w0, W), "num_inference_steps": T})
        return out

    def decode(self, latents: torch.Tensor, chunk: int = 8) -> torch.Tensor:
        imgs = [self.decoder(latents[i:i + chunk]) for i in range(0, latents.shape[0], chunk)]
        return torch.cat(imgs, 0)

    def _scheduler_for(self, T: int):
        if T not in self._schedulers:
            self._schedulers[T] = self.adapter.build_scheduler(T, image_seq_len=self._sched_seq, device=self.device)
        return self._schedulers[T]

    def _run_chunk(self, mb: DataProto, T: int, w0: int, W: int, seed: int, guidance, record: bool,
                   row_seeds: Optional[torch.Tensor], noise_level: float, sde_type: str, sched=None) -> DataProto:
        keys = self.adapter.cond_keys()
        cond = {k: mb.batch[k].to(self.device) for k in keys}
        neg = None
        if guidance is not None and guidance > 1.0 and ("negative_" + keys[0]) in mb.batch:
            neg = {k: mb.batch["negative_" + k].to(self.device) for k in keys}
        b = len(mb)
        if row_seeds is not None:
            row_seeds = row_seeds.to(device=self.device, dtype=torch.int64)
            x = normal_rows(row_seeds, self.latent_shape, _INIT_NOISE_OFFSET, self.device)
        else:
            x = self._initial_noise(b, seed)
        sched = sched or self.scheduler
        traj = [x] if w0 == 0 else []
        logps, steps = [], []
        for t in range(T):
            tt = sched.timesteps[t].expand(b).to(self.device)
            v = self.adapter.predict(self.module, x, tt, cond, neg, guidance)
            in_window = w0 <= t < w0 + W
            nl = noise_level if in_window else 0.0
            out = sched.sample_previous_step(x.float(), v.float(), step_index=t, noise_level=nl,
                                             sde_type=sde_type if in_window else "sde",
                                             seed=seed, noise_offset=t, return_logprobs=in_window and record,
                                             row_seeds=row_seeds)
            if not in_window:
                x = out.prev_sample_mean
            else:
                x = out.prev_sample
            if in_window:
                if record:
                    logps.append(out.log_prob)
                steps.append(t)
                traj.append(x)
            elif t + 1 == w0:
                traj.append(x)
        res = {
            "latents": torch.stack(traj, 1),  # [b, W+1, ...] fp32
            "step_index": torch.tensor(steps, device=self.device).expand(b, W).contiguous(),
            "timesteps": sched.timesteps.to(self.device)[torch.tensor(steps, device=self.device)].expand(b, W).contiguous(),
            "final_latents": x,
        }
        if record:
            res["rollout_log_probs"] = torch.stack(logps, 1)
        for k, v in cond.items():
            res[k] = v
        if neg is not None:
            for k, v in neg.items():
                res["negative_" + k] = v
        return DataProto(res)

    def _initial_noise(self, b: int, seed: int) -> torch.Tensor:
        g = torch.Generator(device="cpu")
        g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
        return torch.randn((b,) + self.latent_shape, generator=g).to(self.device)


class StepwiseBatcher:
    """Step-level continuous batching over a :class:`DiTRolloutEngine` (the step-exec interface of the
    reference's vLLM-Omni adapters, ``pipelines/qwen_image_flow_grpo/vllm_omni_rollout_adapter.py:199-594``:
    ``prepare_encode`` / ``step_scheduler`` / ``denoise_step`` / ``post_decode``).

    Requests join a pool as they are submitted and each carries its own step counter; every iteration runs
    ONE denoising step for up to ``max_num_seqs`` pooled requests in a single forward (rows at different
    timesteps: the models take per-row timesteps), then the SDE update per distinct step (each row's noise
    is keyed by its own seed and its step, so a request's trajectory does not depend on who shared its
    batches).  A request that finishes its ``T`` steps leaves at once and a waiting one takes its slot, so
    the device batch stays full while requests arrive and finish at different times.
    """

    def __init__(self, engine: "DiTRolloutEngine", max_num_seqs: Optional[int] = None, noise_level: Optional[float] = None,
                 sde_type: Optional[str] = None, guidance_scale: Optional[float] = None):
        self.e = engine
        self.max = int(max_num_seqs or engine.cfg.max_num_seqs)
        algo = engine.cfg.algo
        self.nl = algo.noise_level if noise_level is None else float(noise_level)
        self.st = algo.sde_type if sde_type is None else sde_type
        self.guidance = engine.cfg.pipeline.guidance_scale if guidance_scale is None else guidance_scale
        self.T = int(engine.cfg.pipeline.num_inference_steps)
        self.waiting: list = []
        self.active: list = []
        self.finished: dict = {}
        self.iterations = 0
        self.rows_per_iteration: list = []

    def submit(self, request_id, cond: dict, seed: int) -> None:
        """``cond``: one request's conditioning tensors (leading dim 1)."""
        self.waiting.append({"id": request_id, "cond": cond, "seed": int(seed)})

    def _admit(self) -> None:
        e = self.e
        while self.waiting and len(self.active) < self.max:
            r = self.waiting.pop(0)
            rs = torch.tensor([r["seed"]], dtype=torch.int64, device=e.device)
            r["row_seed"] = rs
            r["x"] = normal_rows(rs, e.latent_shape, _INIT_NOISE_OFFSET, e.device)
            r["t"] = 0
            r["traj"], r["logps"] = [r["x"]], []
            self.active.append(r)

    @torch.no_grad()
    def step(self) -> int:
        """One iteration; returns the number of requests that finished in it."""
        self._admit()
        if not self.active:
            return 0
        e, sched = self.e, self.e.scheduler
        rows = self.active[:self.max]
        keys = e.adapter.cond_keys()
        x = torch.cat([r["x"] for r in rows], 0)
        cond = {k: torch.cat([r["cond"][k].to(e.device) for r in rows], 0) for k in keys}
        tvec = torch.tensor([r["t"] for r in rows], device=e.device)
        tt = sched.timesteps.to(e.device)[tvec]
        v = e.adapter.predict(e.module, x, tt, cond, None, self.guidance)
        self.iterations += 1
        self.rows_per_iteration.append(len(rows))
        done = 0
        steps_now = [r["t"] for r in rows]  # grouped before any row advances
        for t in sorted(set(steps_now)):
            idx = [i for i, ti in enumerate(steps_now) if ti == t]
            sel = torch.tensor(idx, device=e.device)
            rs = torch.cat([rows[i]["row_seed"] for i in idx], 0)
            out = sched.sample_previous_step(x[sel].float(), v[sel].float(), step_index=t, noise_level=self.nl,
                                             sde_type=self.st, noise_offset=t, return_logprobs=True, row_seeds=rs)
            for j, i in enumerate(idx):
                r = rows[i]
                r["x"] = out.prev_sample[j:j + 1]
                r["traj"].append(r["x"])
                r["logps"].append(out.log_prob[j:j + 1])
                r["t"] += 1
        for r in list(rows):
            if r["t"] >= self.T:
                self.active.remove(r)
                self.finished[r["id"]] = self._result(r)
                done += 1
        return done

    def _result(self, r) -> DataProto:
        e = self.e
        T = self.T
        res = {"latents": torch.stack(r["traj"], 1)[0:1].reshape((1, T + 1) + tuple(e.latent_shape)),
               "step_index": torch.arange(T, device=e.device)[None],
               "timesteps": e.scheduler.timesteps.to(e.device)[:T][None],
               "final_latents": r["x"], "rollout_log_probs": torch.cat(r["logps"], 0).reshape(1, T)}
        res.update({k: v.to(e.device) for k, v in r["cond"].items()})
        return DataProto(res)

    def run(self) -> dict:
        """Steps until every submitted request has finished; returns ``{request_id: DataProto row}``."""
        while self.waiting or self.active:
            self.step()
        return self.finished
