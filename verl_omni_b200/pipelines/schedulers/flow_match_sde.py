"""Flow-matching reverse-SDE scheduler with per-step log-probabilities.

Behavioural parity with ``verl_omni/pipelines/schedulers/flow_match_sde.py:48-321`` (which
extends diffusers' ``FlowMatchEulerDiscreteScheduler``):

* sigma schedule: ``linspace(sigma_max, sigma_min, N)`` followed by the static shift
  ``s*x/(1+(s-1)*x)`` or the dynamic (resolution dependent) shift ``e^mu/(e^mu+(1/x-1))``,
  with a trailing 0; timesteps are ``sigma * num_train_timesteps``.
* three reverse-step variants ``sde`` (FlowGRPO), ``cps`` and ``dance_sde``; the log-prob is
  averaged over all non-batch dims and optionally includes the Gaussian normaliser.

The step itself is one fused kernel on CUDA tensors (mean, Philox noise, sample, log-prob and
its per-sample reduction in a single pass over the latents); CPU tensors take the fp32 torch
path below, which is also the oracle the kernel is tested against.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from verl_omni_b200.ops import sde as sde_ops


def calculate_shift(image_seq_len: int, base_seq_len: int = 256, max_seq_len: int = 4096,
                    base_shift: float = 0.5, max_shift: float = 1.16) -> float:
    """Linear interpolation of the dynamic-shift ``mu`` in the image sequence length."""
    m = (max_shift - base_shift) / (max_seq_len - base_seq_len)
    b = base_shift - m * base_seq_len
    return image_seq_len * m + b


@dataclass
class SchedulerStepOutput:
    prev_sample: torch.Tensor
    log_prob: Optional[torch.Tensor]
    prev_sample_mean: torch.Tensor
    std_dev_t: torch.Tensor
    sqrt_dt: Optional[torch.Tensor] = None


class FlowMatchSDEDiscreteScheduler:
    def __init__(self, num_train_timesteps: int = 1000, shift: float = 3.0, use_dynamic_shifting: bool = False,
                 base_image_seq_len: int = 256, max_image_seq_len: int = 4096, base_shift: float = 0.5,
                 max_shift: float = 1.16):
        self.num_train_timesteps = num_train_timesteps
        self.shift = shift
        self.use_dynamic_shifting = use_dynamic_shifting
        self.base_image_seq_len = base_image_seq_len
        self.max_image_seq_len = max_image_seq_len
        self.base_shift = base_shift
        self.max_shift = max_shift
        t = np.linspace(1, num_train_timesteps, num_train_timesteps, dtype=np.float32)[::-1].copy()
        s = t / num_train_timesteps
        if not use_dynamic_shifting:
            s = shift * s / (1 + (shift - 1) * s)
        self.sigma_min = float(s[-1])
        self.sigma_max = float(s[0])
        self.sigmas = torch.from_numpy(np.append(s, 0.0).astype(np.float32))
        self.timesteps = self.sigmas[:-1] * num_train_timesteps
        self._step_index: Optional[int] = None

    # ------------------------------------------------------------------ schedule
    def _shift_sigmas(self, sigmas: np.ndarray, mu: Optional[float]) -> np.ndarray:
        if self.use_dynamic_shifting:
            if mu is None:
                raise ValueError("dynamic shifting requires mu")
            return math.exp(mu) / (math.exp(mu) + (1.0 / sigmas - 1.0))
        return self.shift * sigmas / (1 + (self.shift - 1) * sigmas)

    def set_timesteps(self, num_inference_steps: int, device=None, mu: Optional[float] = None,
                      image_seq_len: Optional[int] = None) -> None:
        if self.use_dynamic_shifting and mu is None and image_seq_len is not None:
            mu = calculate_shift(image_seq_len, self.base_image_seq_len, self.max_image_seq_len,
                                 self.base_shift, self.max_shift)
        ts = np.linspace(self.sigma_max * self.num_train_timesteps, self.sigma_min * self.num_train_timesteps,
                         num_inference_steps)
        sig = ts / self.num_train_timesteps
        sig = self._shift_sigmas(sig, mu).astype(np.float32)
        self.num_inference_steps = num_inference_steps
        sig_t = torch.from_numpy(sig)
        self.timesteps = (sig_t * self.num_train_timesteps).to(device=device)
        self.sigmas = torch.cat([sig_t, torch.zeros(1)]).to(device=device)
        self._step_index = None

    @property
    def step_index(self) -> Optional[int]:
        return self._step_index

    def index_for_timestep(self, timestep) -> int:
        t = float(timestep)
        diffs = (self.timesteps.float().cpu() - t).abs()
        return int(torch.argmin(diffs).item())

    def sigma_pair(self, step_idx: torch.Tensor | int) -> tuple[torch.Tensor, torch.Tensor]:
        """(sigma_t, sigma_{t+1}) for each step index (scalar or per-sample LongTensor)."""
        sig = self.sigmas
        if isinstance(step_idx, int):
            return sig[step_idx], sig[step_idx + 1]
        idx = step_idx.to(sig.device).long()
        return sig[idx], sig[idx + 1]

    # ------------------------------------------------------------------ stepping
    def step(self, model_output: torch.Tensor, timestep, sample: torch.Tensor, *, noise_level: float = 0.7,
             prev_sample: Optional[torch.Tensor] = None, sde_type: str = "sde", return_logprobs: bool = True,
             include_logprob_normalizer: bool = True, generator: Optional[torch.Generator] = None,
             seed: Optional[int] = None, noise: Optional[torch.Tensor] = None) -> SchedulerStepOutput:
        """Sequential-loop step at the internal step index (advanced by one per call)."""
        if isinstance(timestep, int) or (isinstance(timestep, torch.Tensor) and not timestep.is_floating_point()):
            raise ValueError("pass one of scheduler.timesteps (a float), not an integer index")
        if self._step_index is None:
            self._step_index = self.index_for_timestep(timestep)
        out = self.sample_previous_step(sample=sample.float(), model_output=model_output.float(),
                                        step_index=self._step_index, noise_level=noise_level,
                                        prev_sample=None if prev_sample is None else prev_sample.float(),
                                        sde_type=sde_type, return_logprobs=return_logprobs,
                                        include_logprob_normalizer=include_logprob_normalizer,
                                        generator=generator, seed=seed, noise=noise)
        self._step_index += 1
        return out

    def sample_previous_step(self, sample: torch.Tensor, model_output: torch.Tensor, *,
                             step_index: torch.Tensor | int | None = None, timestep: Optional[torch.Tensor] = None,
                             noise_level: float = 0.7, prev_sample: Optional[torch.Tensor] = None,
                             sde_type: str = "sde", return_logprobs: bool = True, return_sqrt_dt: bool = False,
                             include_logprob_normalizer: bool = True, generator: Optional[torch.Generator] = None,
                             seed: Optional[int] = None, noise: Optional[torch.Tensor] = None,
                             row_seeds: Optional[torch.Tensor] = None,
                             noise_offset: int = 0) -> SchedulerStepOutput:
        """One reverse step.  ``step_index`` (int or per-sample tensor) or ``timestep`` selects sigma.

        ``noise`` supplies the Gaussian draw explicitly; otherwise the CUDA kernel draws it from a
        counter-based Philox stream keyed by ``seed`` (one stream per sample row, offset by
        ``noise_offset``) or, with ``row_seeds``, by each sample's own seed; the CPU path draws the
        same stream when a seed is given and uses ``generator`` otherwise.
        """
        if sde_type not in ("sde", "cps", "dance_sde"):
            raise ValueError(sde_type)
        if sample.dtype != torch.float32 or model_output.dtype != torch.float32:
            raise TypeError("sample and model_output must be float32")
        if prev_sample is not None and prev_sample.dtype != torch.float32:
            raise TypeError("prev_sample must be float32")
        b = sample.shape[0]
        if step_index is None:
            if timestep is None:
                if self._step_index is None:
                    raise ValueError("no step index: pass step_index or timestep")
                step_index = self._step_index
            else:
                step_index = torch.tensor([self.index_for_timestep(t) for t in timestep.reshape(-1).tolist()])
        sig = self.sigmas.to(sample.device)
        if isinstance(step_index, int):
            sigma = sig[step_index].expand(b).contiguous()
            sigma_prev = sig[step_index + 1].expand(b).contiguous()
        else:
            idx = step_index.to(sample.device).long().reshape(-1)
            if idx.numel() == 1:
                idx = idx.expand(b)
            sigma, sigma_prev = sig[idx].contiguous(), sig[idx + 1].contiguous()
        sigma_max = float(self.sigmas[1])
        res = sde_ops.sde_step(sample, model_output, sigma.float(), sigma_prev.float(), sigma_max=sigma_max,
                               noise_level=float(noise_level), sde_type=sde_type, prev_sample=prev_sample,
                               noise=noise, generator=generator, seed=seed, noise_offset=noise_offset, row_seeds=row_seeds,
                               return_logprobs=return_logprobs,
                               include_logprob_normalizer=include_logprob_normalizer)
        prev, logp, mean, std = res
        sqrt_dt = torch.sqrt(sigma - sigma_prev) if return_sqrt_dt else None
        shape = (b,) + (1,) * (sample.ndim - 1)
        return SchedulerStepOutput(prev, logp, mean, std.reshape(shape), sqrt_dt)


def build_scheduler(kind: str = "sd3", num_inference_steps: int = 10, image_seq_len: Optional[int] = None,
                    device=None) -> FlowMatchSDEDiscreteScheduler:
    """Scheduler presets of the model families (SD3: shift 3; FLUX/Qwen-Image/LTX-2: dynamic; Wan: shift 5)."""
    if kind in ("sd3", "mmdit", "tiny"):
        sch = FlowMatchSDEDiscreteScheduler(shift=3.0)
    elif kind in ("flux", "qwen_image"):
        sch = FlowMatchSDEDiscreteScheduler(shift=1.0, use_dynamic_shifting=True, max_shift=1.15)
    elif kind == "wan":
        sch = FlowMatchSDEDiscreteScheduler(shift=5.0)
    elif kind == "ltx2":  # dynamic shift over the video token count (base 1024 -> 0.95, 4096 -> 2.05)
        sch = FlowMatchSDEDiscreteScheduler(shift=1.0, use_dynamic_shifting=True, base_image_seq_len=1024,
                                            max_image_seq_len=4096, base_shift=0.95, max_shift=2.05)
    else:
        raise ValueError(kind)
    sch.set_timesteps(num_inference_steps, device=device, image_seq_len=image_seq_len)
    return sch
