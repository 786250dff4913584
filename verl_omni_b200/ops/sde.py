"""Fused reverse-SDE step + log-prob (sde / cps / dance_sde).

Math follows ``verl_omni/pipelines/schedulers/flow_match_sde.py:214-313``.  On CUDA the whole
step (mean, Philox4x32-10 Gaussian draw, sample, squared-error log-prob and its per-sample
mean) is one kernel pass that reads ``sample`` and ``model_output`` once; on CPU the
fp32 torch code below runs and serves as the oracle.

Noise: with ``seed`` given, element ``i`` of row ``b`` at step offset ``o`` uses the Philox
counter ``(i // 4, b, o, 0)`` under key ``seed`` and Box-Muller, on both devices, so a rollout is
reproducible from ``(seed, step)`` alone.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from verl_omni_b200.ops._ext import ext

SDE_TYPES = {"sde": 0, "cps": 1, "dance_sde": 2}
_LOG_SQRT_2PI = 0.5 * math.log(2 * math.pi)

_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32(counter: list[torch.Tensor], key: tuple[int, int], rounds: int = 10) -> list[torch.Tensor]:
    """Philox4x32 (Salmon et al., SC'11) on int64 tensors holding uint32 values."""
    c0, c1, c2, c3 = [c & _MASK for c in counter]
    k0, k1 = key[0] & _MASK, key[1] & _MASK
    for r in range(rounds):
        if r:
            k0 = (k0 + _W0) & _MASK
            k1 = (k1 + _W1) & _MASK
        p0 = c0 * _M0
        p1 = c2 * _M1
        hi0, lo0 = (p0 >> 32) & _MASK, p0 & _MASK
        hi1, lo1 = (p1 >> 32) & _MASK, p1 & _MASK
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & _MASK, lo1, (hi0 ^ c3 ^ k1) & _MASK, lo0
    return [c0, c1, c2, c3]


def philox_normal(seed: int, rows: int, n: int, offset: int = 0,
                  row_seeds: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[rows, n] standard normals, bit-for-bit the stream the CUDA kernels draw (up to libm ulps).

    Without ``row_seeds`` one key (``seed``) serves the call and the row index enters the counter;
    with ``row_seeds`` (int64 [rows]) row ``b`` is keyed by its own seed and its counter omits the row,
    so a sample's noise does not depend on where it sits in a batch.
    """
    n4 = (n + 3) // 4
    i4 = torch.arange(n4, dtype=torch.int64).unsqueeze(0).expand(rows, n4)
    off = torch.full_like(i4, offset & _MASK)
    zero = torch.zeros_like(i4)
    if row_seeds is None:
        b = torch.arange(rows, dtype=torch.int64).unsqueeze(1).expand(rows, n4)
        key = (seed & _MASK, (seed >> 32) & _MASK)
    else:
        rs = row_seeds.detach().cpu().to(torch.int64).reshape(rows, 1)
        b = zero
        key = ((rs & _MASK).expand(rows, n4), ((rs >> 32) & _MASK).expand(rows, n4))
    x0, x1, x2, x3 = philox4x32([i4, b, off, zero], key)
    inv = 2.0 ** -32

    def bm(a, c):
        u1 = (a.double() + 1.0) * inv
        u2 = c.double() * inv
        r = torch.sqrt(-2.0 * torch.log(u1.float()))
        ang = (2.0 * math.pi) * u2.float()
        return r * torch.cos(ang), r * torch.sin(ang)

    z0, z1 = bm(x0, x1)
    z2, z3 = bm(x2, x3)
    out = torch.stack([z0, z1, z2, z3], dim=-1).reshape(rows, n4 * 4)
    return out[:, :n].contiguous()


def normal_rows(row_seeds: torch.Tensor, shape: tuple, offset: int, device) -> torch.Tensor:
    """[B, *shape] standard normals, row b keyed by ``row_seeds[b]`` (same stream on CPU and GPU)."""
    B, n = int(row_seeds.numel()), int(math.prod(shape))
    if torch.device(device).type == "cuda":
        z = ext().normal_fill(row_seeds.to(device=device, dtype=torch.int64).contiguous(), n, int(offset))
    else:
        z = philox_normal(0, B, n, offset, row_seeds=row_seeds)
    return z.reshape((B,) + tuple(shape))


def _bcast(v: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    return v.reshape(v.shape[0], *([1] * (ref.ndim - 1)))


def sde_step_reference(sample, model_output, sigma, sigma_prev, *, sigma_max, noise_level, sde_type,
                       prev_sample=None, noise=None, return_logprobs=True, include_logprob_normalizer=True):
    """fp32 torch restatement of the three reverse-step variants (the oracle)."""
    sigma = _bcast(sigma.to(sample.dtype), sample)
    sigma_prev = _bcast(sigma_prev.to(sample.dtype), sample)
    dt = sigma_prev - sigma
    if sde_type == "sde":
        denom = 1 - torch.where(sigma == 1, torch.full_like(sigma, sigma_max), sigma)
        std = torch.sqrt(sigma / denom) * noise_level
        mean = sample * (1 + std ** 2 / (2 * sigma) * dt) + model_output * (1 + std ** 2 * (1 - sigma) / (2 * sigma)) * dt
        scale = std * torch.sqrt(-1 * dt)
    elif sde_type == "cps":
        std = sigma_prev * math.sin(noise_level * math.pi / 2)
        x0 = sample - sigma * model_output
        xn = sample + model_output * (1 - sigma)
        mean = x0 * (1 - sigma_prev) + xn * torch.sqrt(sigma_prev ** 2 - std ** 2)
        scale = std
    else:
        delta_t = sigma - sigma_prev
        mean = sample + dt * model_output
        x0 = sample - sigma * model_output
        score = -(sample - x0 * (1 - sigma)) / (sigma ** 2)
        mean = mean + (-0.5 * noise_level ** 2 * score) * dt
        std = noise_level * torch.sqrt(delta_t)
        scale = std
    if prev_sample is None:
        prev_sample = mean + scale * noise
    logp = None
    if return_logprobs:
        if sde_type == "cps":
            lp = -((prev_sample.detach() - mean) ** 2)
        else:
            lp = -((prev_sample.detach() - mean) ** 2) / (2 * scale ** 2)
            if include_logprob_normalizer:
                lp = lp - torch.log(scale) - _LOG_SQRT_2PI
        logp = lp.mean(dim=tuple(range(1, lp.ndim)))
    return prev_sample, logp, mean, std.reshape(-1)


def sde_step(sample: torch.Tensor, model_output: torch.Tensor, sigma: torch.Tensor, sigma_prev: torch.Tensor, *,
             sigma_max: float, noise_level: float, sde_type: str = "sde", prev_sample: Optional[torch.Tensor] = None,
             noise: Optional[torch.Tensor] = None, generator: Optional[torch.Generator] = None,
             seed: Optional[int] = None, noise_offset: int = 0, return_logprobs: bool = True,
             include_logprob_normalizer: bool = True, row_seeds: Optional[torch.Tensor] = None):
    """Returns ``(prev_sample, log_prob[B] or None, prev_sample_mean, std_dev_t[B])``.

    In-kernel noise is keyed by ``seed`` (whole call) or by ``row_seeds`` (int64 [B], one per sample).

    Differentiable w.r.t. ``model_output`` (the training path backpropagates the log-prob and
    the mean through it); ``sample``/``prev_sample`` are trajectory data and get no gradient.
    """
    b = sample.shape[0]
    need_noise = prev_sample is None and noise is None and seed is None and row_seeds is None
    if need_noise:
        noise = torch.randn(sample.shape, generator=generator, device=sample.device, dtype=torch.float32)
    if not sample.is_cuda:
        if prev_sample is None and noise is None:
            noise = philox_normal(int(seed or 0), b, sample[0].numel(), noise_offset,
                                  row_seeds=row_seeds).reshape(sample.shape)
        return sde_step_reference(sample, model_output, sigma, sigma_prev, sigma_max=sigma_max,
                                  noise_level=noise_level, sde_type=sde_type, prev_sample=prev_sample, noise=noise,
                                  return_logprobs=return_logprobs,
                                  include_logprob_normalizer=include_logprob_normalizer)
    rs = row_seeds.to(device=sample.device, dtype=torch.int64).contiguous() if row_seeds is not None else None
    return _SDEStepFn.apply(sample, model_output, sigma, sigma_prev, prev_sample, noise, float(sigma_max),
                            float(noise_level), SDE_TYPES[sde_type], int(seed or 0), int(noise_offset),
                            bool(return_logprobs), bool(include_logprob_normalizer), rs)


class _SDEStepFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, sample, model_output, sigma, sigma_prev, prev_sample, noise, sigma_max, noise_level, sde_type,
                seed, noise_offset, return_logprobs, include_norm, row_seeds):
        s = sample.contiguous()
        m = model_output.contiguous()
        prev, logp, mean, std = ext().sde_step_fwd(
            s, m, sigma.contiguous().float(), sigma_prev.contiguous().float(),
            prev_sample.contiguous() if prev_sample is not None else None,
            noise.contiguous() if noise is not None else None,
            sigma_max, noise_level, sde_type, seed, noise_offset, return_logprobs, include_norm, row_seeds)
        ctx.save_for_backward(s, prev, mean, sigma, sigma_prev)
        ctx.cfg = (sigma_max, noise_level, sde_type, include_norm)
        return prev, (logp if return_logprobs else None), mean, std

    @staticmethod
    def backward(ctx, g_prev, g_logp, g_mean, g_std):
        s, prev, mean, sigma, sigma_prev = ctx.saved_tensors
        sigma_max, noise_level, sde_type, include_norm = ctx.cfg
        if g_logp is None:
            g_logp = torch.zeros(s.shape[0], device=s.device, dtype=torch.float32)
        if g_mean is None:
            g_mean = torch.zeros_like(s)
        grad_mo = ext().sde_step_bwd(s, prev, mean, sigma.float(), sigma_prev.float(), g_logp.float().contiguous(),
                                     g_mean.float().contiguous(), sigma_max, noise_level, sde_type)
        return (None, grad_mo, None, None, None, None, None, None, None, None, None, None, None, None)
