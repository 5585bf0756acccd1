"""Denoising-loop samplers with the latent update on the device: DDIM and DPM++ 2M, each
fused with classifier-free guidance into one kernel per step, and the host noise schedules
that give their scalars.

Host mirror of crates/sketchpad-samplers/src:
  scheduler.rs:143-207  NoiseSchedule::linear / scaled_linear (alphas_cumprod in f32)
  scheduler.rs:234-257  NoiseSchedule::sd1x / sdxl
  scheduler.rs:344-357  sigmas_from_timesteps; :507-527 compute_sigmas (Normal schedule)
  scheduler.rs:603-609  sampler_timesteps
  ddim.rs:40-133        DdimSampler::{new, timesteps, step};  ddim.rs:158-164 apply_guidance
  dpm.rs:63-171         DpmPlusPlusSampler::{new, sigmas, reset, step}
Host scalars are computed in the reference's precision and order: f64 where it uses f64
(the beta ramps), f32 elsewhere.  Square roots and divisions are IEEE f32; ln and exp are
the correctly rounded f32 of the f64 result (Rust's f32::ln / f32::exp call the platform
libm, which can differ from that in the last place).
"""
from __future__ import annotations

import math
from typing import List, Optional

import numpy as np
import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr

_f32 = np.float32


class NoiseSchedule:
    """scheduler.rs:136-257: alphas_cumprod [num_train_steps] (f32)."""

    def __init__(self, alphas_cumprod: np.ndarray):
        self.alphas_cumprod = np.asarray(alphas_cumprod, np.float32)
        self.num_train_steps = len(self.alphas_cumprod)

    @staticmethod
    def _from_betas(betas: List[np.float32]) -> "NoiseSchedule":
        out, cumprod = [], _f32(1.0)
        for b in betas:
            cumprod = _f32(cumprod * (_f32(1.0) - b))
            out.append(cumprod)
        return NoiseSchedule(np.array(out, np.float32))

    @classmethod
    def linear(cls, num_steps: int, beta_start: float, beta_end: float) -> "NoiseSchedule":
        """scheduler.rs:145-167: betas = beta_start + t (beta_end - beta_start), t = i/(n-1), in f64."""
        return cls._from_betas([_f32(beta_start + (i / (num_steps - 1)) * (beta_end - beta_start))
                                for i in range(num_steps)])

    @classmethod
    def scaled_linear(cls, num_steps: int, beta_start: float, beta_end: float) -> "NoiseSchedule":
        """scheduler.rs:175-207: sqrt(beta) interpolated in f64, squared, cast to f32."""
        s0, s1 = math.sqrt(beta_start), math.sqrt(beta_end)
        betas = []
        for i in range(num_steps):
            sb = s0 + (i / (num_steps - 1)) * (s1 - s0)
            betas.append(_f32(sb * sb))
        return cls._from_betas(betas)

    @classmethod
    def sd1x(cls) -> "NoiseSchedule":
        return cls.linear(1000, 0.00085, 0.012)

    @classmethod
    def sdxl(cls) -> "NoiseSchedule":
        return cls.scaled_linear(1000, 0.00085, 0.012)

    def alpha_cumprod_at(self, t: int) -> np.float32:
        return self.alphas_cumprod[t]


def sampler_timesteps(num_inference_steps: int, num_train_steps: int) -> List[int]:
    """scheduler.rs:603-609."""
    ratio = num_train_steps // num_inference_steps
    return [min(i * ratio, num_train_steps - 1) for i in reversed(range(num_inference_steps))]


def sigmas_from_timesteps(schedule: NoiseSchedule, timesteps: List[int]) -> List[np.float32]:
    """scheduler.rs:344-357: sqrt((1 - alpha) / alpha) in f32."""
    out = []
    for t in timesteps:
        a = schedule.alpha_cumprod_at(t)
        out.append(_f32(np.sqrt(_f32(_f32(1.0) - a) / a)))
    return out


def _ln(x) -> np.float32:
    return _f32(math.log(float(x)))


def _exp(x) -> np.float32:
    return _f32(math.exp(float(x)))


def _check_pair(latent, eps_uncond, eps_cond, out):
    dev = require_cuda(latent, eps_uncond, eps_cond, out)
    for t in (eps_uncond, eps_cond, out):
        if t is not None and (t.shape != latent.shape or t.dtype != latent.dtype or
                              not t.is_contiguous()):
            raise ValueError("eps / out must be contiguous tensors of the latent's shape and dtype")
    if not latent.is_contiguous():
        raise ValueError("latent must be contiguous")
    return dev


class DdimSampler:
    """ddim.rs:40-133 (deterministic for eta = 0)."""

    def __init__(self, schedule: NoiseSchedule, num_inference_steps: int = 50, eta: float = 0.0):
        self.schedule, self.eta = schedule, float(eta)
        ratio = schedule.num_train_steps // num_inference_steps
        self._timesteps = [i * ratio for i in reversed(range(num_inference_steps))]

    def timesteps(self) -> List[int]:
        return self._timesteps

    def num_steps(self) -> int:
        return len(self._timesteps)

    def step_scalars(self, step_index: int):
        """(sqrt(1 - a_t), sqrt(a_t), sqrt(a_prev), dir_xt, sigma) as ddim.rs:79-121 forms them."""
        sch = self.schedule
        a_t = sch.alpha_cumprod_at(self._timesteps[step_index])
        a_prev = (sch.alpha_cumprod_at(self._timesteps[step_index + 1])
                  if step_index + 1 < len(self._timesteps) else _f32(1.0))
        one = _f32(1.0)
        sqrt_at = _f32(np.sqrt(a_t))
        somat = _f32(np.sqrt(_f32(-a_t + one)))
        somp = _f32(np.sqrt(_f32(-a_prev + one)))
        if self.eta > 0.0:
            variance = _f32(_f32(_f32(-a_prev + one) / _f32(-a_t + one)) * _f32(-a_t + a_prev))
            sigma = _f32(_f32(np.sqrt(variance)) * _f32(self.eta))
        else:
            sigma = _f32(0.0)
        dir_xt = _f32(np.sqrt(max(_f32(_f32(somp * somp) - _f32(sigma * sigma)), _f32(0.0))))
        return somat, sqrt_at, _f32(np.sqrt(a_prev)), dir_xt, sigma

    def step(self, latent: torch.Tensor, eps_uncond: torch.Tensor, step_index: int,
             eps_cond: Optional[torch.Tensor] = None, guidance: float = 1.0,
             out: Optional[torch.Tensor] = None, noise: Optional[torch.Tensor] = None):
        """The next latent from the UNet's noise predictions (uncond, and cond for CFG)."""
        dev = _check_pair(latent, eps_uncond, eps_cond, out)
        if self.eta > 0.0 and noise is None:
            raise ValueError("eta > 0 needs the step's N(0,1) noise tensor")
        somat, sqrt_at, sqrt_ap, dir_xt, sigma = self.step_scalars(step_index)
        y = out if out is not None else torch.empty_like(latent)
        _lib.call("sp_cfg_ddim_step", ptr(latent), ptr(eps_uncond), ptr(eps_cond),
                  ptr(noise if self.eta > 0.0 else None), ptr(y), latent.numel(),
                  float(_f32(guidance)), float(somat), float(sqrt_at), float(sqrt_ap),
                  float(dir_xt), float(sigma), dtype_code(latent.dtype), stream_ptr(dev))
        return y


class DpmPlusPlusSampler:
    """dpm.rs:63-171: DPM++ 2M (k-diffusion form) with the Normal sigma schedule."""

    def __init__(self, schedule: NoiseSchedule, num_inference_steps: int = 20):
        self._timesteps = sampler_timesteps(num_inference_steps, schedule.num_train_steps)
        self._sigmas = sigmas_from_timesteps(schedule, self._timesteps) + [_f32(0.0)]
        self._prev: Optional[torch.Tensor] = None
        self._prev_sigma: Optional[np.float32] = None

    def timesteps(self) -> List[int]:
        return self._timesteps

    def sigmas(self) -> List[np.float32]:
        return self._sigmas

    def num_steps(self) -> int:
        return len(self._timesteps)

    def reset(self):
        self._prev, self._prev_sigma = None, None

    def step_scalars(self, step_index: int, second_order: bool):
        """(sigma, sigma_next / sigma, 1 - exp(-h), 1 + c, c) as dpm.rs:107-165 forms them."""
        sigma, sigma_next = self._sigmas[step_index], self._sigmas[step_index + 1]
        t = _f32(-_ln(sigma))
        t_next = _f32(-_ln(sigma_next)) if sigma_next > 0.0 else _f32(np.inf)
        h = _f32(t_next - t)
        ratio = _f32(sigma_next / sigma)
        c1 = _f32(_f32(1.0) - _exp(_f32(-h)))
        if not second_order:
            return sigma, ratio, c1, _f32(1.0), _f32(0.0)
        t_prev = _f32(-_ln(self._prev_sigma))
        r = _f32(_f32(t - t_prev) / h)
        coeff = _f32(_f32(1.0) / _f32(_f32(2.0) * r))
        return sigma, ratio, c1, _f32(_f32(1.0) + coeff), coeff

    def step(self, latent: torch.Tensor, eps_uncond: torch.Tensor, step_index: int,
             eps_cond: Optional[torch.Tensor] = None, guidance: float = 1.0,
             out: Optional[torch.Tensor] = None):
        dev = _check_pair(latent, eps_uncond, eps_cond, out)
        second = self._prev is not None and self._sigmas[step_index + 1] != 0.0
        sigma, ratio, c1, c2, coeff = self.step_scalars(step_index, second)
        if self._prev is None or self._prev.numel() != latent.numel():
            self._prev = torch.empty(latent.shape, dtype=torch.float32, device=dev)
        y = out if out is not None else torch.empty_like(latent)
        _lib.call("sp_cfg_dpmpp_2m_step", ptr(latent), ptr(eps_uncond), ptr(eps_cond),
                  ptr(self._prev), ptr(y), latent.numel(), float(_f32(guidance)), float(sigma),
                  float(ratio), float(c1), float(c2), float(coeff), 1 if second else 0,
                  dtype_code(latent.dtype), stream_ptr(dev))
        self._prev_sigma = sigma
        return y


__all__ = ["NoiseSchedule", "DdimSampler", "DpmPlusPlusSampler", "sampler_timesteps",
           "sigmas_from_timesteps"]
