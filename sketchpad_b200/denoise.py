"""The SD1.x denoising loop on the device: per step one classifier-free-guidance pair of UNet
evaluations (the captured UNet step, batch 2 = uncond + cond) and one fused CFG + sampler
update kernel.

Mirrors the loops of crates/sketchpad/src/pipeline/sd1x.rs: DDIM :285-360 (the UNet sees the
latent as is) and DPM++ 2M :393-490 (the UNet sees latent * c_in, c_in = 1 / sqrt(1 +
sigma^2), and the sampler updates the unscaled latent).  The reference evaluates the UNet
once per conditioning; the pair shares one batch-2 evaluation here, which gives the same
per-sample results.  The latent stays f32 between steps, as in the reference.
"""
from __future__ import annotations

import numpy as np
import torch

from .samplers import DdimSampler, DpmPlusPlusSampler
from .unet import UNetB200, UNetStepGraph


class Sd1xDenoiseLoop:
    def __init__(self, net: UNetB200, sampler, guidance: float = 7.5, hw: int = 64,
                 ctx_len: int = 77):
        if not isinstance(sampler, (DdimSampler, DpmPlusPlusSampler)):
            raise TypeError("sampler must be a DdimSampler or DpmPlusPlusSampler")
        self.sampler, self.guidance = sampler, float(guidance)
        self.graph = UNetStepGraph(net, batch=2, hw=hw, ctx_len=ctx_len, out_dtype=torch.float32)

    def __call__(self, latent: torch.Tensor, ctx_uncond: torch.Tensor,
                 ctx_cond: torch.Tensor) -> torch.Tensor:
        """latent [1, 4, h, w] (initial noise), contexts [1, 77, 768] -> the final latent (f32)."""
        g, smp = self.graph, self.sampler
        g.ctx[0:1].copy_(ctx_uncond)
        g.ctx[1:2].copy_(ctx_cond)
        lat = latent.to(device=g.x.device, dtype=torch.float32).contiguous().clone()
        dpm = isinstance(smp, DpmPlusPlusSampler)
        if dpm:
            smp.reset()
            sigmas = smp.sigmas()
        for i, t in enumerate(smp.timesteps()):
            if dpm:
                s = sigmas[i]
                c_in = float(np.float32(1.0) / np.float32(np.sqrt(np.float32(1.0) + np.float32(s * s))))
                torch.mul(lat, c_in, out=g.x[0:1])
                torch.mul(lat, c_in, out=g.x[1:2])
            else:
                g.x[0:1].copy_(lat)
                g.x[1:2].copy_(lat)
            g.t.fill_(float(t))
            eps = g.replay()
            smp.step(lat, eps[0:1], i, eps[1:2], self.guidance, out=lat)
        return lat


__all__ = ["Sd1xDenoiseLoop"]
