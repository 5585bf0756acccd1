"""Denoising-loop samplers: host schedules (CPU) against the reference's formulas, and the
fused CFG + DDIM / DPM++ 2M device updates against the oracle's f32 restatement
(crates/sketchpad-samplers/src/ddim.rs:72-164, dpm.rs:101-171): bit-exact for f32 latents
given the same step scalars, rel_err < 2e-2 for bf16."""
import numpy as np
import pytest
import torch

import oracle
from helpers import TOL_HALF, rel_err, to_np
from sketchpad_b200.samplers import (DdimSampler, DpmPlusPlusSampler, NoiseSchedule,
                                     sampler_timesteps)


def test_sd1x_schedule_known_values():
    s = NoiseSchedule.sd1x()
    f = np.float32
    b0 = f(0.00085)
    assert s.alphas_cumprod[0] == f(1.0) - b0                 # scheduler.rs:145-167
    b1 = f(0.00085 + (1 / 999) * (0.012 - 0.00085))
    assert s.alphas_cumprod[1] == f((f(1.0) - b0) * (f(1.0) - b1))
    assert np.all(np.diff(s.alphas_cumprod) < 0)
    x = NoiseSchedule.sdxl()
    sb = (0.00085 ** 0.5)
    assert x.alphas_cumprod[0] == f(1.0) - f(sb * sb)         # scheduler.rs:175-207


def test_timesteps_and_sigmas():
    assert DdimSampler(NoiseSchedule.sd1x(), 50).timesteps()[:3] == [980, 960, 940]
    assert sampler_timesteps(20, 1000)[:2] == [950, 900] and sampler_timesteps(20, 1000)[-1] == 0
    p = DpmPlusPlusSampler(NoiseSchedule.sd1x(), 20)
    a = NoiseSchedule.sd1x().alphas_cumprod[950]
    assert p.sigmas()[0] == np.float32(np.sqrt(np.float32(np.float32(1) - a) / a))
    assert p.sigmas()[-1] == 0.0 and len(p.sigmas()) == 21


def _latents(dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, 4, 64, 64, generator=g)
    eu, ec = torch.randn(2, 4, 64, 64, generator=g), torch.randn(2, 4, 64, 64, generator=g)
    return x.to(dtype), eu.to(dtype), ec.to(dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [True, False])
def test_ddim_steps_bit_exact_f32(cfg):
    smp = DdimSampler(NoiseSchedule.sd1x(), 10)
    x, eu, ec = _latents(torch.float32)
    xd, eud, ecd = x.cuda(), eu.cuda(), ec.cuda()
    ref = to_np(x)
    for i in range(smp.num_steps()):
        xd = smp.step(xd, eud, i, ecd if cfg else None, 7.5)
        somat, sat, sap, dxt, _ = smp.step_scalars(i)
        ref = oracle.ddim_step(ref, to_np(eu), to_np(ec) if cfg else None, 7.5, somat, sat, sap, dxt)
    assert np.array_equal(to_np(xd).view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
def test_ddim_eta_noise_and_in_place():
    smp = DdimSampler(NoiseSchedule.sd1x(), 10, eta=0.5)
    x, eu, ec = _latents(torch.float32, 1)
    noise = torch.randn(x.shape, generator=torch.Generator().manual_seed(9))
    xd = x.cuda()
    y = smp.step(xd, eu.cuda(), 3, ec.cuda(), 5.0, out=xd, noise=noise.cuda())
    assert y.data_ptr() == xd.data_ptr()
    somat, sat, sap, dxt, sigma = smp.step_scalars(3)
    assert sigma > 0
    ref = oracle.ddim_step(to_np(x), to_np(eu), to_np(ec), 5.0, somat, sat, sap, dxt, to_np(noise), sigma)
    assert np.array_equal(to_np(y).view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_dpmpp_2m_steps_vs_oracle(dtype):
    smp = DpmPlusPlusSampler(NoiseSchedule.sd1x(), 8)
    x, eu, ec = _latents(dtype, 2)
    xd, eud, ecd = x.cuda(), eu.cuda(), ec.cuda()
    ref, prev = to_np(x), None
    for i in range(smp.num_steps()):
        second = prev is not None and smp.sigmas()[i + 1] != 0.0
        sig, ratio, c1, c2, coeff = smp.step_scalars(i, second)
        xd = smp.step(xd, eud, i, ecd, 6.0)
        ref, den = oracle.dpmpp_2m_step(ref, to_np(eu), to_np(ec), 6.0, sig, ratio, c1,
                                        prev if second else None, c2, coeff)
        if dtype == torch.bfloat16:
            ref = to_np(torch.from_numpy(ref).to(torch.bfloat16))  # the latent is stored bf16
        prev = den
    if dtype == torch.float32:
        assert np.array_equal(to_np(xd).view(np.uint32), ref.view(np.uint32))
    else:
        assert rel_err(to_np(xd), ref) < TOL_HALF


@pytest.mark.gpu
def test_sampler_rejects_mismatched_tensors():
    smp = DdimSampler(NoiseSchedule.sd1x(), 10)
    x = torch.zeros(2, 4, 8, 8, device="cuda")
    with pytest.raises(ValueError):
        smp.step(x, torch.zeros(2, 4, 8, 9, device="cuda"), 0)
    with pytest.raises(ValueError):
        DdimSampler(NoiseSchedule.sd1x(), 10, eta=1.0).step(x, x, 0)
