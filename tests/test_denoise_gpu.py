"""The device denoising loop (captured CFG-pair UNet step + fused CFG/sampler update) against
a step-by-step reference loop: the same UNet run eagerly, the latent update by the oracle's
f32 restatement of DdimSampler::step / DpmPlusPlusSampler::step with the pipeline's order
(crates/sketchpad/src/pipeline/sd1x.rs:285-360, :393-490).  rel_err < 2e-2 (bf16 UNet)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import TOL_HALF, rel_err, to_np
from sketchpad_b200.denoise import Sd1xDenoiseLoop
from sketchpad_b200.samplers import DdimSampler, DpmPlusPlusSampler, NoiseSchedule
from sketchpad_b200.unet import UNetB200, make_unet_params

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def net():
    return UNetB200(make_unet_params(seed=0))


def _inputs():
    rng = np.random.default_rng(3)
    lat = rng.standard_normal((1, 4, 64, 64), dtype=np.float32)
    cu = rng.standard_normal((1, 77, 768), dtype=np.float32)
    cc = rng.standard_normal((1, 77, 768), dtype=np.float32)
    return lat, cu, cc


def _eager_eps(net, x, t, cu, cc):
    x2 = torch.from_numpy(np.concatenate([x, x])).cuda()
    ctx = torch.from_numpy(np.concatenate([cu, cc])).cuda()
    with torch.inference_mode():
        eps = net(x2, torch.full((2,), float(t), device="cuda"), ctx).float()
    e = to_np(eps)
    return e[0:1], e[1:2]


@pytest.mark.parametrize("kind", ["ddim", "dpmpp_2m"])
def test_denoise_loop_matches_stepwise_reference(net, kind):
    lat, cu, cc = _inputs()
    sch = NoiseSchedule.sd1x()
    smp = DdimSampler(sch, 3) if kind == "ddim" else DpmPlusPlusSampler(sch, 3)
    loop = Sd1xDenoiseLoop(net, smp, guidance=7.5)
    out = to_np(loop(torch.from_numpy(lat).cuda(), torch.from_numpy(cu).cuda(),
                     torch.from_numpy(cc).cuda()))
    # reference loop
    ref = DdimSampler(sch, 3) if kind == "ddim" else DpmPlusPlusSampler(sch, 3)
    x, prev = lat.copy(), None
    for i, t in enumerate(ref.timesteps()):
        if kind == "ddim":
            eu, ec = _eager_eps(net, x, t, cu, cc)
            x = oracle.ddim_step(x, eu, ec, 7.5, *ref.step_scalars(i)[:4])
        else:
            s = ref.sigmas()[i]
            c_in = np.float32(1.0) / np.float32(np.sqrt(np.float32(1.0) + np.float32(s * s)))
            eu, ec = _eager_eps(net, (x * c_in).astype(np.float32), t, cu, cc)
            second = prev is not None and ref.sigmas()[i + 1] != 0.0
            sig, ratio, c1, c2, coeff = ref.step_scalars(i, second)
            x, prev = oracle.dpmpp_2m_step(x, eu, ec, 7.5, sig, ratio, c1,
                                           prev if second else None, c2, coeff)
            ref._prev_sigma = sig  # the host state the next step's scalars read
    err = rel_err(out, x)
    print(f"{kind} loop rel_err={err:.3e}")
    assert np.isfinite(out).all() and err < TOL_HALF
