"""The device-side sampler step (nd_op_sampler_step) against the oracle's
restatement of the reference's CPU step: bit-identical, for every sampler,
prediction type, one or two guidance branches, first and second order and
the final step to sigma 0; then whole loops, and a loop through a denoiser."""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import ops
from naivediffusion_b200.sampling import PREDICTIONS, SAMPLERS, DeviceSamplingLoop, StepScalars, model_input_scale

pytestmark = pytest.mark.gpu

SIGMAS_VP = np.array([14.6, 8.1, 4.2, 2.05, 0.91, 0.36, 0.12, 0.029, 0.0], np.float32)
SIGMAS_FLOW = np.array([1.0, 0.93, 0.82, 0.66, 0.45, 0.24, 0.09, 0.02, 0.0], np.float32)


@pytest.mark.parametrize("prediction", sorted(PREDICTIONS))
@pytest.mark.parametrize("sampler", sorted(SAMPLERS))
@pytest.mark.parametrize("branches", [1, 2])
def test_step_is_bit_identical_to_the_oracle(cuda, sampler, prediction, branches):
    rng = np.random.default_rng(hash((sampler, prediction, branches)) % 2**32)
    n = 4 * 64 * 64 + 3
    sigmas = SIGMAS_FLOW if prediction == "flow" else SIGMAS_VP
    sch_h, sch_d = StepScalars(sampler, prediction, sigmas), StepScalars(sampler, prediction, sigmas)
    sample_h = rng.standard_normal(n).astype(np.float32) * sigmas[0]
    last_h = np.zeros(n, np.float32)
    sample_d = torch.from_numpy(sample_h.copy()).cuda()
    last_d = torch.zeros(n, device="cuda")
    den_d = torch.empty(n, device="cuda")
    nxt_d = torch.empty(n, device="cuda")
    for step in range(sch_h.steps):   # covers first / second order and the final step to 0
        out = rng.standard_normal((branches, n)).astype(np.float32)
        noise = rng.standard_normal(n).astype(np.float32) if sch_h.stochastic else None
        dh, dd = sch_h.at(step), sch_d.at(step)
        assert dh == dd
        sample_h, last_h, den_h = O.sampler_step(SAMPLERS[sampler], PREDICTIONS[prediction], out, sample_h,
                                                 guidance=3.5, last=last_h, noise=noise, want_denoised=True, **dh)
        scale = model_input_scale(prediction, dd["sigma_next"])
        ops.sampler_step(SAMPLERS[sampler], PREDICTIONS[prediction], torch.from_numpy(out).cuda(), sample_d,
                         guidance=3.5, last=last_d, noise=None if noise is None else torch.from_numpy(noise).cuda(),
                         denoised_out=den_d, next_input=nxt_d, next_input_scale=scale, **dd)
        torch.cuda.synchronize()
        assert np.array_equal(sample_d.cpu().numpy(), sample_h), (sampler, prediction, step)
        assert np.array_equal(den_d.cpu().numpy(), den_h), (sampler, prediction, step)
        assert np.array_equal(nxt_d.cpu().numpy(), sample_h * np.float32(scale))
        if sampler.startswith("dpmpp") and dh["sigma_next"] > 0:
            assert np.array_equal(last_d.cpu().numpy(), last_h)


def test_step_rejects_missing_inputs(cuda):
    s = torch.zeros(16, device="cuda")
    with pytest.raises(Exception, match="noise"):
        ops.sampler_step(SAMPLERS["euler_a"], 0, s, s, sigma=1.0, sigma_next=0.5)
    with pytest.raises(Exception, match="last_denoised"):
        ops.sampler_step(SAMPLERS["dpmpp_2m"], 0, s, s, sigma=1.0, sigma_next=0.5)


def test_sampling_loop_through_a_denoiser_matches_the_host_loop(cuda):
    """Three DPM++ 2M steps with CFG (batch-2 Anima: uncond, cond) on the
    device against the same steps taken on the host from the same predictions:
    the latents stay bit-identical step after step."""
    from naivediffusion_b200.denoiser import AnimaConfig, Device, build_denoiser, synthetic_weights
    cfg = AnimaConfig(width=256, heads=2, blocks=1, mlp_width=512, adaln_rank=64, context_rows=32,
                      context_width=128, latent_height=16, latent_width=16, batch=2)
    w = dict(synthetic_weights(cfg, seed=2))
    rng = np.random.default_rng(2)
    ctx = torch.from_numpy(rng.standard_normal((2, 32, 128)).astype(np.float32)).cuda()
    n = 16 * 16 * 16
    sigmas = np.array([1.0, 0.7, 0.4, 0.0], np.float32)
    latent0 = rng.standard_normal(n).astype(np.float32)
    with Device(0) as dev, build_denoiser(dev, cfg, w) as d:
        loop = DeviceSamplingLoop("dpmpp_2m", "flow", sigmas, n)
        sample = torch.from_numpy(latent0.copy()).cuda()
        model_in = sample.clone()
        out = torch.empty(2, 16, 16, 16, device="cuda")
        sch = StepScalars("dpmpp_2m", "flow", sigmas)
        host = latent0.copy()
        last = np.zeros(n, np.float32)
        for step in range(loop.steps):
            inp = model_in.view(1, 16, 16, 16).expand(2, 16, 16, 16).contiguous()
            d.predict_device(inp, 0.0, float(sigmas[step]), {"context": ctx}, out)
            torch.cuda.synchronize()
            preds = out.view(2, n).cpu().numpy()
            loop.step(step, out, sample, guidance=4.0, next_input=model_in)
            host, last = O.sampler_step(SAMPLERS["dpmpp_2m"], PREDICTIONS["flow"], preds, host, guidance=4.0,
                                        last=last, **sch.at(step))
            torch.cuda.synchronize()
            assert np.array_equal(sample.cpu().numpy(), host), step
