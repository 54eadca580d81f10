"""Device-side sampling loop: the host half of nd_op_sampler_step.

The reference steps its solvers on the CPU after copying each prediction
back (GenerationPipeline.SampleOne: Combine, then Scheduler.Step,
Pipeline/GenerationPipeline.cs:587-614). Here the latent stays in HBM: per
step the host computes the few double-precision scalars the reference
derives from the sigma schedule (logs and square roots, exactly as it writes
them) and the element work -- guidance combine, the solver update, the next
step's scaled model input -- runs in one kernel.

    loop = DeviceSamplingLoop("dpmpp_2m", "epsilon", sigmas, n)
    for step in range(loop.steps):
        denoiser.predict_device(model_input, ...)          # -> out [branches, n]
        loop.step(step, out, sample, guidance=5.0, next_input=model_input)

The sigma schedule itself (SigmaScheduler.SetTimesteps) is host code the
pipeline keeps; pass its float32 `Sigmas` array.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib, ops

SAMPLERS = {"euler": _lib.ND_SAMPLER_EULER, "euler_a": _lib.ND_SAMPLER_EULER_A,
            "dpmpp_2m": _lib.ND_SAMPLER_DPMPP_2M, "dpmpp_2m_sde": _lib.ND_SAMPLER_DPMPP_2M_SDE}
PREDICTIONS = {"epsilon": _lib.ND_PRED_EPSILON, "velocity": _lib.ND_PRED_VELOCITY, "flow": _lib.ND_PRED_FLOW}


def renoise(prediction: str, sigma_down: float, sigma_next: float) -> tuple[float, float]:
    """Prediction.Renoise (Sampling/Prediction.cs): the rescale and noise scale
    that bring a sample integrated down to sigma_down back up to sigma_next."""
    if prediction == "flow":
        rescale = (1.0 - sigma_next) / (1.0 - sigma_down)
        return rescale, math.sqrt(max(sigma_next * sigma_next - sigma_down * sigma_down * rescale * rescale, 0.0))
    return 1.0, math.sqrt(max(sigma_next * sigma_next - sigma_down * sigma_down, 0.0))


def model_input_scale(prediction: str, sigma: float) -> float:
    """Prediction.ModelInputScale: 1 / sqrt(sigma^2 + 1) as float (epsilon,
    velocity), 1 for flow."""
    if prediction == "flow":
        return 1.0
    return float(np.float32(1.0) / np.float32(math.sqrt(sigma * sigma + 1.0)))


class StepScalars:
    """Per-step scalars of one sampler over a float32 sigma schedule
    (Sigmas[0 .. steps], the last one 0), with the DPM++ history
    (SigmaScheduler.SecondOrderAt: second order except on the last two steps)."""

    def __init__(self, sampler: str, prediction: str, sigmas):
        if sampler not in SAMPLERS or prediction not in PREDICTIONS:
            raise ValueError("unknown sampler or prediction")
        self.sampler, self.prediction = sampler, prediction
        self.sigmas = np.asarray(sigmas, dtype=np.float32)
        self.steps = len(self.sigmas) - 1
        self._last_step_size = None

    def reset(self) -> None:
        self._last_step_size = None

    def at(self, step: int) -> dict:
        sigma = float(self.sigmas[step])
        sigma_next = float(self.sigmas[step + 1])
        d = dict(sigma=sigma, sigma_next=sigma_next, up=0.0, down=0.0, rescale=1.0, noise_scale=0.0,
                 shrink=0.0, weight=0.0, second_order=False)
        if self.sampler == "euler_a":
            up = sigma_next * math.sqrt(max(sigma * sigma - sigma_next * sigma_next, 0.0)) / sigma
            down = math.sqrt(max(sigma_next * sigma_next - up * up, 0.0))
            d["up"], d["down"] = up, down
            d["rescale"], d["noise_scale"] = renoise(self.prediction, down, sigma_next)
        elif self.sampler in ("dpmpp_2m", "dpmpp_2m_sde") and sigma_next > 0.0:
            step_size = math.log(sigma / sigma_next)
            shrink = sigma_next / sigma
            second = step + 2 < self.steps and self._last_step_size is not None
            d["shrink"] = shrink
            if self.sampler == "dpmpp_2m":
                d["weight"] = step_size / (2.0 * self._last_step_size) if second else 0.0
            else:
                take = 1.0 - shrink * shrink
                d["weight"] = 0.5 * take * step_size / self._last_step_size if second else 0.0
                d["rescale"], d["noise_scale"] = renoise(self.prediction, sigma_next * shrink, sigma_next)
            d["second_order"] = second
            self._last_step_size = step_size
        return d

    @property
    def stochastic(self) -> bool:
        return self.sampler in ("euler_a", "dpmpp_2m_sde")


class DeviceSamplingLoop:
    """Steps a device latent through a schedule with nd_op_sampler_step."""

    def __init__(self, sampler: str, prediction: str, sigmas, n: int, device="cuda"):
        self.scalars = StepScalars(sampler, prediction, sigmas)
        self.n = n
        self.last = torch.zeros(n, device=device, dtype=torch.float32)

    @property
    def steps(self) -> int:
        return self.scalars.steps

    def step(self, step: int, out: torch.Tensor, sample: torch.Tensor, *, guidance: float = 1.0,
             noise: torch.Tensor | None = None, next_input: torch.Tensor | None = None,
             denoised_out: torch.Tensor | None = None) -> None:
        d = self.scalars.at(step)
        scale = (model_input_scale(self.scalars.prediction, d["sigma_next"])
                 if next_input is not None and step + 1 < self.steps else 1.0)
        ops.sampler_step(SAMPLERS[self.scalars.sampler], PREDICTIONS[self.scalars.prediction], out, sample,
                         guidance=guidance, last=self.last, noise=noise, denoised_out=denoised_out,
                         next_input=next_input, next_input_scale=scale, **d)
