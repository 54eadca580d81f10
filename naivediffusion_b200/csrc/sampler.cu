// The sampler step on the device, fused with classifier-free guidance: one
// pass over the latent per denoising step instead of copying predictions to
// the host. Every operation is written as the reference writes it, with the
// same float / double types and no contraction into fused multiply-adds
// (explicit _rn intrinsics), so the result is bit-identical to the
// reference's CPU step:
//   ClassifierFreeGuidance.Combine   Pipeline/GuidanceStrategy.cs:32-41
//   EulerScheduler.Step              Sampling/Schedulers.cs:270-280
//   EulerAncestralScheduler.Step     Sampling/Schedulers.cs:298-333
//   DpmPlusPlus2MScheduler.Step      Sampling/Schedulers.cs:348-385
//   DpmPlusPlus2MSdeScheduler.Step   Sampling/Schedulers.cs:404-445
//   Epsilon / Velocity / FlowPrediction.Denoise, Derivative
//                                    Sampling/Prediction.cs
#include <algorithm>

#include "nd_common.cuh"
#include "nd_internal.h"

namespace nd {

namespace {

struct SamplerScalars {
  int sampler, prediction, branches, second_order;
  float guidance, sigma, sigma_next, next_input_scale;
  double up, down, rescale, noise_scale, shrink, weight;
};

__device__ __forceinline__ double dbl(float x) { return static_cast<double>(x); }

// Prediction.Denoise: the clean latent from the prediction at level sigma.
__device__ __forceinline__ float denoise(const SamplerScalars& c, float out, float s, double sigma) {
  if (c.prediction == ND_PRED_VELOCITY) {
    const double variance = __dadd_rn(__dmul_rn(sigma, sigma), 1.0);
    const double skip = __ddiv_rn(1.0, variance);
    const double output = __ddiv_rn(sigma, __dsqrt_rn(variance));
    return __double2float_rn(__dsub_rn(__dmul_rn(dbl(s), skip), __dmul_rn(dbl(out), output)));
  }
  return __double2float_rn(__dsub_rn(dbl(s), __dmul_rn(sigma, dbl(out))));  // epsilon, flow
}

// Prediction.Derivative: d(sample)/d(sigma).
__device__ __forceinline__ float derivative(const SamplerScalars& c, float out, float s, double sigma) {
  if (c.prediction == ND_PRED_VELOCITY) {
    const float d = denoise(c, out, s, sigma);
    return __double2float_rn(__ddiv_rn(dbl(__fsub_rn(s, d)), sigma));  // float difference, double quotient
  }
  return out;  // epsilon and flow predict the derivative itself
}

__global__ void sampler_step_kernel(SamplerScalars c, long long n, const float* __restrict__ out,
                                    float* __restrict__ sample, float* __restrict__ last,
                                    const float* __restrict__ noise, float* __restrict__ denoised_out,
                                    float* __restrict__ next_input) {
  const double sigma = dbl(c.sigma);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float p = out[i];
    if (c.branches == 2) {
      const float cond = out[n + i];
      p = __fadd_rn(p, __fmul_rn(c.guidance, __fsub_rn(cond, p)));
    }
    float s = sample[i];
    if (denoised_out) denoised_out[i] = denoise(c, p, s, sigma);
    switch (c.sampler) {
      case ND_SAMPLER_EULER: {
        const float delta = __fsub_rn(c.sigma_next, c.sigma);
        s = __fadd_rn(s, __fmul_rn(derivative(c, p, s, sigma), delta));
        break;
      }
      case ND_SAMPLER_EULER_A: {
        const float d = derivative(c, p, s, sigma);
        const float delta = __double2float_rn(__dsub_rn(c.down, sigma));
        if (c.rescale == 1.0) {
          const float up_scale = __double2float_rn(c.up);
          s = __fadd_rn(s, __fadd_rn(__fmul_rn(d, delta), __fmul_rn(noise[i], up_scale)));
        } else {
          const float moved = __fadd_rn(s, __fmul_rn(d, delta));
          s = __double2float_rn(__dadd_rn(__dmul_rn(c.rescale, dbl(moved)), __dmul_rn(dbl(noise[i]), c.noise_scale)));
        }
        break;
      }
      case ND_SAMPLER_DPMPP_2M: {
        const float den = denoise(c, p, s, sigma);
        if (c.sigma_next <= 0.f) {
          s = den;
          break;
        }
        const double pred = c.second_order
                                ? __dsub_rn(__dmul_rn(__dadd_rn(1.0, c.weight), dbl(den)), __dmul_rn(c.weight, dbl(last[i])))
                                : dbl(den);
        s = __double2float_rn(__dadd_rn(__dmul_rn(c.shrink, dbl(s)), __dmul_rn(__dsub_rn(1.0, c.shrink), pred)));
        last[i] = den;
        break;
      }
      default: {  // ND_SAMPLER_DPMPP_2M_SDE
        const float den = denoise(c, p, s, sigma);
        if (c.sigma_next <= 0.f) {
          s = den;
          break;
        }
        const double keep = __dmul_rn(c.shrink, c.shrink);
        const double take = __dsub_rn(1.0, keep);
        double next = __dadd_rn(__dmul_rn(keep, dbl(s)), __dmul_rn(take, dbl(den)));
        if (c.second_order) next = __dadd_rn(next, __dmul_rn(c.weight, dbl(__fsub_rn(den, last[i]))));
        const float noise_scale = __double2float_rn(c.noise_scale);
        s = __double2float_rn(__dadd_rn(__dmul_rn(c.rescale, next), dbl(__fmul_rn(noise[i], noise_scale))));
        last[i] = den;
        break;
      }
    }
    sample[i] = s;
    if (next_input) next_input[i] = __fmul_rn(s, c.next_input_scale);
  }
}

}  // namespace

int sampler_step(const nd_sampler_args& a, cudaStream_t stream) {
  if (a.sampler < ND_SAMPLER_EULER || a.sampler > ND_SAMPLER_DPMPP_2M_SDE)
    return fail(ND_ERR_INVALID, "sampler_step: unknown sampler");
  if (a.prediction < ND_PRED_EPSILON || a.prediction > ND_PRED_FLOW)
    return fail(ND_ERR_INVALID, "sampler_step: unknown prediction type");
  if (a.n <= 0 || (a.branches != 1 && a.branches != 2)) return fail(ND_ERR_INVALID, "sampler_step: bad shape");
  if (!a.out || !a.sample) return fail(ND_ERR_INVALID, "sampler_step: null operand");
  const bool dpm = a.sampler == ND_SAMPLER_DPMPP_2M || a.sampler == ND_SAMPLER_DPMPP_2M_SDE;
  if (dpm && !a.last_denoised) return fail(ND_ERR_INVALID, "sampler_step: DPM++ needs last_denoised");
  const bool stochastic = a.sampler == ND_SAMPLER_EULER_A || a.sampler == ND_SAMPLER_DPMPP_2M_SDE;
  if (stochastic && !a.noise && !(a.sampler == ND_SAMPLER_DPMPP_2M_SDE && a.sigma_next <= 0.f))
    return fail(ND_ERR_INVALID, "sampler_step: this sampler needs the step's noise");
  if (a.sigma <= 0.f) return fail(ND_ERR_INVALID, "sampler_step: sigma must be positive");
  SamplerScalars c{};
  c.sampler = a.sampler;
  c.prediction = a.prediction;
  c.branches = a.branches;
  c.second_order = a.second_order ? 1 : 0;
  c.guidance = a.guidance;
  c.sigma = a.sigma;
  c.sigma_next = a.sigma_next;
  c.next_input_scale = a.next_input_scale;
  c.up = a.up;
  c.down = a.down;
  c.rescale = a.rescale;
  c.noise_scale = a.noise_scale;
  c.shrink = a.shrink;
  c.weight = a.weight;
  const unsigned grid = static_cast<unsigned>(std::min<long long>((a.n + 255) / 256, sm_count() * 8LL));
  sampler_step_kernel<<<grid, 256, 0, stream>>>(c, a.n, a.out, a.sample, a.last_denoised, a.noise,
                                                a.denoised_out, a.next_input);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd

extern "C" int nd_op_sampler_step(const nd_sampler_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_sampler_step: null args");
  return nd::sampler_step(*args, static_cast<cudaStream_t>(stream));
}
