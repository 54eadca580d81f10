// int8 weight storage: the device-side quantizer and the int8 GEMV.
//
// quantize_weights restates BlockQuantizer.Quantize
// (Tensors/BlockQuantizer.cs:34-105) per row and group of `group` columns:
//   peak   = max |w| over the group
//   scale  = peak / 127, stored as fp16 (round to nearest even) for the
//            reference's blocks, or kept fp32 (per-output-channel scheme)
//   q      = clamp(rint(w * (1 / stored)), -127, 127); a zero stored scale
//            leaves the group zero
// with IEEE division and round-half-even, so q and the scales match the host
// quantizer (and the oracle's restatement) bit for bit.
#include <algorithm>
#include <climits>

#include "nd_common.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {

__device__ __forceinline__ float load_as_float(const void* src, int dt, long long i) {
  if (dt == ND_F32) return static_cast<const float*>(src)[i];
  if (dt == ND_F16) return __half2float(static_cast<const __half*>(src)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
}

// One block per row; the row's groups are spread over the block's warps
// (group <= 32: one lane per element; wider groups: lanes stride the group).
__global__ void __launch_bounds__(256) quantize_kernel(const void* __restrict__ src, int src_dt,
                                                       long long rows, int cols, int group,
                                                       int scale_f16, int8_t* __restrict__ q,
                                                       void* __restrict__ scales) {
  const long long r = blockIdx.x;
  if (r >= rows) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int groups = cols / group;
  const long long base = r * cols;
  for (int g = warp; g < groups; g += nwarps) {
    const long long g0 = base + static_cast<long long>(g) * group;
    float peak = 0.f;
    for (int i = lane; i < group; i += 32) peak = fmaxf(peak, fabsf(load_as_float(src, src_dt, g0 + i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    float stored;
    const long long si = r * groups + g;
    if (scale_f16) {
      const __half h = __float2half_rn(__fdiv_rn(peak, 127.0f));
      stored = __half2float(h);
      if (lane == 0) static_cast<__half*>(scales)[si] = h;
    } else {
      stored = __fdiv_rn(peak, 127.0f);
      if (lane == 0) static_cast<float*>(scales)[si] = stored;
    }
    const float inverse = stored != 0.f ? __fdiv_rn(1.0f, stored) : 0.f;
    for (int i = lane; i < group; i += 32) {
      float v = 0.f;
      if (stored != 0.f) {
        v = rintf(__fmul_rn(load_as_float(src, src_dt, g0 + i), inverse));
        v = fmaxf(-127.f, fminf(127.f, v));
      }
      q[g0 + i] = static_cast<int8_t>(v);
    }
  }
}

__device__ __forceinline__ float warp_sum_w8(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// y[b][n] = act(sum_k q[n][k] * scale(n, k) * pre(x[b][k]) + bias[n]) for int8
// q; one warp per output row, 16 weights (one 16-byte load) per lane step.
__global__ void __launch_bounds__(256) gemv_w8_kernel(const int8_t* __restrict__ W, long long N, int K,
                                                      const void* __restrict__ scales, int scale_f16,
                                                      int group, int scale_cols,
                                                      const float* __restrict__ x, int B, int pre,
                                                      const float* __restrict__ bias, int act,
                                                      float* __restrict__ y, long long xrows, int nvec,
                                                      long long bias_period) {
  extern __shared__ float xs[];
  for (int i = threadIdx.x; i < nvec * K; i += blockDim.x) {
    float v = x[i];
    if (pre == 1) v = v / (1.0f + __expf(-v));
    xs[i] = v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int k16 = K >> 4;
  for (long long n = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; n < N;
       n += warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(W + n * K);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // Four 16-byte loads (and their scales) per lane in flight before any
    // arithmetic: the weight stream is read once, bound by bytes in flight.
    for (int c0 = lane; c0 < k16; c0 += 128) {
      uint4 p[4];
      float sc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        p[u] = make_uint4(0u, 0u, 0u, 0u);
        sc[u] = 0.f;
        if (c < k16) {
          asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(p[u].x), "=r"(p[u].y), "=r"(p[u].z), "=r"(p[u].w)
                       : "l"(wr + c));
          const long long si = n * scale_cols + (c * 16) / group;
          sc[u] = scale_f16 ? __half2float(static_cast<const __half*>(scales)[si])
                            : static_cast<const float*>(scales)[si];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        if (c >= k16) break;
        float wv[16];
        const uint32_t w4[4] = {p[u].x, p[u].y, p[u].z, p[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float f[4];
          i8x4_to_f32(w4[i], f);
#pragma unroll
          for (int j = 0; j < 4; ++j) wv[4 * i + j] = f[j] * sc[u];
        }
#pragma unroll 4
        for (int b = 0; b < 4; ++b) {
          if (b < B) {
            const float* xb = xs + (xrows > 0 ? (n / xrows) : b) * K + 16 * c;
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) sum += wv[i] * xb[i];
            acc[b] += sum;
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      if (b < B) {
        float v = acc[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) {
          if (bias) v += bias[bias_period > 0 ? n % bias_period : n];
          if (act == 1) v = v / (1.0f + __expf(-v));
          else if (act == 2) v = tanhf(v);
          y[static_cast<long long>(b) * N + n] = v;
        }
      }
    }
  }
}

// The int8 GEMV for one input vector and K = 512 * KC (cfg4's modulation
// GEMV: 6.8 GB of int8 weights per step): as gemv_rows_kernel, lane l always
// covers the same 16-column groups {l + 32 j}, so its 16 * KC values of x
// (SiLU applied) stay in registers, and each warp keeps two rows' loads in
// flight. The scale is constant over a lane's 16 weights (per output channel,
// or a group of 16 k or more), so it multiplies each 16-term partial sum once:
// sum_j s_j * sum_i q_i x_i.
template <int KC>
__device__ __forceinline__ void gemv_w8_row_load(const int8_t* __restrict__ W, long long n, int lane,
                                                 uint4 (&p)[KC]) {
  const uint4* wr = reinterpret_cast<const uint4*>(W + n * (512LL * KC));
#pragma unroll
  for (int j = 0; j < KC; ++j)
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(p[j].x), "=r"(p[j].y), "=r"(p[j].z), "=r"(p[j].w)
                 : "l"(wr + lane + 32 * j));
}

template <int KC>
__device__ __forceinline__ float gemv_w8_row_dot(const uint4 (&p)[KC], const float (&xv)[KC][16], long long n,
                                                 int lane, const void* __restrict__ scales, int scale_f16,
                                                 int group, int scale_cols) {
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    const long long si = n * scale_cols + (16 * (lane + 32 * j)) / group;
    const float s = scale_f16 ? __half2float(__ldg(static_cast<const __half*>(scales) + si))
                              : __ldg(static_cast<const float*>(scales) + si);
    const uint32_t w4[4] = {p[j].x, p[j].y, p[j].z, p[j].w};
    float2 part = make_float2(0.f, 0.f);
    const float2 m2 = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u = w4[i] ^ 0x80808080u;  // exact int8 -> fp32 (magic 2^23 + 128 offset)
      const float2 lo = fadd2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)),
                                          __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541u))), m2);
      const float2 hi = fadd2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542u)),
                                          __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543u))), m2);
      part = ffma2(lo, make_float2(xv[j][4 * i], xv[j][4 * i + 1]), part);
      part = ffma2(hi, make_float2(xv[j][4 * i + 2], xv[j][4 * i + 3]), part);
    }
    acc = fmaf(s, part.x + part.y, acc);
  }
  return acc;
}

template <int KC>
__global__ void __launch_bounds__(128) gemv_w8_rows_kernel(const int8_t* __restrict__ W, long long N,
                                                           const void* __restrict__ scales, int scale_f16,
                                                           int group, int scale_cols, const float* __restrict__ x,
                                                           int pre, const float* __restrict__ bias, int act,
                                                           float* __restrict__ y, long long bias_period) {
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  float xv[KC][16];
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    const float4* xs = reinterpret_cast<const float4*>(x + 16 * (lane + 32 * j));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 a = __ldg(xs + q);
      const float t[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[j][4 * q + i] = pre ? t[i] / (1.0f + __expf(-t[i])) : t[i];
    }
  }
  auto finish = [&](float v, long long n) {
    v = warp_sum_w8(v);
    if (lane == 0) {
      if (bias) v += bias[bias_period > 0 ? n % bias_period : n];
      if (act == 1) v = v / (1.0f + __expf(-v));
      else if (act == 2) v = tanhf(v);
      y[n] = v;
    }
  };
  const long long stride = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  long long n = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  uint4 pa[KC], pb[KC];
  if (n < N) gemv_w8_row_load<KC>(W, n, lane, pa);
  while (n < N) {
    const long long n1 = n + stride;
    if (n1 < N) gemv_w8_row_load<KC>(W, n1, lane, pb);
    finish(gemv_w8_row_dot<KC>(pa, xv, n, lane, scales, scale_f16, group, scale_cols), n);
    if (n1 >= N) break;
    const long long n2 = n1 + stride;
    if (n2 < N) gemv_w8_row_load<KC>(W, n2, lane, pa);
    finish(gemv_w8_row_dot<KC>(pb, xv, n1, lane, scales, scale_f16, group, scale_cols), n1);
    n = n2;
  }
}

}  // namespace

int quantize_weights(const void* src, int src_dtype, int64_t rows, int64_t cols, int64_t group,
                     int scale_f16, int8_t* q, void* scales, cudaStream_t stream) {
  if (!src || !q || !scales) return fail(ND_ERR_INVALID, "quantize: null operand");
  if (rows <= 0 || cols <= 0 || cols > INT_MAX || rows > INT_MAX) return fail(ND_ERR_INVALID, "quantize: bad shape");
  const int64_t g = group > 0 ? group : cols;
  if (cols % g) return fail(ND_ERR_INVALID, "quantize: columns do not split into whole groups");
  quantize_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(src, src_dtype, rows, static_cast<int>(cols),
                                                                   static_cast<int>(g), scale_f16, q, scales);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int gemv_w8(const nd_gemv_args& a, cudaStream_t stream) {
  if (!a.scales) return fail(ND_ERR_INVALID, "gemv: int8 weights need scales");
  if (a.k % 16) return fail(ND_ERR_INVALID, "gemv: int8 weights need k % 16 == 0");
  const int64_t group = a.quant_group > 0 ? a.quant_group : a.k;
  if (group % 16 || a.k % group) return fail(ND_ERR_INVALID, "gemv: quant_group must be a multiple of 16 dividing k");
  const long long nvec = a.x_rows_per_vec > 0 ? (a.n + a.x_rows_per_vec - 1) / a.x_rows_per_vec : a.batch;
  const size_t shmem = static_cast<size_t>(a.k) * nvec * sizeof(float);
  if (nvec == 1 && a.k % 512 == 0 && a.k / 512 <= 8 && (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(a.w) & 15u) == 0) {
    // One input vector, K a multiple of 512: x in registers, two rows in flight per warp.
    const int kc = static_cast<int>(a.k / 512);
    const int8_t* w = static_cast<const int8_t*>(a.w);
    const int pre = a.pre_silu ? 1 : 0;
    const int f16 = a.scale_dtype == ND_F16;
    const int g = static_cast<int>(group), sc = static_cast<int>(a.k / group);
#define ND_GW8(KC)                                                                                           \
  do {                                                                                                       \
    int per_sm = 0;                                                                                          \
    ND_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_w8_rows_kernel<KC>, 128, 0));        \
    const long long cap = static_cast<long long>(sm_count()) * std::max(per_sm, 1);                          \
    const unsigned grid = static_cast<unsigned>(std::min<long long>((a.n + 3) / 4, cap));                    \
    ND_CUDA(launch_pdl(gemv_w8_rows_kernel<KC>, dim3(grid), dim3(128), 0, stream, w, a.n, a.scales, f16, g,  \
                       sc, a.x, pre, a.bias, a.act, a.y, a.bias_period));                                    \
  } while (0)
    switch (kc) {
      case 1: ND_GW8(1); break;
      case 2: ND_GW8(2); break;
      case 3: ND_GW8(3); break;
      case 4: ND_GW8(4); break;
      case 5: ND_GW8(5); break;
      case 6: ND_GW8(6); break;
      case 7: ND_GW8(7); break;
      default: ND_GW8(8); break;
    }
#undef ND_GW8
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }
  long long blocks = (a.n + 7) / 8;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  gemv_w8_kernel<<<static_cast<unsigned>(blocks), 256, shmem, stream>>>(
      static_cast<const int8_t*>(a.w), a.n, static_cast<int>(a.k), a.scales, a.scale_dtype == ND_F16,
      static_cast<int>(group), static_cast<int>(a.k / group), a.x, a.batch, a.pre_silu ? 1 : 0, a.bias,
      a.act, a.y, a.x_rows_per_vec, static_cast<int>(nvec), a.bias_period);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd
