// Memory-bound kernels of the denoiser step: adaLN modulation (LayerNorm
// without affine, x (1 + scale) + shift), RMSNorm, the modulation GEMVs,
// patchify / unpatchify. All are one pass over HBM with 128-bit accesses and
// warp-shuffle reductions; their roofline is HBM bandwidth.
#include <algorithm>
#include <climits>

#include "nd_common.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Four consecutive values at element idx; ND_BF16X2 puts the lo halves
// lo_off elements further along the row.
__device__ __forceinline__ void store4(void* out, long long idx, float4 v, int out_type,
                                       long long lo_off = 0) {
  if (out_type == ND_BF16X2) {
    uint2 h, l;
    pack_split(v.x, v.y, h.x, l.x);
    pack_split(v.z, v.w, h.y, l.y);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + idx) = h;
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + idx + lo_off) = l;
  } else if (out_type == ND_F32) {
    reinterpret_cast<float4*>(static_cast<float*>(out) + idx)[0] = v;
  } else if (out_type == ND_F16) {
    uint2 p = make_uint2(pack_f16(v.x, v.y), pack_f16(v.z, v.w));
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + idx) = p;
  } else {
    uint2 p = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + idx) = p;
  }
}

// 128 threads (4 warps) per row, two rows per 256-thread block; V float4 per
// thread hold the row (width <= 512 * V). y = LN(x) * (1 + scale[g]) + shift[g]
// (Transformer.Modulate, Graph/Transformer.cs:72-80), statistics in fp32 over
// the row held in registers: the mean first, then the centred second moment
// (the two-pass form of CpuMath.LayerNorm, Tensors/CpuMath.cs:100-115).
template <int V>
__global__ void __launch_bounds__(256) modulate_kernel(const float* __restrict__ x, long long ldx,
                                                       void* __restrict__ y, long long ldy,
                                                       int out_type, int rows, int width,
                                                       const float* __restrict__ shift,
                                                       const float* __restrict__ scale,
                                                       int vec_stride, int split, float eps,
                                                       int affine) {
  griddep_launch();
  griddep_wait();
  __shared__ float red[2][2][4];
  const int half = threadIdx.x >> 7;        // which of the block's two rows
  const int t = threadIdx.x & 127;
  const int w = t >> 5;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 2 + half;
  const bool live = row < rows;
  const int w4 = width >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(live ? row : 0) * ldx);
  float4 v[V];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = t + 128 * i;
    v[i] = (live && c < w4) ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  if (lane == 0) red[half][0][w] = s;
  __syncthreads();
  const float mean = (red[half][0][0] + red[half][0][1] + red[half][0][2] + red[half][0][3]) / width;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = t + 128 * i;
    if (c < w4) {
      const float a = v[i].x - mean, b = v[i].y - mean, cc = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (cc * cc + d * d);
    }
  }
  q = warp_sum(q);
  if (lane == 0) red[half][1][w] = q;
  __syncthreads();
  if (!live) return;
  const float var = (red[half][1][0] + red[half][1][1] + red[half][1][2] + red[half][1][3]) / width;
  const float rstd = rsqrtf(var + eps);
  const int g = row >= split ? 1 : 0;
  const float4* sc = reinterpret_cast<const float4*>(scale + g * vec_stride);
  const float4* sh = shift ? reinterpret_cast<const float4*>(shift + g * vec_stride) : nullptr;
  const float one = affine ? 0.f : 1.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = t + 128 * i;
    if (c < w4) {
      const float4 k = __ldg(sc + c);
      const float4 b = sh ? __ldg(sh + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 o;
      o.x = (v[i].x - mean) * rstd * (one + k.x) + b.x;
      o.y = (v[i].y - mean) * rstd * (one + k.y) + b.y;
      o.z = (v[i].z - mean) * rstd * (one + k.z) + b.z;
      o.w = (v[i].w - mean) * rstd * (one + k.w) + b.w;
      store4(y, static_cast<long long>(row) * ldy + 4 * c, o, out_type, width);
    }
  }
}

// The same modulation for a 16-bit output (bf16 / fp16: the operand of the
// next GEMM), as a persistent loop: each block keeps one pair of rows (128
// threads per row) in registers while the next pair's loads are already in
// flight, so the grid is one wave of resident blocks with no tail and no
// block launches per row pair. A thread covers the same columns of every
// row, so it keeps its columns of (1 + scale) and shift in registers (loaded
// again only when a row's vector group differs from its previous row's), and
// the arithmetic runs as paired f32x2 operations: inside the power-capped DiT
// step the kernel is bound by instruction issue, not bytes. The statistics
// are those of modulate_kernel (the mean, then the centred second moment over
// the registers); the output is (x * rstd - mean * rstd) * (1 + scale) + shift.
// The two block-wide reductions of an iteration use a parity-indexed slot so
// the next iteration's writes never race this one's reads.
template <int V, int F16OUT>
__global__ void __launch_bounds__(256, V <= 6 ? 2 : 1) modulate16_kernel(const float* __restrict__ x, long long ldx,
                                                            uint16_t* __restrict__ y, long long ldy, int rows,
                                                            int width, const float* __restrict__ shift,
                                                            const float* __restrict__ scale, int vec_stride,
                                                            int split, float eps, int affine) {
  griddep_launch();
  griddep_wait();
  __shared__ float red[2][2][2][4];  // [parity][row of the pair][mean / second moment][warp]
  const int half = threadIdx.x >> 7;
  const int t = threadIdx.x & 127;
  const int w = t >> 5;
  const int lane = threadIdx.x & 31;
  const int w4 = width >> 2;
  const int pairs = (rows + 1) >> 1;
  const float one = affine ? 0.f : 1.f;
  auto load_row = [&](int row, float4 (&v)[V]) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(row < rows ? row : 0) * ldx);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = t + 128 * i;
      v[i] = (row < rows && c < w4) ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 k1[V], sb[V];  // this thread's columns of (1 + scale) and shift for vector group cur_g
  int cur_g = -1;
  auto load_vecs = [&](int g) {
    const float4* sc = reinterpret_cast<const float4*>(scale + g * vec_stride);
    const float4* sh = shift ? reinterpret_cast<const float4*>(shift + g * vec_stride) : nullptr;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = t + 128 * i;
      float4 k = make_float4(0.f, 0.f, 0.f, 0.f), bb = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < w4) {
        k = __ldg(sc + c);
        if (sh) bb = __ldg(sh + c);
      }
      k1[i] = make_float4(one + k.x, one + k.y, one + k.z, one + k.w);
      sb[i] = bb;
    }
    cur_g = g;
  };
  float4 v[V], nv[V];
  int pair = blockIdx.x;
  if (pair < pairs) load_row(2 * pair + half, v);
  for (int it = 0; pair < pairs; ++it) {
    const int next = pair + gridDim.x;
    if (next < pairs) load_row(2 * next + half, nv);
    const int row = 2 * pair + half;
    const int par = it & 1;
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      s2 = fadd2(s2, make_float2(v[i].x, v[i].y));
      s2 = fadd2(s2, make_float2(v[i].z, v[i].w));
    }
    float s = warp_sum(s2.x + s2.y);
    if (lane == 0) red[par][half][0][w] = s;
    __syncthreads();
    const float mean = (red[par][half][0][0] + red[par][half][0][1] + red[par][half][0][2] + red[par][half][0][3]) / width;
    const float2 nm2 = make_float2(-mean, -mean);
    float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      if (t + 128 * i < w4) {
        const float2 d0 = fadd2(make_float2(v[i].x, v[i].y), nm2);
        const float2 d1 = fadd2(make_float2(v[i].z, v[i].w), nm2);
        q2 = ffma2(d0, d0, q2);
        q2 = ffma2(d1, d1, q2);
      }
    }
    const float q = warp_sum(q2.x + q2.y);
    if (lane == 0) red[par][half][1][w] = q;
    __syncthreads();
    if (row < rows) {
      const float var = (red[par][half][1][0] + red[par][half][1][1] + red[par][half][1][2] + red[par][half][1][3]) / width;
      const float rstd = rsqrtf(var + eps);
      const int g = row >= split ? 1 : 0;
      if (g != cur_g) load_vecs(g);
      // n = x * rstd - mean * rstd, y = n * (1 + scale) + shift: two paired
      // FMAs per two values
      const float2 rs2 = make_float2(rstd, rstd);
      const float2 nb2 = make_float2(-mean * rstd, -mean * rstd);
      uint2* yr = reinterpret_cast<uint2*>(y + static_cast<long long>(row) * ldy);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int c = t + 128 * i;
        if (c < w4) {
          const float2 o0 = ffma2(ffma2(make_float2(v[i].x, v[i].y), rs2, nb2), make_float2(k1[i].x, k1[i].y),
                                  make_float2(sb[i].x, sb[i].y));
          const float2 o1 = ffma2(ffma2(make_float2(v[i].z, v[i].w), rs2, nb2), make_float2(k1[i].z, k1[i].w),
                                  make_float2(sb[i].z, sb[i].w));
          yr[c] = F16OUT ? make_uint2(pack_f16(o0.x, o0.y), pack_f16(o1.x, o1.y))
                         : make_uint2(pack_bf16(o0.x, o0.y), pack_bf16(o1.x, o1.y));
        }
      }
    }
    pair = next;
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = nv[i];
  }
}

// RMSNorm over rows (CpuMath.RmsNorm, Tensors/CpuMath.cs:128-146):
// y = x * rsqrt(mean(x^2) + eps) * (w + plus_one). x fp32 or bf16/f16.
template <int V>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void* __restrict__ x, int in_type,
                                                      long long ldx, void* __restrict__ y,
                                                      long long ldy, int out_type, int rows,
                                                      int width, const float* __restrict__ w,
                                                      float plus_one, float eps, int silu_after) {
  griddep_launch();
  griddep_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int w4 = width >> 2;
  float4 v[V];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < w4) {
      if (in_type == ND_F32) {
        t = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + static_cast<long long>(warp) * ldx) + c);
      } else {
        const uint2 p = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + static_cast<long long>(warp) * ldx) + c);
        if (in_type == ND_F16) {
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&p.x));
          const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&p.y));
          t = make_float4(a.x, a.y, b.x, b.y);
        } else {
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&p.x));
          const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&p.y));
          t = make_float4(a.x, a.y, b.x, b.y);
        }
      }
    }
    v[i] = t;
    s += (t.x * t.x + t.y * t.y) + (t.z * t.z + t.w * t.w);
  }
  const float r = rsqrtf(warp_sum(s) / width + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c < w4) {
      float4 k = w ? __ldg(reinterpret_cast<const float4*>(w) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (!w) plus_one = 1.f;
      float4 o;
      o.x = v[i].x * r * (k.x + plus_one);
      o.y = v[i].y * r * (k.y + plus_one);
      o.z = v[i].z * r * (k.z + plus_one);
      o.w = v[i].w * r * (k.w + plus_one);
      if (silu_after) {
        o.x = silu(o.x);
        o.y = silu(o.y);
        o.z = silu(o.z);
        o.w = silu(o.w);
      }
      store4(y, static_cast<long long>(warp) * ldy + 4 * c, o, out_type, width);
    }
  }
}

int pick_bucket(int width) {
  const int per_lane = (width / 4 + 31) / 32;
  if (per_lane <= 2) return 2;
  if (per_lane <= 4) return 4;
  if (per_lane <= 8) return 8;
  if (per_lane <= 16) return 16;
  if (per_lane <= 24) return 24;
  if (per_lane <= 32) return 32;
  return 0;
}

// y[b][n] = act(sum_k W[n][k] * pre(x[b][k]) + bias[n]); W bf16/f16 [N, K]
// (w_type 0 / 1), or a bf16 hi|lo pair [N, 2K] (w_type 2, fp32 weights);
// x fp32 [B, K] (B <= 4); one warp per output row, x staged in shared memory.
// The modulation vectors of every block at once (one HBM pass over the
// modulation weights: QwenImageDit's modulation.1, AnimaDit.Modulation).
__global__ void __launch_bounds__(256) gemv_kernel(const uint16_t* __restrict__ W, int w_type,
                                                   long long N, int K, const float* __restrict__ x,
                                                   int B, int pre, const float* __restrict__ bias,
                                                   int act, float* __restrict__ y, long long xrows,
                                                   int nvec, long long bias_period) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float xs[];
  for (int i = threadIdx.x; i < nvec * K; i += blockDim.x) {
    float v = x[i];
    if (pre == 1) v = v / (1.0f + __expf(-v));
    xs[i] = v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int k8 = K >> 3;
  for (long long n = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; n < N;
       n += warps) {
    const bool split = w_type == 2;
    const uint4* wr = reinterpret_cast<const uint4*>(W + n * K * (split ? 2 : 1));
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // Four 16-byte loads per lane in flight before any arithmetic: the
    // weight stream is read once, so the loop is bound by bytes in flight.
    for (int c0 = lane; c0 < k8; c0 += 128) {
      uint4 p[4], q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        p[u] = q[u] = make_uint4(0u, 0u, 0u, 0u);
        if (c < k8) {
          asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(p[u].x), "=r"(p[u].y), "=r"(p[u].z), "=r"(p[u].w)
                       : "l"(wr + c));
          if (split)
            asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(q[u].x), "=r"(q[u].y), "=r"(q[u].z), "=r"(q[u].w)
                         : "l"(wr + k8 + c));
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        if (c >= k8) break;
        float wv[8];
        const uint32_t uh[4] = {p[u].x, p[u].y, p[u].z, p[u].w};
        const uint32_t ul[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 f;
          if (split) f = unpack_split(uh[i], ul[i]);
          else if (w_type == 1) f = __half22float2(*reinterpret_cast<const __half2*>(&uh[i]));
          else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uh[i]));
          wv[2 * i] = f.x;
          wv[2 * i + 1] = f.y;
        }
#pragma unroll 4
        for (int b = 0; b < 4; ++b) {
          if (b < B) {
            const float* xb = xs + (xrows > 0 ? (n / xrows) : b) * K + 8 * c;
            const float4 x0 = *reinterpret_cast<const float4*>(xb);
            const float4 x1 = *reinterpret_cast<const float4*>(xb + 4);
            float s0 = wv[0] * x0.x;
            s0 = fmaf(wv[1], x0.y, s0);
            s0 = fmaf(wv[2], x0.z, s0);
            s0 = fmaf(wv[3], x0.w, s0);
            float s1 = wv[4] * x1.x;
            s1 = fmaf(wv[5], x1.y, s1);
            s1 = fmaf(wv[6], x1.z, s1);
            s1 = fmaf(wv[7], x1.w, s1);
            acc[b] += s0 + s1;
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      if (b < B) {
        float v = warp_sum(acc[b]);
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

// The GEMV for 16-bit weights: one warp per output row, U 16-byte loads per
// lane issued before any arithmetic (no pair registers), so that enough bytes
// are in flight per SM to cover HBM latency at the occupancy the registers allow.
template <int F16, int U>
__global__ void __launch_bounds__(256) gemv16_kernel(const uint16_t* __restrict__ W, long long N, int K,
                                                     const float* __restrict__ x, int B, int pre,
                                                     const float* __restrict__ bias, int act,
                                                     float* __restrict__ y, long long xrows, int nvec,
                                                     long long bias_period) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float xs[];
  for (int i = threadIdx.x; i < nvec * K; i += blockDim.x) {
    float v = x[i];
    if (pre == 1) v = v / (1.0f + __expf(-v));
    xs[i] = v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int k8 = K >> 3;
  for (long long n = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; n < N;
       n += warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(W + n * K);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c0 = lane; c0 < k8; c0 += 32 * U) {
      uint4 p[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        p[u] = make_uint4(0u, 0u, 0u, 0u);
        if (c < k8)
          asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(p[u].x), "=r"(p[u].y), "=r"(p[u].z), "=r"(p[u].w)
                       : "l"(wr + c));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c >= k8) break;
        float wv[8];
        const uint32_t uh[4] = {p[u].x, p[u].y, p[u].z, p[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = F16 ? __half22float2(*reinterpret_cast<const __half2*>(&uh[i]))
                               : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uh[i]));
          wv[2 * i] = f.x;
          wv[2 * i + 1] = f.y;
        }
#pragma unroll 4
        for (int b = 0; b < 4; ++b) {
          if (b < B) {
            const float* xb = xs + (xrows > 0 ? (n / xrows) : b) * K + 8 * c;
            const float4 x0 = *reinterpret_cast<const float4*>(xb);
            const float4 x1 = *reinterpret_cast<const float4*>(xb + 4);
            float s0 = wv[0] * x0.x;
            s0 = fmaf(wv[1], x0.y, s0);
            s0 = fmaf(wv[2], x0.z, s0);
            s0 = fmaf(wv[3], x0.w, s0);
            float s1 = wv[4] * x1.x;
            s1 = fmaf(wv[5], x1.y, s1);
            s1 = fmaf(wv[6], x1.z, s1);
            s1 = fmaf(wv[7], x1.w, s1);
            acc[b] += s0 + s1;
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      if (b < B) {
        float v = warp_sum(acc[b]);
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

// The GEMV for one input vector and K = 256 * KC (the modulation GEMVs:
// every block's adaLN vectors from one timestep embedding, cfg3 13.6 GB of
// bf16 weights per step). Lane l of a warp always covers the same 8-column
// groups {l + 32 j} of K, so it holds its share of x (K / 32 floats, SiLU
// already applied) in registers for the whole launch instead of re-reading it
// from shared memory for every weight vector; each warp walks rows with a
// stride of all warps, and the KC 16-byte loads of its next row are issued
// before the arithmetic of the current one (two register buffers), so a warp
// keeps about 2 x 6 KB of weights in flight. bf16 -> fp32 is a shift or a
// mask, the products run as paired f32x2 FMAs into two partial sums.
template <int F16, int KC>
__device__ __forceinline__ void gemv_row_acc(const uint4 (&p)[KC], const float (&xv)[KC][8], float2& acc) {
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    const uint32_t u[4] = {p[j].x, p[j].y, p[j].z, p[j].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 w;
      if (F16) {
        w = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
      } else {
        w = make_float2(__uint_as_float(u[i] << 16), __uint_as_float(u[i] & 0xffff0000u));
      }
      acc = ffma2(w, make_float2(xv[j][2 * i], xv[j][2 * i + 1]), acc);
    }
  }
}

template <int F16, int KC>
__device__ __forceinline__ void gemv_row_load(const uint16_t* __restrict__ W, long long n, int lane, uint4 (&p)[KC]) {
  const uint4* wr = reinterpret_cast<const uint4*>(W + n * (256LL * KC));
#pragma unroll
  for (int j = 0; j < KC; ++j)
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(p[j].x), "=r"(p[j].y), "=r"(p[j].z), "=r"(p[j].w)
                 : "l"(wr + lane + 32 * j));
}

template <int F16, int KC>
__device__ __forceinline__ void gemv_row_finish(float2 acc, long long n, int lane, const float* __restrict__ bias,
                                                int act, float* __restrict__ y, long long bias_period) {
  float v = warp_sum(acc.x + acc.y);
  if (lane == 0) {
    if (bias) v += bias[bias_period > 0 ? n % bias_period : n];
    if (act == 1) v = v / (1.0f + __expf(-v));
    else if (act == 2) v = tanhf(v);
    y[n] = v;
  }
}

template <int F16, int KC>
__global__ void __launch_bounds__(128) gemv_rows_kernel(const uint16_t* __restrict__ W, long long N,
                                                        const float* __restrict__ x, int pre,
                                                        const float* __restrict__ bias, int act,
                                                        float* __restrict__ y, long long bias_period) {
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  float xv[KC][8];
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    const float4* xs = reinterpret_cast<const float4*>(x + 8 * (lane + 32 * j));
    const float4 a = __ldg(xs), b = __ldg(xs + 1);
    const float t[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[j][i] = pre ? t[i] / (1.0f + __expf(-t[i])) : t[i];
  }
  const long long stride = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  long long n = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  uint4 pa[KC], pb[KC];
  if (n < N) gemv_row_load<F16, KC>(W, n, lane, pa);
  while (n < N) {
    const long long n1 = n + stride;
    if (n1 < N) gemv_row_load<F16, KC>(W, n1, lane, pb);
    float2 acc = make_float2(0.f, 0.f);
    gemv_row_acc<F16, KC>(pa, xv, acc);
    gemv_row_finish<F16, KC>(acc, n, lane, bias, act, y, bias_period);
    if (n1 >= N) break;
    const long long n2 = n1 + stride;
    if (n2 < N) gemv_row_load<F16, KC>(W, n2, lane, pa);
    acc = make_float2(0.f, 0.f);
    gemv_row_acc<F16, KC>(pb, xv, acc);
    gemv_row_finish<F16, KC>(acc, n1, lane, bias, act, y, bias_period);
    n = n2;
  }
}

// RMSNorm over short 16-bit rows (an image's pixels x channels, the Wan VAE's
// channel norm): L lanes per row (L = 8, 16 or 32), each holding up to V
// 16-byte vectors, so one warp keeps 32 / L rows' bytes in flight instead of
// one row's. Same arithmetic as rmsnorm_kernel.
template <int V>
__global__ void __launch_bounds__(256) rms_rows16_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                                                         int f16, long long rows, int c8, int L,
                                                         const float* __restrict__ w, float plus_one,
                                                         float eps, int silu_after, int width) {
  griddep_launch();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const int sub = lane % L;  // lane within the row's segment
  const long long warp = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
  const long long row = warp * (32 / L) + lane / L;
  const bool live = row < rows;
  uint4 v[V];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int c = sub + k * L;
    v[k] = make_uint4(0u, 0u, 0u, 0u);
    if (live && c < c8) v[k] = __ldg(x + row * c8 + c);
    const uint32_t u[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&u[i]))
                           : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
  for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / width + eps);
  if (!live) return;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int c = sub + k * L;
    if (c >= c8) break;
    const uint32_t u[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
    uint32_t o4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&u[i]))
                     : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
      const int ch = c * 8 + 2 * i;
      const float w0 = (w ? __ldg(w + ch) : 0.f) + (w ? plus_one : 1.f);
      const float w1 = (w ? __ldg(w + ch + 1) : 0.f) + (w ? plus_one : 1.f);
      f.x = f.x * r * w0;
      f.y = f.y * r * w1;
      if (silu_after) {
        f.x = silu(f.x);
        f.y = silu(f.y);
      }
      o4[i] = f16 ? pack_f16(f.x, f.y) : pack_bf16(f.x, f.y);
    }
    y[row * c8 + c] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// latent [B][C][H][W] fp32 -> tokens [B][(H/p)(W/p)][C p p] (bf16/f16/fp32);
// feature c*p*p + m*p + n of patch (i, j) is channel c at (p*i + m, p*j + n)
// (AnimaDit.Patchify, Models/Anima/AnimaDit.cs:193-247).
__global__ void patchify_kernel(const float* __restrict__ lat, void* __restrict__ tok, int out_type,
                                int B, int C, int H, int W, int p, long long ldt) {
  const long long total = static_cast<long long>(B) * C * H * W;
  const int rows = H / p, cols = W / p, feat = C * p * p;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int w = idx % W;
    const int h = (idx / W) % H;
    const int c = (idx / (static_cast<long long>(W) * H)) % C;
    const int b = idx / (static_cast<long long>(W) * H * C);
    const int i = h / p, m = h % p, j = w / p, n = w % p;
    const long long t = static_cast<long long>(b) * rows * cols + i * cols + j;
    const long long o = t * ldt + c * p * p + m * p + n;
    const float v = lat[idx];
    if (out_type == ND_BF16X2) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      static_cast<__nv_bfloat16*>(tok)[o] = hi;
      static_cast<__nv_bfloat16*>(tok)[o + feat] = __float2bfloat16_rn(v - __bfloat162float(hi));
    } else if (out_type == ND_F32) static_cast<float*>(tok)[o] = v;
    else if (out_type == ND_F16) static_cast<__half*>(tok)[o] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(tok)[o] = __float2bfloat16_rn(v);
  }
}

// The inverse of patchify_kernel: fp32 tokens -> fp32 latent.
__global__ void unpatchify_kernel(const float* __restrict__ tok, long long ldt, float* __restrict__ lat,
                                  int B, int C, int H, int W, int p) {
  const long long total = static_cast<long long>(B) * C * H * W;
  const int rows = H / p, cols = W / p;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int w = idx % W;
    const int h = (idx / W) % H;
    const int c = (idx / (static_cast<long long>(W) * H)) % C;
    const int b = idx / (static_cast<long long>(W) * H * C);
    const int i = h / p, m = h % p, j = w / p, n = w % p;
    const long long t = static_cast<long long>(b) * rows * cols + i * cols + j;
    lat[idx] = tok[t * ldt + c * p * p + m * p + n];
  }
  (void)rows;
}

}  // namespace

int modulate(const nd_modulate_args& a, cudaStream_t stream) {
  if (a.rows <= 0 || a.width <= 0) return fail(ND_ERR_INVALID, "modulate: empty shape");
  if (a.width % 4 || a.ldx % 4 || a.ldy % 4) return fail(ND_ERR_INVALID, "modulate: width and strides must be multiples of 4");
  if (a.out_dtype != ND_F32 && a.out_dtype != ND_F16 && a.out_dtype != ND_BF16 && a.out_dtype != ND_BF16X2)
    return fail(ND_ERR_INVALID, "modulate: out_dtype must be f32, f16, bf16 or bf16x2");
  if (a.ldy < (a.out_dtype == ND_BF16X2 ? 2 : 1) * a.width)
    return fail(ND_ERR_INVALID, "modulate: ldy too small (a bf16x2 output needs 2 * width)");
  if (!a.x || !a.y || !a.scale) return fail(ND_ERR_INVALID, "modulate: null operand");
  if (a.rows > INT_MAX) return fail(ND_ERR_INVALID, "modulate: too many rows");
  if (a.width > 4096) return fail(ND_ERR_UNSUPPORTED, "modulate: width above 4096");
  const int rows = static_cast<int>(a.rows);
  const int split = a.group_split < a.rows ? static_cast<int>(a.group_split) : INT_MAX;
  const int vs = a.vec_stride ? static_cast<int>(a.vec_stride) : static_cast<int>(a.width);
  const unsigned grid = static_cast<unsigned>((rows + 1) / 2);
  const int per_thread = (static_cast<int>(a.width) / 4 + 127) / 128;
  if ((a.out_dtype == ND_BF16 || a.out_dtype == ND_F16) && (reinterpret_cast<uintptr_t>(a.y) & 7u) == 0 &&
      (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) {
    const int f16 = a.out_dtype == ND_F16;
    uint16_t* y = static_cast<uint16_t*>(a.y);
#define ND_MOD16(V, F)                                                                                        \
  do {                                                                                                        \
    int per_sm = 0;                                                                                           \
    ND_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, modulate16_kernel<V, F>, 256, 0));         \
    const unsigned g16 = static_cast<unsigned>(std::min<long long>(grid, static_cast<long long>(sm_count()) * \
                                                                             std::max(per_sm, 1)));           \
    ND_CUDA(launch_pdl(modulate16_kernel<V, F>, dim3(g16), dim3(256), 0, stream, a.x, a.ldx, y, a.ldy, rows,   \
                       static_cast<int>(a.width), a.shift, a.scale, vs, split, a.eps, a.affine));            \
  } while (0)
#define ND_MOD16V(F)                      \
    if (per_thread <= 1) ND_MOD16(1, F);  \
    else if (per_thread <= 2) ND_MOD16(2, F); \
    else if (per_thread <= 4) ND_MOD16(4, F); \
    else if (per_thread <= 6) ND_MOD16(6, F); \
    else ND_MOD16(8, F);
    if (f16) {
      ND_MOD16V(1)
    } else {
      ND_MOD16V(0)
    }
#undef ND_MOD16V
#undef ND_MOD16
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }
#define ND_MOD(V) ND_CUDA(launch_pdl(modulate_kernel<V>, dim3(grid), dim3(256), 0, stream, a.x, a.ldx, a.y, a.ldy, a.out_dtype, rows, static_cast<int>(a.width), a.shift, a.scale, vs, split, a.eps, a.affine))
  if (per_thread <= 1) ND_MOD(1);
  else if (per_thread <= 2) ND_MOD(2);
  else if (per_thread <= 4) ND_MOD(4);
  else if (per_thread <= 6) ND_MOD(6);
  else ND_MOD(8);
#undef ND_MOD
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int rmsnorm(const nd_rmsnorm_args& a, cudaStream_t stream) {
  if (a.rows <= 0 || a.width <= 0) return fail(ND_ERR_INVALID, "rmsnorm: empty shape");
  if (a.width % 4 || a.ldx % 4 || a.ldy % 4) return fail(ND_ERR_INVALID, "rmsnorm: width and strides must be multiples of 4");
  if (a.in_dtype != ND_F32 && a.in_dtype != ND_F16 && a.in_dtype != ND_BF16)
    return fail(ND_ERR_INVALID, "rmsnorm: in_dtype must be f32, f16 or bf16");
  if (a.out_dtype != ND_F32 && a.out_dtype != ND_F16 && a.out_dtype != ND_BF16 && a.out_dtype != ND_BF16X2)
    return fail(ND_ERR_INVALID, "rmsnorm: out_dtype must be f32, f16, bf16 or bf16x2");
  if (a.ldy < (a.out_dtype == ND_BF16X2 ? 2 : 1) * a.width)
    return fail(ND_ERR_INVALID, "rmsnorm: ldy too small (a bf16x2 output needs 2 * width)");
  if (!a.x || !a.y) return fail(ND_ERR_INVALID, "rmsnorm: null operand");
  // Short contiguous 16-bit rows: several rows per warp.
  const bool narrow16 = (a.in_dtype == ND_F16 || a.in_dtype == ND_BF16) && a.out_dtype == a.in_dtype &&
                        a.width % 8 == 0 && a.width <= 1280 && a.ldx == a.width && a.ldy == a.width &&
                        (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15u) == 0;
  if (narrow16) {
    const int c8 = static_cast<int>(a.width / 8);
    const int L = c8 >= 64 ? 32 : (c8 >= 24 ? 16 : 8);
    const int per = (c8 + L - 1) / L;  // vectors per lane, <= 5
    const long long warps = (a.rows + 32 / L - 1) / (32 / L);
    const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
    const int f16 = a.in_dtype == ND_F16 ? 1 : 0;
    const float po = a.plus_one ? 1.f : 0.f;
#define ND_RR(V)                                                                                               \
  ND_CUDA(launch_pdl(rms_rows16_kernel<V>, dim3(grid), dim3(256), 0, stream, static_cast<const uint4*>(a.x),    \
                     static_cast<uint4*>(a.y), f16, static_cast<long long>(a.rows), c8, L, a.weight, po, a.eps, \
                     a.silu, static_cast<int>(a.width)))
    switch (per) {
      case 1: ND_RR(1); break;
      case 2: ND_RR(2); break;
      case 3: ND_RR(3); break;
      case 4: ND_RR(4); break;
      default: ND_RR(5); break;
    }
#undef ND_RR
    return ND_OK;
  }
  const int bucket = pick_bucket(static_cast<int>(a.width));
  if (!bucket) return fail(ND_ERR_UNSUPPORTED, "rmsnorm: width above 4096");
  const int rows = static_cast<int>(a.rows);
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
#define ND_RMS(V) ND_CUDA(launch_pdl(rmsnorm_kernel<V>, dim3(grid), dim3(256), 0, stream, a.x, a.in_dtype, a.ldx, a.y, a.ldy, a.out_dtype, rows, static_cast<int>(a.width), a.weight, a.plus_one ? 1.f : 0.f, a.eps, a.silu))
  switch (bucket) {
    case 2: ND_RMS(2); break;
    case 4: ND_RMS(4); break;
    case 8: ND_RMS(8); break;
    case 16: ND_RMS(16); break;
    case 24: ND_RMS(24); break;
    default: ND_RMS(32); break;
  }
#undef ND_RMS
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int gemv(const nd_gemv_args& a, cudaStream_t stream) {
  if (a.n <= 0 || a.k <= 0 || a.batch <= 0 || a.batch > 4) return fail(ND_ERR_INVALID, "gemv: bad shape (batch 1..4)");
  if (a.x_rows_per_vec < 0 || a.bias_period < 0) return fail(ND_ERR_INVALID, "gemv: negative period");
  if (a.x_rows_per_vec > 0 && a.batch != 1) return fail(ND_ERR_INVALID, "gemv: x_rows_per_vec needs batch 1");
  const long long nvec = a.x_rows_per_vec > 0 ? (a.n + a.x_rows_per_vec - 1) / a.x_rows_per_vec : a.batch;
  if (a.k * nvec > 12288) return fail(ND_ERR_UNSUPPORTED, "gemv: input vectors above 12288 floats");
  if (a.w_dtype == ND_I8) {
    if (!a.w || !a.x || !a.y) return fail(ND_ERR_INVALID, "gemv: null operand");
    return gemv_w8(a, stream);
  }
  if (a.k % 8) return fail(ND_ERR_INVALID, "gemv: k must be a multiple of 8");
  if (a.w_dtype != ND_BF16 && a.w_dtype != ND_F16 && a.w_dtype != ND_BF16X2)
    return fail(ND_ERR_INVALID, "gemv: weight must be bf16, f16, bf16x2 or int8");
  if (!a.w || !a.x || !a.y) return fail(ND_ERR_INVALID, "gemv: null operand");
  // The kernels read W in 16-byte vectors.
  if (reinterpret_cast<uintptr_t>(a.w) & 15u) return fail(ND_ERR_INVALID, "gemv: weight must be 16-byte aligned");
  const size_t shmem = static_cast<size_t>(a.k) * nvec * sizeof(float);
  long long blocks = (a.n + 7) / 8;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (a.w_dtype != ND_BF16X2 && nvec == 1 && a.k % 256 == 0 && a.k / 256 <= 12 &&
      (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0) {
    // One input vector and K a multiple of 256: x in registers, two rows in flight per warp.
    const int kc = static_cast<int>(a.k / 256);
    const uint16_t* w = static_cast<const uint16_t*>(a.w);
    const int pre = a.pre_silu ? 1 : 0;
    // One wave of resident blocks (the register budget allows about two per SM).
#define ND_GR(F, KC)                                                                                          \
  do {                                                                                                        \
    int per_sm = 0;                                                                                           \
    ND_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_rows_kernel<F, KC>, 128, 0));         \
    const long long cap = static_cast<long long>(sm_count()) * std::max(per_sm, 1);                           \
    const unsigned g = static_cast<unsigned>(std::min<long long>((a.n + 3) / 4, cap));                       \
    ND_CUDA(launch_pdl(gemv_rows_kernel<F, KC>, dim3(g), dim3(128), 0, stream, w, a.n, a.x, pre, a.bias,      \
                       a.act, a.y, a.bias_period));                                                           \
  } while (0)
#define ND_GRK(F)                   \
  switch (kc) {                     \
    case 1: ND_GR(F, 1); break;     \
    case 2: ND_GR(F, 2); break;     \
    case 3: ND_GR(F, 3); break;     \
    case 4: ND_GR(F, 4); break;     \
    case 5: ND_GR(F, 5); break;     \
    case 6: ND_GR(F, 6); break;     \
    case 7: ND_GR(F, 7); break;     \
    case 8: ND_GR(F, 8); break;     \
    case 9: ND_GR(F, 9); break;     \
    case 10: ND_GR(F, 10); break;   \
    case 11: ND_GR(F, 11); break;   \
    default: ND_GR(F, 12); break;   \
  }
    if (a.w_dtype == ND_F16) {
      ND_GRK(1)
    } else {
      ND_GRK(0)
    }
#undef ND_GRK
#undef ND_GR
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }
  if (a.w_dtype != ND_BF16X2) {
    const unsigned g = static_cast<unsigned>(blocks);
    const uint16_t* w = static_cast<const uint16_t*>(a.w);
    const int k = static_cast<int>(a.k);
    const int pre = a.pre_silu ? 1 : 0;
    const int nv = static_cast<int>(nvec);
    if (a.w_dtype == ND_F16)
      ND_CUDA(launch_pdl(gemv16_kernel<1, 8>, dim3(g), dim3(256), shmem, stream, w, a.n, k, a.x, a.batch, pre,
                         a.bias, a.act, a.y, a.x_rows_per_vec, nv, a.bias_period));
    else
      ND_CUDA(launch_pdl(gemv16_kernel<0, 8>, dim3(g), dim3(256), shmem, stream, w, a.n, k, a.x, a.batch, pre,
                         a.bias, a.act, a.y, a.x_rows_per_vec, nv, a.bias_period));
    return ND_OK;
  }
  gemv_kernel<<<static_cast<unsigned>(blocks), 256, shmem, stream>>>(
      static_cast<const uint16_t*>(a.w), a.w_dtype == ND_BF16X2 ? 2 : (a.w_dtype == ND_F16 ? 1 : 0), a.n, static_cast<int>(a.k), a.x,
      a.batch, a.pre_silu ? 1 : 0, a.bias, a.act, a.y, a.x_rows_per_vec, static_cast<int>(nvec),
      a.bias_period);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int patchify(const float* lat, void* tok, int out_dtype, int B, int C, int H, int W, int p,
             int64_t ldt, cudaStream_t stream) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || p <= 0 || H % p || W % p)
    return fail(ND_ERR_INVALID, "patchify: latent does not divide into patches");
  if (out_dtype != ND_F32 && out_dtype != ND_F16 && out_dtype != ND_BF16 && out_dtype != ND_BF16X2)
    return fail(ND_ERR_INVALID, "patchify: out_dtype must be f32, f16, bf16 or bf16x2");
  if (ldt < static_cast<int64_t>(C) * p * p * (out_dtype == ND_BF16X2 ? 2 : 1))
    return fail(ND_ERR_INVALID, "patchify: ldt smaller than the token width");
  const long long total = static_cast<long long>(B) * C * H * W;
  const unsigned grid = static_cast<unsigned>(std::min<long long>((total + 255) / 256, sm_count() * 16LL));
  patchify_kernel<<<grid, 256, 0, stream>>>(lat, tok, out_dtype, B, C, H, W, p, ldt);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int unpatchify(const float* tok, int64_t ldt, float* lat, int B, int C, int H, int W, int p,
               cudaStream_t stream) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || p <= 0 || H % p || W % p)
    return fail(ND_ERR_INVALID, "unpatchify: latent does not divide into patches");
  const long long total = static_cast<long long>(B) * C * H * W;
  const unsigned grid = static_cast<unsigned>(std::min<long long>((total + 255) / 256, sm_count() * 16LL));
  unpatchify_kernel<<<grid, 256, 0, stream>>>(tok, ldt, lat, B, C, H, W, p);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd
