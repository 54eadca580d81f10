// The UNet's memory-bound kernels over NHWC fp16 activations: GroupNorm
// (+ SiLU), GEGLU, nearest 2x upsample, channel concat, NCHW <-> NHWC.
//
// GroupNorm (Layers.GroupNorm, Graph/Layers.cs:166-185: mean-variance
// normalization over (C/G, H, W) of each group, then the per-channel affine)
// runs in two launches: per-block channel and group sums, whose last block per
// image forms each group's mean and 1/sqrt(var + eps) in fp64, then one
// vectorized pass applying it (fused with the SiLU
// the ResBlocks put after it, UNetModel.ResnetBlock, Models/Sdxl/UNetModel.cs:230-254).
#include <algorithm>
#include <climits>

#include "nd_common.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {

__device__ __forceinline__ float ld16(const void* p, long long i, int f16) {
  const uint16_t h = static_cast<const uint16_t*>(p)[i];
  return f16 ? __half2float(*reinterpret_cast<const __half*>(&h))
             : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&h));
}

__device__ __forceinline__ void unpack8(const uint4& u, int f16, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[i]))
                         : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8], int f16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = f16 ? pack_f16(v[2 * i], v[2 * i + 1]) : pack_bf16(v[2 * i], v[2 * i + 1]);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Per (image, run of pixels): channel sums and sums of squares, then group
// totals. One wave of blocks (about two per SM) each streams a long run of
// pixels: threads read 16-byte vectors (8 channels), consecutive threads on
// consecutive vectors of a pixel row and several rows per pass, eight loads
// in flight, every load coalesced; each thread sums its 8 channels in fp32,
// the block adds the pixel rows' sums per channel and then each group's
// channels, in a fixed order. The last block of an image to write its
// partials (one counter per image, reset by that block) adds them per group
// in fp64 and writes the group's mean and 1/sqrt(var + eps).
constexpr int kGnChunk = 32;           // fewest pixels per block (bounds the partials)
constexpr int kGnMaxC = 3072;          // channels (shared memory: two sums per channel)
constexpr int kGnCounterBytes = 4096;  // one arrival counter per image, at the start of the scratch

template <int f16>  // fp16 (1) or bf16 (0) x, fixed at compile time so no conversion runs both ways
__global__ void __launch_bounds__(256) gn_stats_kernel(const void* __restrict__ x, int hw, int C, int G,
                                                       int chunk, float2* __restrict__ part,
                                                       unsigned* __restrict__ arrived, float eps,
                                                       float2* __restrict__ stats) {
  griddep_launch();
  griddep_wait();
  __shared__ float red[256][17];
  __shared__ float csum[2][kGnMaxC];
  __shared__ int is_last;
  const int blk = blockIdx.x, b = blockIdx.y, nblk = gridDim.x;
  const int c8 = C / 8;
  const int tpr = min(c8, 256);  // threads per pixel row
  const int rows = 256 / tpr;    // pixel rows per pass
  const int t = threadIdx.x;
  const int pr = t / tpr;
  const int p0 = blk * chunk, p1 = min(hw, p0 + chunk);
  const uint4* xv = reinterpret_cast<const uint4*>(x) + static_cast<long long>(b) * hw * c8;
  for (int j0 = 0; j0 < c8; j0 += tpr) {  // (more than 2048 channels: vector runs of 256)
    const int j = j0 + t % tpr;
    float s1[8], s2[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) s1[k] = s2[k] = 0.f;
    if (pr < rows && j < c8) {
#pragma unroll 8
      for (int p = p0 + pr; p < p1; p += rows) {
        float v[8];
        unpack8(__ldg(xv + static_cast<long long>(p) * c8 + j), f16, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          s1[k] += v[k];
          s2[k] = fmaf(v[k], v[k], s2[k]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      red[t][k] = s1[k];
      red[t][8 + k] = s2[k];
    }
    __syncthreads();
    for (int e = t; e < tpr * 8; e += 256) {  // e = vector of the run x 8 + channel
      const int jj = e >> 3, k = e & 7;
      if (j0 + jj < c8) {
        float a = 0.f, q = 0.f;
        for (int r = 0; r < rows; ++r) {
          a += red[r * tpr + jj][k];
          q += red[r * tpr + jj][8 + k];
        }
        csum[0][(j0 + jj) * 8 + k] = a;
        csum[1][(j0 + jj) * 8 + k] = q;
      }
    }
    __syncthreads();
  }
  const int cg = C / G;
  for (int g = t; g < G; g += 256) {
    float a = 0.f, q = 0.f;
    for (int c = g * cg; c < (g + 1) * cg; ++c) {
      a += csum[0][c];
      q += csum[1][c];
    }
    part[(static_cast<long long>(b) * nblk + blk) * G + g] = make_float2(a, q);
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const unsigned prev = atomicAdd(&arrived[b], 1u);
    is_last = prev == static_cast<unsigned>(nblk - 1);
    if (is_last) arrived[b] = 0u;  // every block of this image has counted
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Eight threads per group, each over every eighth block's partial, then a
  // fixed shuffle tree: the same order every run.
  const double n = static_cast<double>(hw) * cg;
  const int sub = t & 7;
  for (int g0 = 0; g0 < G; g0 += 32) {
    const int g = g0 + (t >> 3);
    double s1 = 0.0, s2 = 0.0;
    if (g < G) {
#pragma unroll 4
      for (int i = sub; i < nblk; i += 8) {
        const float2 v = __ldcg(part + (static_cast<long long>(b) * nblk + i) * G + g);
        s1 += v.x;
        s2 += v.y;
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (g < G && sub == 0) {
      const double mean = s1 / n;
      const double var = fmax(s2 / n - mean * mean, 0.0);
      stats[b * G + g] = make_float2(static_cast<float>(mean), static_cast<float>(1.0 / sqrt(var + eps)));
    }
  }
}

// y = (x - mean_g) * rstd_g * w_c + b_c (then SiLU), one block per (run of
// pixels, image), about four blocks per SM: each thread owns fixed 8-channel
// vectors, so the per-channel factors are formed once and the loop is loads
// (four in flight), 8 FMAs (and SiLU: an exponential and a fast reciprocal
// division) and stores, with no index division.
template <int f16>
__global__ void __launch_bounds__(256) gn_apply_kernel(const void* __restrict__ x, void* __restrict__ y,
                                                       int hw, int C, int G, int chunk,
                                                       const float2* __restrict__ stats,
                                                       const float* __restrict__ w,
                                                       const float* __restrict__ bias, int silu_after) {
  griddep_launch();
  griddep_wait();
  const int b = blockIdx.y;
  const int p0 = blockIdx.x * chunk, p1 = min(hw, p0 + chunk);
  const int c8 = C / 8;
  const int tpr = min(c8, 256);
  const int rows = 256 / tpr;
  const int t = threadIdx.x;
  const int pr = t / tpr;
  if (pr >= rows) return;
  const int cg = C / G;
  const long long base = static_cast<long long>(b) * hw * c8;
  for (int cv = t % tpr; cv < c8; cv += tpr) {
    float sc[8], sh[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = cv * 8 + k;
      const float2 st = stats[b * G + c / cg];
      const float wc = w ? __ldg(w + c) : 1.0f;
      sc[k] = st.y * wc;
      sh[k] = (bias ? __ldg(bias + c) : 0.0f) - st.x * st.y * wc;
    }
#pragma unroll 4
    for (int p = p0 + pr; p < p1; p += rows) {
      const long long i = base + static_cast<long long>(p) * c8 + cv;
      float v[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(x) + i), f16, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float o = fmaf(v[k], sc[k], sh[k]);
        if (silu_after) o = __fdividef(o, 1.0f + __expf(-o));
        v[k] = o;
      }
      reinterpret_cast<uint4*>(y)[i] = pack8(v, f16);
    }
  }
}

// GEGLU (UNetLayers.Geglu, Models/Sdxl/UNetLayers.cs:30-46): the projection's
// first half times the exact GELU of its second half.
__global__ void geglu_kernel(const void* __restrict__ in, void* __restrict__ out, int f16, long long rows,
                             int F) {
  griddep_launch();
  griddep_wait();
  const int f8 = F / 8;
  const long long n = rows * f8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / f8;
    const int c = static_cast<int>(i % f8);
    const uint4* row = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(in) + r * 2 * F);
    float h[8], g[8];
    unpack8(row[c], f16, h);
    unpack8(row[f8 + c], f16, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] *= gelu_erf(g[k]);
    reinterpret_cast<uint4*>(out)[i] = pack8(h, f16);
  }
}

__global__ void upsample2x_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, int B, int H, int W,
                                  int c8) {
  griddep_launch();
  griddep_wait();
  const long long n = static_cast<long long>(B) * 2 * H * 2 * W * c8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % c8);
    const long long pix = i / c8;
    const int xo = static_cast<int>(pix % (2 * W));
    const int yo = static_cast<int>((pix / (2 * W)) % (2 * H));
    const int b = static_cast<int>(pix / (4LL * H * W));
    out[i] = in[((static_cast<long long>(b) * H + yo / 2) * W + xo / 2) * c8 + c];
  }
}

__global__ void concat_kernel(const uint4* __restrict__ a, int ca8, const uint4* __restrict__ b, int cb8,
                              uint4* __restrict__ out, long long pixels) {
  griddep_launch();
  griddep_wait();
  const int c8 = ca8 + cb8;
  const long long n = pixels * c8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long p = i / c8;
    const int c = static_cast<int>(i % c8);
    out[i] = c < ca8 ? a[p * ca8 + c] : b[p * cb8 + (c - ca8)];
  }
}

// NCHW fp32 -> NHWC 16-bit with the channels zero-padded to cpad.
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ in, void* __restrict__ out, int f16, int B,
                                    int C, int HW, int cpad) {
  const long long n = static_cast<long long>(B) * HW * cpad;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cpad);
    const long long pix = i / cpad;
    const int p = static_cast<int>(pix % HW);
    const int b = static_cast<int>(pix / HW);
    const float v = c < C ? in[(static_cast<long long>(b) * C + c) * HW + p] : 0.f;
    if (f16) static_cast<__half*>(out)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  }
}

// NHWC fp32 [B, HW, C] -> NCHW fp32.
__global__ void nhwc_to_nchw_kernel(const float* __restrict__ in, float* __restrict__ out, int B, int C,
                                    int HW) {
  const long long n = static_cast<long long>(B) * C * HW;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(i % HW);
    const int c = static_cast<int>((i / HW) % C);
    const int b = static_cast<int>(i / (static_cast<long long>(HW) * C));
    out[i] = in[(static_cast<long long>(b) * HW + p) * C + c];
  }
}

__global__ void add_vec_kernel(float* __restrict__ dst, const float* __restrict__ a, const float* __restrict__ b,
                               long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    dst[i] = a[i] + b[i];
}

unsigned grid_for(long long n) {
  return static_cast<unsigned>(std::max<long long>(1, std::min<long long>((n + 255) / 256, sm_count() * 16LL)));
}

}  // namespace

int group_norm(const void* x, void* y, int dtype, int B, int HW, int C, int G, const float* w,
               const float* bias, float eps, int silu_after, void* scratch, size_t scratch_bytes,
               cudaStream_t s) {
  if (dtype != ND_F16 && dtype != ND_BF16) return fail(ND_ERR_INVALID, "group_norm: dtype must be f16 or bf16");
  if (B <= 0 || HW <= 0 || C <= 0 || G <= 0 || C % G || C % 8) return fail(ND_ERR_INVALID, "group_norm: bad shape");
  if (C > kGnMaxC) return fail(ND_ERR_UNSUPPORTED, "group_norm: more than 3072 channels");
  if (B > kGnCounterBytes / 4) return fail(ND_ERR_UNSUPPORTED, "group_norm: batch above 1024");
  if (!x || !y) return fail(ND_ERR_INVALID, "group_norm: null operand");
  if (scratch_bytes < group_norm_scratch(B, HW, C, G))
    return fail(ND_ERR_INVALID, "group_norm: scratch too small");
  const int rows = 256 / std::min(C / 8, 256);  // pixel rows a block covers per pass
  // Statistics: about two blocks per SM over all images, at least kGnChunk
  // pixels each (so the partials fit the scratch bound).
  const long long stat_blocks = std::max<long long>(1, 2LL * sm_count() / B);
  const long long sc = std::max<long long>(kGnChunk, (HW + stat_blocks - 1) / stat_blocks);
  const int chunk = static_cast<int>((sc + rows - 1) / rows * rows);
  const int nblk = (HW + chunk - 1) / chunk;
  // Scratch: the per-image arrival counters at a fixed place (zero before
  // the first call; the last block of each image resets its counter, so
  // calls of any shape find them zero), the partials and the statistics.
  const size_t part_bytes = static_cast<size_t>(B) * nblk * G * sizeof(float2);
  unsigned* arrived = static_cast<unsigned*>(scratch);
  float2* part = reinterpret_cast<float2*>(static_cast<uint8_t*>(scratch) + kGnCounterBytes);
  float2* stats = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(part) + ((part_bytes + 255) & ~size_t{255}));
  const int f16 = dtype == ND_F16;
  ND_CUDA(launch_pdl(f16 ? gn_stats_kernel<1> : gn_stats_kernel<0>, dim3(nblk, B), dim3(256), 0, s, x, HW, C, G,
                     chunk, part, arrived, eps, stats));
  // Normalization: about four blocks per SM.
  const long long apply_blocks = std::max<long long>(1, 4LL * sm_count() / B);
  const long long ac = (HW + apply_blocks - 1) / apply_blocks;
  const int achunk = static_cast<int>((ac + rows - 1) / rows * rows);
  ND_CUDA(launch_pdl(f16 ? gn_apply_kernel<1> : gn_apply_kernel<0>, dim3((HW + achunk - 1) / achunk, B), dim3(256), 0,
                     s, x, y, HW, C, G, achunk, stats, w, bias, silu_after));
  return ND_OK;
}

size_t group_norm_scratch(int B, int HW, int C, int G) {
  (void)C;
  const size_t nchunks = (static_cast<size_t>(HW) + kGnChunk - 1) / kGnChunk;
  const size_t part = static_cast<size_t>(B) * nchunks * G * sizeof(float2);
  return kGnCounterBytes + ((part + 255) & ~size_t{255}) + static_cast<size_t>(B) * G * sizeof(float2) + 256;
}

int geglu(const void* in, void* out, int dtype, int64_t rows, int64_t F, cudaStream_t s) {
  if (F % 8 || rows <= 0) return fail(ND_ERR_INVALID, "geglu: bad shape");
  ND_CUDA(launch_pdl(geglu_kernel, dim3(grid_for(rows * (F / 8))), dim3(256), 0, s, in, out, dtype == ND_F16 ? 1 : 0,
                     rows, static_cast<int>(F)));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int upsample2x(const void* in, void* out, int B, int H, int W, int C, cudaStream_t s) {
  if (C % 8) return fail(ND_ERR_INVALID, "upsample2x: channels must be a multiple of 8");
  const long long n = static_cast<long long>(B) * 4 * H * W * (C / 8);
  ND_CUDA(launch_pdl(upsample2x_kernel, dim3(grid_for(n)), dim3(256), 0, s, static_cast<const uint4*>(in),
                     static_cast<uint4*>(out), B, H, W, C / 8));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int concat_channels(const void* a, int ca, const void* b, int cb, void* out, int64_t pixels, cudaStream_t s) {
  if (ca % 8 || cb % 8) return fail(ND_ERR_INVALID, "concat: channels must be multiples of 8");
  concat_kernel<<<grid_for(pixels * ((ca + cb) / 8)), 256, 0, s>>>(static_cast<const uint4*>(a), ca / 8,
                                                                    static_cast<const uint4*>(b), cb / 8,
                                                                    static_cast<uint4*>(out), pixels);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int nchw_to_nhwc(const float* in, void* out, int dtype, int B, int C, int HW, int cpad, cudaStream_t s) {
  nchw_to_nhwc_kernel<<<grid_for(static_cast<long long>(B) * HW * cpad), 256, 0, s>>>(in, out, dtype == ND_F16, B, C,
                                                                                         HW, cpad);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int add_vectors(float* dst, const float* src, int64_t n, cudaStream_t s) {
  add_vec_kernel<<<grid_for(n), 256, 0, s>>>(dst, dst, src, n);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int add_vectors2(float* out, const float* a, const float* b, int64_t n, cudaStream_t s) {
  add_vec_kernel<<<grid_for(n), 256, 0, s>>>(out, a, b, n);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int nhwc_to_nchw(const float* in, float* out, int B, int C, int HW, cudaStream_t s) {
  nhwc_to_nchw_kernel<<<grid_for(static_cast<long long>(B) * HW * C), 256, 0, s>>>(in, out, B, C, HW);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd
