// Persistent tcgen05 + TMA GEMM for sm_100a:  C[M, N] = A[M, K] . W[N, K]^T
//
// This replaces the reference's `Layers.Linear` (Graph/Layers.cs:131-160),
// which lowers to DirectML's GEMM with transB (Dml/DmlOps.cs:231-262): the
// weight is stored [out, in] as nn.Linear keeps it, so both operands are
// K-major and land in shared memory as 128-byte-swizzled tiles straight from
// TMA.
//
// Work split (one CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile [128 x 64] + W tile [BN x 64] per stage
//   warp 1      MMA issuer: tcgen05.mma 128 x BN x 16, accumulating in TMEM;
//               also allocates the 2 x BN TMEM columns (double buffer)
//   warps 2..5  epilogue: tcgen05.ld rows out of TMEM, apply the fused
//               epilogue and write to global memory, while the MMA warp
//               already fills the other accumulator buffer.
//
// Row groups: a dual-stream block (image rows then text rows) runs both
// streams' projections in one launch. Rows >= group_split take weight rows
// [N, 2N) and the second group's epilogue vectors. The split is a multiple of
// the 128-row tile.
#pragma once

#include "nd_common.cuh"

namespace nd {

enum GemmEpilogue : int {
  kEpiStore = 0,          // out = acc + bias                       (bf16/f16)
  kEpiGeluTanh = 1,       // out = gelu_tanh(acc + bias)
  kEpiGeluErf = 2,        // out = gelu(acc + bias), exact erf form
  kEpiSilu = 3,           // out = silu(acc + bias)
  kEpiResidualGate = 4,   // resid(f32) += gate[c] * (acc + bias)
  kEpiStoreF32 = 5,       // outf(f32) = acc + bias
  kEpiQkNormRope = 6,     // columns < qk_cols: per-head RMSNorm * w, then RoPE
  kEpiResidualAdd = 7,    // resid(f32) += acc + bias
  kEpiAddStore = 8,       // out = acc + bias + addend[row, col]     (bf16/f16)
  kEpiSwiGlu = 9,         // out[:, j] = silu(gate_j) * up_j  (W = [gate rows; up rows])
  kEpiGeGlu = 10,         // out[:, j] = h_j * gelu(g_j)      (W = [h rows; g rows])
};

struct GemmArgs {
  int M, N, K;
  int group_split;  // first row of the second weight group (>= M: one group)
  int epi;
  int out_f16;      // 0: bf16 output, 1: fp16 output
  void* out;        // bf16/f16 output, leading dimension ldo (elements)
  long long ldo;
  float* resid;     // fp32 residual / fp32 output, leading dimension ldr
  long long ldr;
  const float* bias;  // [groups][bias_stride] or null
  int bias_stride;
  const float* gate;  // [groups][gate_stride] (kEpiResidualGate)
  int gate_stride;
  const float* qk_norm;   // [groups][2][head_dim]: q weight then k weight
  const float* rope_cos;  // [M][head_dim / 2]
  const float* rope_sin;
  int qk_cols;            // leading columns that get the head norm
  int norm_span;          // columns per norm weight set (qk_norm[group][col / norm_span])
  int norm_sets;          // weight sets per group
  int rope_period;        // RoPE table row = row % rope_period (rope_cos null: no rotation)
  int head_dim;           // 128
  float norm_eps;
  uint32_t idesc;
  unsigned* status;
  // int8 weight-only (gemm_w8_sm100_kernel): scale of weight (n, k) is
  // w8_scales[n * w8_scale_cols + k / w8_group] (fp16 or fp32).
  const void* w8_scales;
  int w8_group;
  int w8_scale_cols;
  int w8_scale_f16;
  // kEpiAddStore: the tensor added to the result, like out (ld_add elements)
  const void* addend;
  long long ld_add;
  // groups of rows: periodic (group = row / group_split: one per batch item)
  // and weights shared by every group (only bias / gate differ)
  int periodic_groups;
  int shared_weights;
  // implicit-GEMM conv3x3 (pad 1): A rows are output pixels, K = 9 taps x Cin
  int conv_kpc;      // Cin / 64 channel chunks per tap
  int conv_hw;       // H_out * W_out pixels per image
  int conv_w_out;
  int conv_stride;
  // fp32 compute on bf16 hi|lo pairs (ND_BF16X2): A is [M, 2K'] and W is
  // [N, 2K'] with K' = split_kb * 64; the K loop runs three segments,
  // hi.lo + lo.hi + hi.hi, reading the lo halves split_koff columns along.
  int split_kb;     // 0: plain operands
  int split_koff;
  int out_kind;     // 0: bf16/f16 out, 1: hi|lo pair out (lo at column + N), 2: fp32 out
  // kEpiSwiGlu: W is [gate rows; up rows] with the up rows starting at row
  // swiglu_half (= the output width F; N = 2F). Tile nt loads gate rows
  // [nt*BN/2, +BN/2) into the first half of its B tile and the matching up
  // rows into the second, so the epilogue finds both operands of output
  // column j in one accumulator.
  int swiglu_half;
  // Bias / gate group chosen per row (rows >= group_split take the second
  // vectors) with one weight matrix for every row: a single-stream block
  // whose image and text rows differ only in their modulation.
  int row_groups;
};

// Tile order of the persistent loop: bands of kTileBandM row tiles, each
// band walked column tile by column tile. The ~148 tiles in flight at once
// then share a few A row panels and W column panels, which stay in L2,
// instead of every CTA streaming its own panels from HBM.
constexpr int kTileBandM = 16;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mt, int& nt) {
  const int per_band = kTileBandM * num_n;
  const int band = t / per_band;
  const int first = band * kTileBandM;
  const int rows = min(kTileBandM, num_m - first);
  const int r = t - band * per_band;
  mt = first + r % rows;
  nt = r / rows;
}

__device__ __forceinline__ int row_group(const GemmArgs& a, int m0) {
  if (a.periodic_groups) return m0 / a.group_split;
  return m0 >= a.group_split ? 1 : 0;
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kBM = 128;
  static constexpr int kBK = 64;
  static constexpr int kABytes = kBM * kBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTiles = STAGES * kStageBytes;
  // Epilogue staging: 4 warps x 2 buffers x [32 rows x 128 B] for TMA stores.
  static constexpr int kStageBuf = 4096;
  static constexpr int kEpiOffset = kTiles;
  static constexpr int kBarOffset = kEpiOffset + 4 * 2 * kStageBuf;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kTotal = kMiscOffset + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;  // + alignment slack
  // TMEM: two accumulators of BN fp32 columns, allocated as a power of two.
  static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
};

enum EmitKind : int { kEmitBf16 = 0, kEmitF16 = 1, kEmitF32 = 2, kEmitAddF32 = 3, kEmitSplit = 4 };

// The store kind of a 16-bit-class output under the args' out_kind.
__device__ __forceinline__ int out_emit_kind(const GemmArgs& a) {
  if (a.out_kind == 1) return kEmitSplit;
  if (a.out_kind == 2) return kEmitF32;
  return a.out_f16 ? kEmitF16 : kEmitBf16;
}

__device__ __forceinline__ void load_vec32(const float* src, int col, int N, float (&v)[32]) {
  if (src == nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    return;
  }
  if (col + 32 <= N) {
    const float4* s = reinterpret_cast<const float4*>(src + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 t = __ldg(s + i);
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (col + i < N) ? __ldg(src + col + i) : 0.f;
  }
}

// Stage one warp's [32 rows x 32 columns] chunk (lane = row) in shared memory
// in the tensor map's swizzled layout and hand it to TMA: a store (bf16, fp16,
// fp32, or a bf16 hi|lo pair whose lo chunk goes to column col + lo_off) or
// an fp32 reduce-add into global memory. Rows / columns past the tensor's
// edge are clipped by TMA. Two staging buffers per warp alternate; a buffer is
// rewritten only after the store issued from it two chunks ago has finished
// reading it.
__device__ __forceinline__ void emit_chunk(const CUtensorMap* tm, int kind, uint32_t buf0, int& sb,
                                           int lane, int row0, int rows, int col,
                                           const float (&v)[32], int lo_off = 0) {
  if (row0 >= rows) return;  // the whole warp's rows are past the tensor's edge
  const uint32_t buf = buf0 + static_cast<uint32_t>(sb) * 4096u;
  sb ^= 1;
  if (lane == 0) bulk_wait_read<1>();
  __syncwarp();
  if (kind == kEmitSplit) {
    uint32_t h[16], l[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pack_split(v[2 * i], v[2 * i + 1], h[i], l[i]);
    // hi rows in the first 2 KB, lo rows in the second, each 64B-swizzled.
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t off = lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4);
      st_shared_v4(buf + off, h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
      st_shared_v4(buf + 2048 + off, l[4 * c], l[4 * c + 1], l[4 * c + 2], l[4 * c + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm, buf, col, row0);
      tma_store_2d(tm, buf + 2048, col + lo_off, row0);
      bulk_commit();
    }
    return;
  }
  if (kind == kEmitBf16 || kind == kEmitF16) {
    uint32_t p[16];
    if (kind == kEmitF16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = pack_f16(v[2 * i], v[2 * i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
    }
    // 64-byte rows, 64B swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3).
#pragma unroll
    for (int c = 0; c < 4; ++c)
      st_shared_v4(buf + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4), p[4 * c], p[4 * c + 1],
                   p[4 * c + 2], p[4 * c + 3]);
  } else {
    // 128-byte rows, 128B swizzle: 16-byte chunk c of row r at c ^ (r & 7).
#pragma unroll
    for (int c = 0; c < 8; ++c)
      st_shared_v4(buf + lane * 128 + ((c ^ (lane & 7)) << 4), __float_as_uint(v[4 * c]),
                   __float_as_uint(v[4 * c + 1]), __float_as_uint(v[4 * c + 2]),
                   __float_as_uint(v[4 * c + 3]));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (kind == kEmitAddF32) tma_reduce_add_2d(tm, buf, col, row0);
    else tma_store_2d(tm, buf, col, row0);
    bulk_commit();
  }
}

// One 32-column chunk of a plain epilogue (everything but kEpiQkNormRope).
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, const CUtensorMap* tmC, int group,
                                               int row0, int col, const uint32_t (&r)[32],
                                               uint32_t buf0, int& sb, int lane) {
  if (a.row_groups) group = (row0 + lane) >= a.group_split ? 1 : 0;
  float v[32];
  float b[32];
  load_vec32(a.bias ? a.bias + group * a.bias_stride : nullptr, col, a.N, b);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + b[i];
  int kind = out_emit_kind(a);
  switch (a.epi) {
    case kEpiGeluTanh:
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_fast(v[i]);
      break;
    case kEpiGeluErf:
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
      break;
    case kEpiSilu:
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = silu(v[i]);
      break;
    case kEpiResidualGate: {
      float g[32];
      load_vec32(a.gate + group * a.gate_stride, col, a.N, g);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= g[i];
      kind = kEmitAddF32;
      break;
    }
    case kEpiResidualAdd:
      kind = kEmitAddF32;
      break;
    case kEpiStoreF32:
      kind = kEmitF32;
      break;
    case kEpiAddStore: {
      const int row = row0 + lane;
      if (row < a.M) {
        const uint16_t* ad = static_cast<const uint16_t*>(a.addend) + static_cast<long long>(row) * a.ld_add + col;
        if (col + 32 <= a.N) {
          const uint4* a4 = reinterpret_cast<const uint4*>(ad);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 t = __ldg(a4 + i);
            const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float2 f = a.out_f16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[j]))
                                   : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
              v[8 * i + 2 * j] += f.x;
              v[8 * i + 2 * j + 1] += f.y;
            }
          }
        } else {
          for (int i = 0; i < 32 && col + i < a.N; ++i) {
            const uint16_t h = ad[i];
            v[i] += a.out_f16 ? __half2float(*reinterpret_cast<const __half*>(&h))
                              : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&h));
          }
        }
      }
      break;
    }
    default:
      break;
  }
  emit_chunk(tmC, kind, buf0, sb, lane, row0, a.M, col, v, a.N);
}

// SwiGLU / GEGLU over one tile: output columns [ocol0, ocol0 + half) from
// the first half's accumulator columns [0, half) and the second half's
// [half, 2 * half), biases at bias[j] and bias[F + j] -- QwenImageDit.
// FeedForward's Silu(gate) * up (Models/QwenImage/QwenImageDit.cs:386-403), or
// UNetLayers.Geglu's h * gelu(g) (Models/Sdxl/UNetLayers.cs:30-46), where the
// two products already sit.
template <int HALF>
__device__ __forceinline__ void epilogue_swiglu(const GemmArgs& a, const CUtensorMap* tmC, int group,
                                                int row0, int ocol0, uint32_t tbase, uint32_t buf0,
                                                int& sb, int lane) {
  const int F = a.swiglu_half;
  if (a.row_groups) group = (row0 + lane) >= a.group_split ? 1 : 0;
  const float* bias = a.bias ? a.bias + group * a.bias_stride : nullptr;
#pragma unroll 1
  for (int c = 0; c < HALF / 32; ++c) {
    const int ocol = ocol0 + c * 32;
    if (ocol >= F) break;
    uint32_t rg[32], ru[32];
    tmem_ld32(tbase + c * 32, rg);
    tmem_ld32(tbase + HALF + c * 32, ru);
    tmem_ld_wait();
    float bg[32], bu[32], v[32];
    load_vec32(bias, ocol, F, bg);
    load_vec32(bias ? bias + F : nullptr, ocol, F, bu);
    if (a.epi == kEpiGeGlu) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = (__uint_as_float(rg[i]) + bg[i]) * gelu_erf(__uint_as_float(ru[i]) + bu[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = silu(__uint_as_float(rg[i]) + bg[i]) * (__uint_as_float(ru[i]) + bu[i]);
    }
    emit_chunk(tmC, out_emit_kind(a), buf0, sb, lane, row0, a.M, ocol, v, F);
  }
}

// The Q/K projection epilogue for one 128-wide head: RMSNorm over the head's
// features with the stored per-feature weight, then the rotate-half RoPE with
// this row's angle tables -- Transformer.HeadNorm + Transformer.Rotate
// (Graph/Transformer.cs:37-64) fused where the accumulator already sits.
__device__ __forceinline__ void epilogue_head_norm_rope(const GemmArgs& a, const CUtensorMap* tmC,
                                                        int group, int row0, int row, int col0,
                                                        uint32_t tbase, bool row_ok, uint32_t buf0,
                                                        int& sb, int lane) {
  const float* bias = a.bias ? a.bias + group * a.bias_stride + col0 : nullptr;
  const int which = col0 / a.norm_span;
  const float* w = a.qk_norm + (group * a.norm_sets + which) * 128;
  const bool rope = a.rope_cos != nullptr;
  const int trow = row_ok ? (a.rope_period > 0 ? row % a.rope_period : row) : 0;
  const int kind = out_emit_kind(a);
  uint32_t r[32];
  float sumsq = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    tmem_ld32(tbase + c * 32, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float x = __uint_as_float(r[i]) + (bias ? __ldg(bias + c * 32 + i) : 0.f);
      sumsq = fmaf(x, x, sumsq);
    }
  }
  const float scale = rsqrtf(sumsq * (1.0f / 128.0f) + a.norm_eps);
  const float* cs = rope ? a.rope_cos + static_cast<long long>(trow) * 64 : nullptr;
  const float* sn = rope ? a.rope_sin + static_cast<long long>(trow) * 64 : nullptr;
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t lo[32], hi[32];
    tmem_ld32(tbase + c * 32, lo);
    tmem_ld32(tbase + 64 + c * 32, hi);
    tmem_ld_wait();
    float olo[32], ohi[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 co = (row_ok && rope) ? __ldg(reinterpret_cast<const float4*>(cs + c * 32 + i))
                                         : make_float4(1.f, 1.f, 1.f, 1.f);
      const float4 si = (row_ok && rope) ? __ldg(reinterpret_cast<const float4*>(sn + c * 32 + i))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
      const float cv[4] = {co.x, co.y, co.z, co.w};
      const float sv[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int f = c * 32 + i + u;
        const float l = (__uint_as_float(lo[i + u]) + (bias ? __ldg(bias + f) : 0.f)) * scale * __ldg(w + f);
        const float h = (__uint_as_float(hi[i + u]) + (bias ? __ldg(bias + 64 + f) : 0.f)) * scale *
                        __ldg(w + 64 + f);
        olo[i + u] = l * cv[u] - h * sv[u];
        ohi[i + u] = h * cv[u] + l * sv[u];
      }
    }
    emit_chunk(tmC, kind, buf0, sb, lane, row0, a.M, col0 + c * 32, olo, a.N);
    emit_chunk(tmC, kind, buf0, sb, lane, row0, a.M, col0 + 64 + c * 32, ohi, a.N);
  }
}

template <int BN, int STAGES, bool CONV = false>
__global__ void __launch_bounds__(192, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kBarOffset;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
  auto accf_bar = [&](int s) { return bars + 8u * (2 * STAGES + s); };
  auto acce_bar = [&](int s) { return bars + 8u * (2 * STAGES + 2 + s); };
  const uint32_t drain_bar = bars + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int num_m = (args.M + 127) / 128;
  const int num_n = (args.N + BN - 1) / BN;
  const int total = num_m * num_n;
  const int num_kb = args.split_kb > 0 ? 3 * args.split_kb : (args.K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(accf_bar(s), 1);
      mbar_init(acce_bar(s), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch();
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, num_m, num_n, mt, nt);
        const int m0 = mt * 128;
        const int n0 = nt * BN;
        const int group = row_group(args, m0);
        const int brow = (args.shared_weights ? 0 : group * args.N) + n0;
        // The tile's W rows: one box of BN rows, or (SwiGLU) BN/2 gate rows
        // and the BN/2 matching up rows, each box BN/2 rows high.
        auto load_b = [&](uint32_t dst, int kcol, uint32_t bar) {
          if (!CONV && args.swiglu_half > 0) {
            tma_load_2d(dst, &tmB, bar, kcol, nt * (BN / 2));
            tma_load_2d(dst + (BN / 2) * 128, &tmB, bar, kcol, args.swiglu_half + nt * (BN / 2));
          } else {
            tma_load_2d(dst, &tmB, bar, kcol, brow);
          }
        };
        int img = 0, y0 = 0, x0 = 0;
        if constexpr (CONV) {
          img = m0 / args.conv_hw;
          const int rem = m0 - img * args.conv_hw;
          y0 = rem / args.conv_w_out;
          x0 = rem - y0 * args.conv_w_out;  // 0 unless a row holds several tiles
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status,
                         kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = sbase + stage * L::kStageBytes;
          const uint32_t b_dst = a_dst + L::kABytes;
          mbar_arrive_expect_tx(full_bar(stage), L::kStageBytes);
          if constexpr (CONV) {
            // 128 output pixels x 64 input channels of tap (dy, dx): a 4-D box
            // (channels, x, y, image) of the NHWC input, borders zero-filled.
            const int tap = kb / args.conv_kpc;
            const int c0 = (kb - tap * args.conv_kpc) * 64;
            const int dy = tap / 3, dx = tap - dy * 3;
            tma_load_4d(a_dst, &tmA, full_bar(stage), c0, x0 * args.conv_stride + dx - 1,
                        y0 * args.conv_stride + dy - 1, img);
          } else if (args.split_kb > 0) {
            // segments 0, 1, 2 = (A hi, W lo), (A lo, W hi), (A hi, W hi): the
            // two small cross terms first, into a still-small accumulator (the
            // tensor cores' fp32 accumulation loses bits relative to the
            // accumulator's magnitude at every step, so the small terms are
            // summed before the large one arrives).
            const int seg = kb / args.split_kb;
            const int kc = (kb - seg * args.split_kb) * 64;
            tma_load_2d(a_dst, &tmA, full_bar(stage), kc + (seg == 1 ? args.split_koff : 0), m0);
            load_b(b_dst, kc + (seg == 0 ? args.split_koff : 0), full_bar(stage));
          } else {
            tma_load_2d(a_dst, &tmA, full_bar(stage), kb * 64, m0);
          }
          if (CONV || args.split_kb == 0) load_b(b_dst, kb * 64, full_bar(stage));
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Aborted: let every load this thread started land before the CTA
        // (and its shared memory) goes away.
        volatile int never = 0;
        for (int s = 0; s < STAGES; ++s) {
          if (issued & (1u << s)) {
            mbar_wait(full_bar(s), (issued_parity >> s) & 1u, &never, nullptr, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, abort_flag, args.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, args.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + stage * L::kStageBytes;
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = make_sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_ss(d_tmem, ad, bd, args.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(accf_bar(acc));
      }
      // Wait until every MMA this thread issued has retired before TMEM is
      // released (bounded, and independent of the abort flag).
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, args.status, kStatusTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp & 3;  // TMEM lane quarter this warp may read
    const int row_in_tile = ew * 32 + lane;
    const uint32_t buf0 = sbase + L::kEpiOffset + (ew * 2) * L::kStageBuf;  // + sb * 4 KB
    int sb = 0;
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(accf_bar(acc), acc_phase, abort_flag, args.status, kStatusTimeoutEpilogue)) {
        break;
      }
      __syncwarp();
      tc_fence_after();
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const int m0 = mt * 128;
      const int n0 = nt * BN;
      // row_groups: the plain and SwiGLU epilogues pick the vectors per row;
      // the head norm uses the one shared set.
      const int group = args.row_groups ? 0 : row_group(args, m0);
      const int row0 = m0 + ew * 32;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + acc * BN;

      if (args.epi == kEpiSwiGlu || args.epi == kEpiGeGlu) {
        epilogue_swiglu<BN / 2>(args, &tmC, group, row0, nt * (BN / 2), tbase, buf0, sb, lane);
      } else if (args.epi == kEpiQkNormRope) {
#pragma unroll 1
        for (int h = 0; h < BN / 128; ++h) {
          const int col0 = n0 + h * 128;
          if (col0 >= args.N) break;
          if (col0 < args.qk_cols) {
            epilogue_head_norm_rope(args, &tmC, group, row0, row, col0, tbase + h * 128, row_ok,
                                    buf0, sb, lane);
          } else {
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              tmem_ld32(tbase + h * 128 + c * 32, r);
              tmem_ld_wait();
              GemmArgs plain = args;
              plain.epi = kEpiStore;
              epilogue_chunk(plain, &tmC, group, row0, col0 + c * 32, r, buf0, sb, lane);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col = n0 + c * 32;
          if (col >= args.N) break;
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
          epilogue_chunk(args, &tmC, group, row0, col, r, buf0, sb, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(acc));
    }
    // Every store this warp handed to TMA must finish before the CTA exits.
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, L::kTmemCols);
}

}  // namespace nd
