// int8 weight-only GEMM for sm_100a with the dequantization fused into the
// mainloop:  C[M, N] = A[M, K] . bf16(q[N, K] * s)^T
//
// Replaces the reference's int8 path, ModelBuilder.Weight -> DmlOps.Dequantize
// -> Gemm (Graph/ModelBuilder.cs:65-93, Dml/DmlOps.cs:208-228), where the
// dequantized copy of every weight is written to scratch per dispatch. Here
// the int8 tile goes HBM -> shared memory by TMA and is widened in shared
// memory right before the tensor core reads it; no bf16 copy of the weight
// ever exists in HBM. The weight scheme is BlockQuantizer's (symmetric, one
// scale per run of `group` columns; group 32 with fp16 scales is the
// reference's, group == K with fp32 scales is per output channel).
//
// Dequantized value: bf16(round-to-nearest-even(float(q) * float(s))). The
// product of an int8 and an fp16 (or the fp32 scale of a per-channel scheme
// whose mantissa product still fits) is formed exactly in fp32, so the
// widened weight is the oracle's dequantized weight rounded once.
//
// Warp roles (512 threads, one CTA per SM, persistent over tiles):
//   warp 0       TMA: A tile [128 x 64] bf16 + raw W tile [BN x 64] int8
//   warp 1       tcgen05.mma issuer (as in gemm_sm100_kernel)
//   warps 4-11   converters (two per SM sub-partition): raw int8 -> bf16 *
//                scale into the 128B-swizzled K-major operand layout, then
//                release the stage to the MMA. A thread converts 16-byte
//                pieces (16 weights), so its shared-memory reads and writes
//                are free of bank conflicts; per-channel scales are loaded
//                once per tile, group scales once per k block.
//   warps 12-15  epilogue (shared with gemm_sm100_kernel)
// Registers are rebalanced per warpgroup with setmaxnreg: 56 / 104 / 104 /
// 200 per thread of warpgroups 0-3, summing to 59,392 of what the block is
// launched with (512 x its compiled count; the host checks it covers this).
#pragma once

#include "gemm_sm100.cuh"

namespace nd {

// Two rings: STAGES slots of (A tile + raw int8 W tile) fed by TMA, deep
// enough to cover the load latency, and kBStages slots of widened bf16 W
// tiles between the converters and the tensor core.
template <int BN, int STAGES>
struct GemmW8Smem {
  static constexpr int kABytes = 128 * 64 * 2;   // 16 KB
  static constexpr int kRawBytes = BN * 64;      // int8 tile
  static constexpr int kBBytes = BN * 64 * 2;    // widened bf16 tile
  static constexpr int kBStages = 2;
  static constexpr int kStageBytes = kABytes + kRawBytes;
  static constexpr int kBOffset = STAGES * kStageBytes;
  static constexpr int kTiles = kBOffset + kBStages * kBBytes;
  static constexpr int kStageBuf = 4096;
  static constexpr int kEpiOffset = kTiles;
  static constexpr int kBarOffset = kEpiOffset + 4 * 2 * kStageBuf;
  // full[S], empty[S], conv[BS], bempty[BS], acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * STAGES + 2 * kBStages + 5;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kTotal = kMiscOffset + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
  static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
  static constexpr int kConverters = 8;          // warps 4..11
};

constexpr int kW8Threads = 512;
constexpr int kW8RegsNeeded = 128 * (56 + 104 + 104 + 200);

// F16: fp16 activations (W widened to fp16), else bf16 (compile time, so
// each widened pair is packed one way only).
template <int BN, int STAGES, bool F16>
__global__ void __launch_bounds__(kW8Threads, 1)
    gemm_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmW,
                         const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using L = GemmW8Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kBarOffset;
  constexpr int BS = L::kBStages;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
  auto conv_bar = [&](int s) { return bars + 8u * (2 * STAGES + s); };
  auto bempty_bar = [&](int s) { return bars + 8u * (2 * STAGES + BS + s); };
  auto accf_bar = [&](int s) { return bars + 8u * (2 * STAGES + 2 * BS + s); };
  auto acce_bar = [&](int s) { return bars + 8u * (2 * STAGES + 2 * BS + 2 + s); };
  const uint32_t drain_bar = bars + 8u * (2 * STAGES + 2 * BS + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);
  auto a_buf = [&](int s) { return sbase + s * L::kStageBytes; };
  auto raw_buf = [&](int s) { return sbase + s * L::kStageBytes + L::kABytes; };
  auto b_buf = [&](int s) { return sbase + L::kBOffset + s * L::kBBytes; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (args.M + 127) / 128;
  const int num_n = (args.N + BN - 1) / BN;
  const int total = num_m * num_n;
  const int num_kb = (args.K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(conv_bar(s), L::kConverters);
      mbar_init(bempty_bar(s), 1);
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
    tma_prefetch_desc(&tmW);
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

  // Each role's code sits inside its warpgroup's setmaxnreg branch so the
  // compiler budgets each region with that branch's register count.
  if (warp < 4) {
    reg_dealloc<56>();
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
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), L::kABytes + L::kRawBytes);
          tma_load_2d(a_buf(stage), &tmA, full_bar(stage), kb * 64, m0);
          if (args.swiglu_half > 0) {
            // BN/2 gate rows, then the matching BN/2 up rows (boxes BN/2 high)
            tma_load_2d(raw_buf(stage), &tmW, full_bar(stage), kb * 64, nt * (BN / 2));
            tma_load_2d(raw_buf(stage) + (BN / 2) * 64, &tmW, full_bar(stage), kb * 64,
                        args.swiglu_half + nt * (BN / 2));
          } else {
            tma_load_2d(raw_buf(stage), &tmW, full_bar(stage), kb * 64, brow);
          }
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        volatile int never = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(full_bar(s), (issued_parity >> s) & 1u, &never, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int stage = 0, bstage = 0;
      uint32_t phase = 0, bphase = 0;
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
          // the widened tile is ready only after its A + raw slot landed
          if (!mbar_wait(conv_bar(bstage), bphase, abort_flag, args.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = make_sdesc_sw128(a_buf(stage) + k * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(b_buf(bstage) + k * 32, 16, 1024);
            umma_ss(d_tmem, ad, bd, args.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          umma_commit(bempty_bar(bstage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (++bstage == BS) {
            bstage = 0;
            bphase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(accf_bar(acc));
      }
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, args.status, kStatusTimeoutDrain);
    }
  }
  } else if (warp < 12) {
    reg_dealloc<104>();
    // ------------------------------------------------------------ converters
    // Unit u = (row r of the W tile, quarter q of the 64-column k block): 16
    // int8 at raw[r * 64 + q * 16] -> 16 bf16, the 16-byte chunks 2q and
    // 2q + 1 of operand row r, chunk c stored at c ^ (r & 7) (128B swizzle).
    // A warp's 32 units are 8 rows x 4 quarters: 512 contiguous bytes read,
    // 4 x 128 bytes written per store, no bank conflicts either way.
    constexpr int kUnits = BN * 4;
    constexpr int kPer = kUnits / (L::kConverters * 32);  // units per thread (4 or 2)
    static_assert(kUnits % (L::kConverters * 32) == 0, "tile rows must fill the converters");
    const int ct = threadIdx.x - 128;  // 0 .. 255
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    bool ok = true;
    const bool f16_scales = args.w8_scale_f16 != 0;
    const bool per_channel = args.w8_scale_cols == 1;
    const long long w_rows = (args.shared_weights || args.group_split >= args.M ? 1LL : 2LL) * args.N;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const int m0 = mt * 128;
      const int n0 = nt * BN;
      const int group = row_group(args, m0);
      const long long wrow0 = (args.shared_weights ? 0LL : static_cast<long long>(group) * args.N) + n0;
      // W row of tile row r (SwiGLU: gate rows, then the matching up rows)
      auto wrow_of = [&](int r) -> long long {
        if (args.swiglu_half > 0)
          return (r < BN / 2 ? 0LL : static_cast<long long>(args.swiglu_half) - BN / 2) +
                 static_cast<long long>(nt) * (BN / 2) + r;
        return wrow0 + r;
      };
      auto load_scale = [&](long long wrow, int kcol) {
        if (wrow >= w_rows || kcol >= args.K) return 0.f;
        const long long si = wrow * args.w8_scale_cols + (per_channel ? 0 : kcol / args.w8_group);
        return f16_scales ? __half2float(__ldg(static_cast<const __half*>(args.w8_scales) + si))
                          : __ldg(static_cast<const float*>(args.w8_scales) + si);
      };
      float sc[kPer];
      if (per_channel) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) sc[j] = load_scale(wrow_of((ct + j * 256) >> 2), 0);
      }
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!per_channel) {
#pragma unroll
          for (int j = 0; j < kPer; ++j) {
            const int u = ct + j * 256;
            sc[j] = load_scale(wrow_of(u >> 2), kb * 64 + (u & 3) * 16);
          }
        }
        if (!mbar_wait(full_bar(stage), phase, abort_flag, args.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        // the widened slot must have been read by the MMAs of two k blocks ago
        if (!mbar_wait(bempty_bar(bstage), bphase ^ 1u, abort_flag, args.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        uint4 raw[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int u = ct + j * 256;
          ld_shared_v4(raw_buf(stage) + (u >> 2) * 64 + (u & 3) * 16, raw[j].x, raw[j].y, raw[j].z, raw[j].w);
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int u = ct + j * 256;
          const int r = u >> 2, q = u & 3;
          const uint32_t w4[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
          const float2 s2 = make_float2(sc[j], sc[j]);
          const float2 m2 = make_float2(-8388736.0f, -8388736.0f);
          uint32_t p[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            // exact int8 -> fp32 (magic 2^23 + 128 offset), fp32 product, one RNE rounding
            const uint32_t x = w4[i] ^ 0x80808080u;
            const float2 lo = fadd2(make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u)),
                                                __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7541u))), m2);
            const float2 hi = fadd2(make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7542u)),
                                                __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7543u))), m2);
            const float2 a = fmul2(lo, s2), b = fmul2(hi, s2);
            p[2 * i] = F16 ? pack_f16(a.x, a.y) : pack_bf16(a.x, a.y);
            p[2 * i + 1] = F16 ? pack_f16(b.x, b.y) : pack_bf16(b.x, b.y);
          }
          const uint32_t dst = b_buf(bstage) + r * 128;
          st_shared_v4(dst + (((2 * q) ^ (r & 7)) << 4), p[0], p[1], p[2], p[3]);
          st_shared_v4(dst + (((2 * q + 1) ^ (r & 7)) << 4), p[4], p[5], p[6], p[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(conv_bar(bstage));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        if (++bstage == BS) {
          bstage = 0;
          bphase ^= 1u;
        }
      }
    }
  } else {
    reg_alloc<200>();
    // ------------------------------------------------------------ epilogue
    const int ew = warp & 3;
    const int row_in_tile = ew * 32 + lane;
    const uint32_t buf0 = sbase + L::kEpiOffset + (ew * 2) * L::kStageBuf;
    int sb = 0;
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(accf_bar(acc), acc_phase, abort_flag, args.status, kStatusTimeoutEpilogue)) break;
      __syncwarp();
      tc_fence_after();
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const int m0 = mt * 128;
      const int n0 = nt * BN;
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
            epilogue_head_norm_rope(args, &tmC, group, row0, row, col0, tbase + h * 128, row_ok, buf0, sb, lane);
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
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, L::kTmemCols);
}

// Standalone dequantization, the same arithmetic as the converters:
// w[n, k] = bf16/f16(float(q[n, k]) * scale(n, k)). For the bit-exact check
// against the oracle and for callers that want the widened weight.
__global__ void dequant_w8_kernel(const int8_t* __restrict__ q, const void* __restrict__ scales,
                                  int scale_f16, int group, int scale_cols, long long rows, int cols,
                                  void* __restrict__ out, int out_f16) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols;
    const int c = static_cast<int>(i % cols);
    const long long si = r * scale_cols + c / group;
    const float s = scale_f16 ? __half2float(static_cast<const __half*>(scales)[si])
                              : static_cast<const float*>(scales)[si];
    float f[4];
    const uint32_t packed = static_cast<uint32_t>(static_cast<uint8_t>(q[i]));
    i8x4_to_f32(packed, f);  // byte 0 is q[i]; the zero bytes above it are unused
    const float v = f[0] * s;
    if (out_f16) static_cast<__half*>(out)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  }
}

}  // namespace nd
