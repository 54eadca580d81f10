// Two-SM (cta_group::2) variant of the int8 weight-only GEMM:
//   C[M, N] = A[M, K] . bf16(q[N, K] * s)^T   in 256 x BN tiles per CTA pair.
//
// As in gemm2_sm100.cuh, CTA r of a cluster pair loads A rows [m0 + 128 r,
// +128) and W rows [n0 + BN/2 r, +BN/2); here the W rows arrive as int8 and
// each CTA's converter warps widen only its own half of the tile. The
// widening (int8 -> fp32 -> x scale -> one RNE rounding to bf16 / fp16, the
// same arithmetic as gemm_w8_sm100_kernel and the oracle's dequantization)
// and its shared-memory traffic per SM halve against the one-SM kernel,
// which is what bounds that kernel.
//
// Barriers: each CTA's producer loads (plain TMA) into its own ring and
// completes its own full[s]; each CTA's converters wait on their own full[s],
// widen, and arrive on the LEADER's conv[bs] (16 arrivals: eight converter
// warps per CTA, the peer's through its shared::cluster address), so the
// leader's MMAs start on a k block only when both halves of the W tile are
// widened and (behind them) both A tiles landed. The arrivals carry the
// default CTA-scope release: with a cluster-scope release every converter
// warp stalled on the implied memory barrier (measured 600 TFLOP/s, membar
// the top stall, against 1116 at the qkv shape now). The leader's commits
// multicast to both CTAs' empty[s] / bempty[bs] / acc_full; both CTAs'
// epilogues arrive on the leader's acc_empty (8).
#pragma once

#include "gemm2_sm100.cuh"
#include "gemm_w8_sm100.cuh"

namespace nd {

template <int BN, int STAGES, int BSTAGES>
struct Gemm2W8Smem {
  static constexpr int kHalf = BN / 2;            // W rows per CTA
  static constexpr int kABytes = 128 * 64 * 2;    // 16 KB
  static constexpr int kRawBytes = kHalf * 64;    // int8 half tile
  static constexpr int kBBytes = kHalf * 64 * 2;  // widened half tile
  static constexpr int kBStages = BSTAGES;       // widened slots: the pair's signalling crosses SMs
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
  static constexpr int kConverters = 8;           // warps 4..11 of each CTA
};

// F16: fp16 activations (W widened to fp16), else bf16; a compile-time
// choice, so each widened pair is packed one way only.
template <int BN, int STAGES, int BSTAGES, bool F16>
__global__ void __launch_bounds__(kW8Threads, 1)
    gemm2_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmW,
                          const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using L = Gemm2W8Smem<BN, STAGES, BSTAGES>;
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
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int num_m2 = (args.M + 255) / 256;
  const int num_n = (args.N + BN - 1) / BN;
  const int total = num_m2 * num_n;
  const int num_kb = (args.K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(conv_bar(s), 2 * L::kConverters);
      mbar_init(bempty_bar(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(accf_bar(s), 1);
      mbar_init(acce_bar(s), 8);
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
    tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch();
  griddep_wait();

  // This CTA's first W row of pair tile (mt2, nt): its half of the tile's
  // rows, or (SwiGLU) the gate rows in the leader and the up rows in the peer.
  auto half_row0 = [&](int pm0, int nt) -> long long {
    if (args.swiglu_half > 0)
      return (rank ? static_cast<long long>(args.swiglu_half) : 0LL) + static_cast<long long>(nt) * L::kHalf;
    const int group = row_group(args, pm0);
    return (args.shared_weights ? 0LL : static_cast<long long>(group) * args.N) + static_cast<long long>(nt) * BN +
           static_cast<long long>(rank) * L::kHalf;
  };

  if (warp < 4) {
    reg_dealloc<56>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += pairs) {
        int mt2, nt;
        pair_tile_coords(t, num_m2, num_n, mt2, nt);
        const int pm0 = mt2 * 256;
        const int m0 = pm0 + static_cast<int>(rank) * 128;
        const int wrow = static_cast<int>(half_row0(pm0, nt));
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), L::kStageBytes);
          tma_load_2d(a_buf(stage), &tmA, full_bar(stage), kb * 64, m0);
          tma_load_2d(raw_buf(stage), &tmW, full_bar(stage), kb * 64, wrow);
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
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && elect_one()) {
      int stage = 0, bstage = 0;
      uint32_t phase = 0, bphase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, abort_flag, args.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(conv_bar(bstage), bphase, abort_flag, args.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = make_sdesc_sw128(a_buf(stage) + k * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(b_buf(bstage) + k * 32, 16, 1024);
            umma_ss_pair(d_tmem, ad, bd, args.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(empty_bar(stage), 0x3);
          umma_commit_pair(bempty_bar(bstage), 0x3);
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
        umma_commit_pair(accf_bar(acc), 0x3);
      }
      umma_commit_pair(drain_bar, 0x1);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, args.status, kStatusTimeoutDrain);
    }
  }
  } else if (warp < 12) {
    reg_dealloc<104>();
    // ------------------------------------------------------------ converters (both CTAs)
    // Unit u = (row r of this CTA's half tile, quarter q of the 64-column k
    // block), as in gemm_w8_sm100_kernel: 16 int8 -> 16-byte chunks 2q and
    // 2q + 1 of operand row r, chunk c stored at c ^ (r & 7).
    constexpr int kUnits = L::kHalf * 4;
    constexpr int kPer = kUnits / (L::kConverters * 32);
    static_assert(kUnits % (L::kConverters * 32) == 0, "half-tile rows must fill the converters");
    const int ct = threadIdx.x - 128;
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    bool ok = true;
    const bool f16_scales = args.w8_scale_f16 != 0;
    const bool per_channel = args.w8_scale_cols == 1;
    const long long w_rows = (args.shared_weights || args.group_split >= args.M ? 1LL : 2LL) * args.N;
    for (int t = pair; t < total && ok; t += pairs) {
      int mt2, nt;
      pair_tile_coords(t, num_m2, num_n, mt2, nt);
      const long long wrow0 = half_row0(mt2 * 256, nt);
      auto load_scale = [&](long long wrow, int kcol) {
        if (wrow >= w_rows || kcol >= args.K) return 0.f;
        const long long si = wrow * args.w8_scale_cols + (per_channel ? 0 : kcol / args.w8_group);
        return f16_scales ? __half2float(__ldg(static_cast<const __half*>(args.w8_scales) + si))
                          : __ldg(static_cast<const float*>(args.w8_scales) + si);
      };
      float sc[kPer];
      if (per_channel) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) sc[j] = load_scale(wrow0 + ((ct + j * 256) >> 2), 0);
      }
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!per_channel) {
#pragma unroll
          for (int j = 0; j < kPer; ++j) {
            const int u = ct + j * 256;
            sc[j] = load_scale(wrow0 + (u >> 2), kb * 64 + (u & 3) * 16);
          }
        }
        if (!mbar_wait(full_bar(stage), phase, abort_flag, args.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
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
        if (lane == 0) mbar_arrive_cluster(mapa_shared(conv_bar(bstage), 0));
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
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp & 3;
    const int row_in_tile = ew * 32 + lane;
    const uint32_t buf0 = sbase + L::kEpiOffset + (ew * 2) * L::kStageBuf;
    const uint32_t acce_leader0 = mapa_shared(acce_bar(0), 0), acce_leader1 = mapa_shared(acce_bar(1), 0);
    int sb = 0;
    int local = 0;
    for (int t = pair; t < total; t += pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(accf_bar(acc), acc_phase, abort_flag, args.status, kStatusTimeoutEpilogue)) break;
      __syncwarp();
      tc_fence_after();
      int mt2, nt;
      pair_tile_coords(t, num_m2, num_n, mt2, nt);
      const int m0 = mt2 * 256 + static_cast<int>(rank) * 128;
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
      if (lane == 0) mbar_arrive_cluster(acc ? acce_leader1 : acce_leader0);
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, L::kTmemCols);
}

}  // namespace nd
