// Two-SM (cta_group::2) variant of the persistent tcgen05 GEMM:
//   C[M, N] = A[M, K] . W[N, K]^T   in 256 x BN tiles, one tile per CTA pair.
//
// A cluster of two CTAs on two SMs shares each tile: CTA r (r = its rank in
// the cluster) loads A rows [m0 + 128 r, +128) and W rows [n0 + BN/2 r,
// +BN/2) of every 64-deep k block into its own shared memory; the even CTA
// (the leader) issues tcgen05.mma.cta_group::2 with M = 256, N = BN, which
// reads A from each CTA's shared memory for that CTA's half of the rows and
// the two W halves from both, and accumulates rows [128 r, +128) of the tile
// into CTA r's tensor memory. Per SM, every k block then moves 16 KB of A and
// BN/2 x 128 B of W instead of BN x 128 B: each W tile serves 256 rows, so
// the W traffic from L2 (and from HBM, for the panels L2 cannot keep) halves.
//
// Synchronisation across the pair (no TMA multicast: every load fills only
// the issuing CTA's shared memory):
//   full[s]     in the leader only: its producer arms it with the bytes of
//               both CTAs' loads; both CTAs' loads complete on it (the
//               cta_group::2 form of the TMA load may signal the peer's barrier)
//   empty[s]    in both CTAs: the leader's tcgen05.commit multicasts to both
//   acc_full    in both CTAs: multicast commit after a tile's last k block
//   acc_empty   in the leader: the four epilogue warps of BOTH CTAs arrive
//               (the peer's remotely), so the leader reuses an accumulator
//               only after both halves of it were read
// TMEM is allocated and freed by warp 1 of both CTAs (cta_group::2 alloc /
// dealloc are collective over the pair). Every wait is bounded as in the
// one-SM kernel, and every role of both CTAs ends its loop on a timeout, so
// both CTAs always reach the closing cluster barrier.
#pragma once

#include "gemm_sm100.cuh"

namespace nd {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of `addr` (a shared::cta address of this CTA's
// layout) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier anywhere in the cluster (a shared::cluster address),
// with the default release semantics at CTA scope: a cluster-scope release
// is a memory barrier the arriving warp stalls on.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// TMA loads into this CTA's shared memory whose completion is counted on a
// barrier of either CTA of the pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* desc, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const void* desc, uint32_t bar, int c0, int c1,
                                                 int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[smem of both] . B[smem of both]^T, M = 256.
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the barrier at shared::cta offset `bar` in every CTA of
// `mask` when this thread's earlier pair MMAs have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

template <int BN, int STAGES>
struct Gemm2Smem {
  static constexpr int kABytes = 128 * 64 * 2;        // this CTA's 128 A rows x 64 k
  static constexpr int kBBytes = (BN / 2) * 64 * 2;   // this CTA's half of the W tile
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTiles = STAGES * kStageBytes;
  static constexpr int kStageBuf = 4096;
  static constexpr int kEpiOffset = kTiles;
  static constexpr int kBarOffset = kEpiOffset + 4 * 2 * kStageBuf;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kTotal = kMiscOffset + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
  static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
};

// Pair tile order: bands of kTileBandM / 2 pair rows (the same 16 rows of
// 128 as the one-SM kernel's bands), walked column tile by column tile.
__device__ __forceinline__ void pair_tile_coords(int t, int num_m2, int num_n, int& mt2, int& nt) {
  constexpr int band_m = kTileBandM / 2;
  const int per_band = band_m * num_n;
  const int band = t / per_band;
  const int first = band * band_m;
  const int rows = min(band_m, num_m2 - first);
  const int r = t - band * per_band;
  mt2 = first + r % rows;
  nt = r / rows;
}

template <int BN, int STAGES, bool CONV = false>
__global__ void __launch_bounds__(192, 1)
    gemm2_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using L = Gemm2Smem<BN, STAGES>;
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
  const uint32_t rank = cluster_ctarank();  // 0: leader, 1: peer
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  const int num_m2 = (args.M + 255) / 256;
  const int num_n = (args.N + BN - 1) / BN;
  const int total = num_m2 * num_n;
  const int num_kb = args.split_kb > 0 ? 3 * args.split_kb : (args.K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(accf_bar(s), 1);
      mbar_init(acce_bar(s), 8);  // four epilogue warps in each CTA of the pair
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
    tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers are initialised and the TMEM address is written
  // before any thread of the pair uses them.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch();
  griddep_wait();

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
        const int n0 = nt * BN;
        const int group = row_group(args, pm0);  // the host keeps a pair inside one group
        // This CTA's W rows: the rank's half of the tile, or (SwiGLU) the
        // gate rows in the leader and the matching up rows in the peer.
        int brow;
        if (!CONV && args.swiglu_half > 0) {
          brow = (rank ? args.swiglu_half : 0) + nt * (BN / 2);
        } else {
          brow = (args.shared_weights ? 0 : group * args.N) + n0 + static_cast<int>(rank) * (BN / 2);
        }
        int img = 0, y0 = 0, x0 = 0;
        if constexpr (CONV) {
          img = m0 / args.conv_hw;
          const int rem = m0 - img * args.conv_hw;
          y0 = rem / args.conv_w_out;
          x0 = rem - y0 * args.conv_w_out;
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = sbase + stage * L::kStageBytes;
          const uint32_t b_dst = a_dst + L::kABytes;
          const uint32_t fbar = mapa_shared(full_bar(stage), 0);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * L::kStageBytes);
          int akc = kb * 64, bkc = kb * 64;
          if (!CONV && args.split_kb > 0) {
            const int seg = kb / args.split_kb;
            const int kc = (kb - seg * args.split_kb) * 64;
            akc = kc + (seg == 1 ? args.split_koff : 0);
            bkc = kc + (seg == 0 ? args.split_koff : 0);
          }
          if constexpr (CONV) {
            const int tap = kb / args.conv_kpc;
            const int c0 = (kb - tap * args.conv_kpc) * 64;
            const int dy = tap / 3, dx = tap - dy * 3;
            tma_load_4d_pair(a_dst, &tmA, fbar, c0, x0 * args.conv_stride + dx - 1, y0 * args.conv_stride + dy - 1,
                             img);
          } else {
            tma_load_2d_pair(a_dst, &tmA, fbar, akc, m0);
          }
          tma_load_2d_pair(b_dst, &tmB, fbar, bkc, brow);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        // Aborted: let the loads this pair started land (the leader's full
        // barriers count both CTAs' bytes) before shared memory goes away.
        volatile int never = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(full_bar(s), (issued_parity >> s) & 1u, &never, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
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
            umma_ss_pair(d_tmem, ad, bd, args.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(accf_bar(acc), 0x3);
      }
      umma_commit_pair(drain_bar, 0x1);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, args.status, kStatusTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp & 3;
    const int row_in_tile = ew * 32 + lane;
    const uint32_t buf0 = sbase + L::kEpiOffset + (ew * 2) * L::kStageBuf;
    const uint32_t acce_leader0 = mapa_shared(acce_bar(0), 0);
    const uint32_t acce_leader1 = mapa_shared(acce_bar(1), 0);
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

  // Both CTAs: every MMA into this pair's TMEM has retired (the leader waited
  // on its drain barrier) and every read of it is done before it is freed.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, L::kTmemCols);
}

}  // namespace nd
