// Flash attention forward for sm_100a, head_dim 128 or 64, bf16/fp16 in, fp32
// softmax and accumulation:   O = softmax(Q K^T / sqrt(d) + mask) V
//
// Replaces DmlOps.MultiheadAttention (Dml/DmlOps.cs:480-524) as Layers.Attend
// uses it (Graph/Layers.cs:260-279): packed heads ([rows, heads * 128]),
// unmasked or under a key-count mask (keys >= key_limit are left out, as the
// KeySequenceLength mask and the reference's CPU check do), optionally causal
// (row i sees keys 0..i, the text-row table of QwenImageConditioning).
//
// One CTA = one head x two 128-row query tiles (A and B) ping-ponging on the
// tensor core; 12 warps in three warpgroups:
//   warp 0      TMA: Q_A, Q_B once; K_j, V_j per key tile (2 stages)
//   warp 1      MMA: S_t = Q_t K_j^T (SS, into TMEM); O_t += P_t V_j (TS: P
//               read from TMEM, V from shared memory as an MN-major operand)
//   warps 2-3   idle; the first warpgroup gives up registers (setmaxnreg) so
//               the softmax warpgroups hold a whole 128-value score row each
//   warps 4-7   softmax of tile A (thread = query row), warps 8-11 tile B:
//               row max / exp2 / row sum in registers, P written back over
//               S in TMEM as bf16, lazy O rescale (only when the running max
//               grows by more than 2^8), final 1/l scaling and store.
// TMEM columns: S_A [0,128) S_B [128,256) O_A [256, 256+HD) O_B [256+HD, 256+2HD).
// While tile A's softmax runs, the tensor core does PV_B and S_B of the
// next step, and the other way round. The softmax hands P over in parts (32
// keys at d = 128, 64 at d = 64), each with its own barrier, so PV over the
// first keys runs while the exponentials of the last are still computed.
#pragma once

#include "nd_common.cuh"

namespace nd {

struct AttnArgs {
  int q_rows;       // query rows per batch item
  int kv_rows;      // key rows per batch item
  int key_limit;    // keys visible per batch item (<= kv_rows)
  int causal;       // row i sees keys [0, i]
  int kv_group;     // query heads per key / value head (grouped-query attention)
  float scale_log2; // softmax scale * log2(e)
  void* out;        // [batch * q_rows, ldo], head h at columns [h*128, h*128+128)
  long long ldo;
  int out_f16;
  uint32_t idesc_s, idesc_pv, idesc_s64;
  unsigned* status;
  // 1-D grid over units = query-tile pairs x heads x batch (pair fastest).
  // Units [0, full_units) run whole, one CTA each; every later unit runs as
  // `split` CTAs over consecutive key ranges, and the last of them to finish
  // merges the pieces.
  int q_pairs, heads;
  int full_units, split;
  float* part_o;      // [piece][tile][HD][128]: each piece's unnormalised O, row fastest
  float2* part_ml;    // [piece][tile][128]: (running max in log2 units, row sum)
  unsigned* counters; // [split unit]: pieces arrived (the merging piece resets it to 0)
};

// Largest split of one unit (the host never asks for more).
constexpr int kAttnMaxSplit = 16;

template <int HD>
struct AttnSmem {
  static constexpr int kChunks = HD / 64;       // 64-column (128-byte) chunks of a row
  static constexpr int kTile = 128 * HD * 2;    // one [128 x HD] tile (32 KB at HD 128)
  static constexpr int kQ = 0;                  // Q_A, Q_B
  static constexpr int kK = 2 * kTile;          // K stages
  static constexpr int kV = 4 * kTile;          // V stages
  static constexpr int kBar = 6 * kTile;        // 192 KB at HD 128
  // q_full, k_full[2], v_full[2], kv_empty[2], s_full[2], p_full[2][4 parts], o_full[2], drain, s_loaded[2]
  static constexpr int kNumBars = 22;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kTotal = kMisc + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
};

__device__ __forceinline__ void attn_store_row(uint16_t* dst_row, int col, const float (&v)[32], int f16) {
  uint32_t p[16];
  if (f16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) p[i] = pack_f16(v[2 * i], v[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) p[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
  }
  uint4* dst = reinterpret_cast<uint4*>(dst_row + col);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
}

// Register split: 384 threads x 168 at launch = 64512 = 128 x 72 (first
// warpgroup) + 256 x 216 (the two softmax warpgroups). The host checks the
// launch count before every launch.
constexpr int kAttnThreads = 384;
constexpr int kAttnRegsLow = 72;
constexpr int kAttnRegsHigh = 216;
constexpr int kAttnRegsNeeded = 128 * kAttnRegsLow + 256 * kAttnRegsHigh;

// SPLIT: the 1-D grid of whole units and key-range pieces (AttnArgs::split);
// otherwise a (query-tile pair, head, batch) grid of whole units, with none
// of the pieces' code (it costs the d = 128 loop ~3 % in registers).
// F16: fp16 operands (P packed to fp16), else bf16. A compile-time choice: a
// run-time select packs every P pair both ways (two SFU conversions per pair
// instead of one, on the unit the exponentials saturate).
template <int HD, bool SPLIT, bool F16>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  using L = AttnSmem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kBar;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto v_full = [&](int s) { return bars + 8u * (3 + s); };
  auto kv_empty = [&](int s) { return bars + 8u * (5 + s); };
  auto s_full = [&](int t) { return bars + 8u * (7 + t); };
  // P of part h (128 / kParts keys) of tile t's current key block
  constexpr int kParts = HD == 128 ? 4 : 2;  // measured: quarters at d = 128, halves at d = 64
  // At d = 64 the next key block's upper-half scores are computed before
  // this block's PV (+6 % measured); at d = 128 that delays PV (-18 %).
  constexpr bool kEarlyS = HD == 64;
  auto p_full = [&](int t, int h) { return bars + 8u * (9 + 4 * t + h); };
  auto o_full = [&](int t) { return bars + 8u * (17 + t); };
  const uint32_t drain_bar = bars + 8u * 19;
  // the softmax has read tile t's scores into registers: S columns [64, 128)
  // may take the next key block's scores
  auto s_loaded = [&](int t) { return bars + 8u * (20 + t); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int unit = 0, piece = 0, nsplit = 1, head, batch, q_tile0;  // q_tile0: within the batch item
  if constexpr (SPLIT) {
    unit = blockIdx.x;
    if (unit >= a.full_units) {
      nsplit = a.split;
      piece = (unit - a.full_units) % nsplit;
      unit = a.full_units + (unit - a.full_units) / nsplit;
    }
    head = (unit / a.q_pairs) % a.heads;
    batch = unit / (a.q_pairs * a.heads);
    q_tile0 = (unit % a.q_pairs) * 256;
  } else {
    head = blockIdx.y;
    batch = blockIdx.z;
    q_tile0 = blockIdx.x * 256;
  }
  const long long q_row0 = static_cast<long long>(batch) * a.q_rows + q_tile0;
  const int kv_row0 = batch * a.kv_rows;
  // Key tiles this CTA visits: all visible keys, or (causal) up to its last
  // row; a piece of a split unit takes its share [j_begin, j_begin + n_kv).
  int limit = a.key_limit;
  if (a.causal) limit = min(limit, q_tile0 + 256);
  const int n_all = (limit + 127) / 128;
  const int j_begin = piece * n_all / nsplit;
  const int n_kv = (piece + 1) * n_all / nsplit - j_begin;
  // the piece's first key row, and the key limit counted from it (the roles
  // below take these, so the piece offset is not one more live value)
  const int kv_row_first = kv_row0 + j_begin * 128;
  const int limit_rel = limit - j_begin * 128;
  const int col0 = head * HD;
  const int kv_col0 = (head / a.kv_group) * HD;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
      mbar_init(s_full(s), 1);
      for (int h = 0; h < kParts; ++h) mbar_init(p_full(s, h), 4);
      mbar_init(o_full(s), 1);
      mbar_init(s_loaded(s), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch();
  griddep_wait();

  // Each role's code sits inside its warpgroup's setmaxnreg branch, so the
  // compiler budgets each region with that branch's register count.
  if (warp < 4) {
    reg_dealloc<kAttnRegsLow>();
  if (warp == 0) {
    // ------------------------------------------------------------ loads
    if (elect_one()) {
      uint32_t issued = 0, issued_parity = 0;  // K/V stages with loads in flight
      bool q_issued = false;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, 2 * L::kTile);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_2d(sbase + L::kQ + t * L::kTile + c * 16384, &tmQ, q_full, col0 + c * 64,
                      static_cast<int>(q_row0) + t * 128);
      q_issued = true;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(kv_empty(st), ph ^ 1u, abort_flag, a.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        const int krow = kv_row_first + j * 128;
        mbar_arrive_expect_tx(k_full(st), L::kTile);
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_2d(sbase + L::kK + st * L::kTile + c * 16384, &tmK, k_full(st),
                      kv_col0 + c * 64, krow);
        mbar_arrive_expect_tx(v_full(st), L::kTile);
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_2d(sbase + L::kV + st * L::kTile + c * 16384, &tmV, v_full(st),
                      kv_col0 + c * 64, krow);
        issued |= 1u << st;
        issued_parity = (issued_parity & ~(1u << st)) | (ph << st);
      }
      if (!ok) {
        volatile int never = 0;
        if (q_issued) mbar_wait(q_full, 0, &never, nullptr, 0);
        for (int s = 0; s < 2; ++s) {
          if (issued & (1u << s)) {
            mbar_wait(k_full(s), (issued_parity >> s) & 1u, &never, nullptr, 0);
            mbar_wait(v_full(s), (issued_parity >> s) & 1u, &never, nullptr, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (elect_one()) {
      bool ok = mbar_wait(q_full, 0, abort_flag, a.status, kStatusTimeoutMma);
      auto issue_s = [&](int t, int st) {
        const uint32_t q_addr = sbase + L::kQ + t * L::kTile;
        const uint32_t k_addr = sbase + L::kK + st * L::kTile;
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t off = c * 16384 + kk * 32;
            umma_ss(tmem + t * 128, make_sdesc_sw128(q_addr + off, 16, 1024),
                    make_sdesc_sw128(k_addr + off, 16, 1024), a.idesc_s, (c | kk) != 0 ? 1u : 0u);
          }
        umma_commit(s_full(t));
      };
      // S of one half of the key block (keys [64 hi, 64 hi + 64)) into the
      // matching half of the tile's S columns
      auto issue_s_half = [&](int t, int st, int hi) {
        const uint32_t q_addr = sbase + L::kQ + t * L::kTile;
        const uint32_t k_addr = sbase + L::kK + st * L::kTile + hi * 64 * 128;
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t off = c * 16384 + kk * 32;
            umma_ss(tmem + t * 128 + hi * 64, make_sdesc_sw128(q_addr + off, 16, 1024),
                    make_sdesc_sw128(k_addr + off, 16, 1024), a.idesc_s64, (c | kk) != 0 ? 1u : 0u);
          }
      };
      auto issue_pv = [&](int t, int st, bool acc, int kk0) {  // keys [16 kk0, 16 kk0 + 128 / kParts)
        const uint32_t v_addr = sbase + L::kV + st * L::kTile;
#pragma unroll
        for (int kk = kk0; kk < kk0 + 8 / kParts; ++kk) {
          // V as the B operand [N = d, K = keys], d contiguous: MN-major,
          // 64-wide d chunks 16 KB apart (LBO), 8-key groups 1 KB apart (SBO).
          umma_ts(tmem + 256 + t * HD, tmem + t * 128 + kk * 8,
                  make_sdesc_sw128(v_addr + kk * 16 * 128, 16384, 1024), a.idesc_pv,
                  (acc || kk > 0) ? 1u : 0u);
        }
      };
      if (ok && n_kv > 0) {
        ok = mbar_wait(k_full(0), 0, abort_flag, a.status, kStatusTimeoutMma);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_s(1, 0);
        }
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const bool more = j + 1 < n_kv;
        const int nst = (j + 1) & 1;
        const uint32_t nph = ((j + 1) >> 1) & 1;
        if (!mbar_wait(v_full(st), ph, abort_flag, a.status, kStatusTimeoutMma)) break;
        for (int t = 0; t < 2; ++t) {
          if (kEarlyS && more) {
            // the next key block's scores for keys 64..127 go to S columns the
            // softmax has already read, before this block's PV
            if (t == 0 && !mbar_wait(k_full(nst), nph, abort_flag, a.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            if (!mbar_wait(s_loaded(t), j & 1, abort_flag, a.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s_half(t, nst, 1);
          }
          // PV over each part of the keys as soon as its P is in TMEM, while
          // the softmax still works on the rest
          for (int h = 0; h < kParts && ok; ++h) {
            if (!mbar_wait(p_full(t, h), j & 1, abort_flag, a.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, st, j > 0 || h > 0, h * (8 / kParts));
          }
          if (!ok) break;
          if (t == 1) umma_commit(kv_empty(st));
          if (more) {
            if (kEarlyS) {
              issue_s_half(t, nst, 0);  // keys 0..63: over P, after the PVs that read it
              umma_commit(s_full(t));
            } else {
              if (t == 0 && !mbar_wait(k_full(nst), nph, abort_flag, a.status, kStatusTimeoutMma)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(t, nst);  // the whole block's scores (commits s_full)
            }
          } else {
            umma_commit(o_full(t));
          }
        }
      }
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, a.status, kStatusTimeoutDrain);
    }
  }
  } else {
    reg_alloc<kAttnRegsHigh>();
    // ------------------------------------------------------------ softmax
    const int t = (warp - 4) >> 2;  // query tile of this warpgroup
    const int ew = warp & 3;        // TMEM lane quarter
    const int r = ew * 32 + lane;   // row within the tile
    const int q_in_batch = q_tile0 + t * 128 + r;
    // this row's output (head columns included); null past the batch item's rows
    uint16_t* const out_row = q_in_batch < a.q_rows
        ? reinterpret_cast<uint16_t*>(a.out) + (q_row0 + t * 128 + r) * a.ldo + col0 : nullptr;
    const uint32_t lane_off = static_cast<uint32_t>(ew * 32) << 16;
    const uint32_t s_tm = tmem + lane_off + t * 128;
    const uint32_t o_tm = tmem + lane_off + 256 + t * HD;
    // keys of this piece's block j visible to this row: vis_end - 128 j
    // (the key count, and with causal the row's own position)
    const int vis_end = a.causal ? min(limit, q_in_batch + 1) : limit_rel;  // causal launches are never split
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait(s_full(t), j & 1, abort_flag, a.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_tm + c * 32, sr[c]);
      tmem_ld_wait();
      if (kEarlyS) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_loaded(t));
      }
      // Masks: keys past the visible count (and past the end), causal.
      const int vis = vis_end - j * 128;
      if (vis < 128) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i >= vis) sr[c][i] = __float_as_uint(-INFINITY);
      }
      // Row max and (below) row sum over 8 / 4 independent partials (one serial
      // chain over 128 values would cost its full latency per element); the
      // loop is issue-bound, so the max takes three inputs and the scale and
      // sum run as paired f32x2 operations.
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = fmaxf(__uint_as_float(sr[0][2 * k]), __uint_as_float(sr[0][2 * k + 1]));
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = (c == 0 ? 16 : 0); i < 32; i += 2)
          m8[(i >> 1) & 7] = fmax3(m8[(i >> 1) & 7], __uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1]));
      float mx = fmaxf(fmax3(m8[0], m8[1], m8[2]), fmax3(fmax3(m8[3], m8[4], m8[5]), m8[6], m8[7]));
      mx *= a.scale_log2;
      const float m_new = fmaxf(m, mx);
      const bool need = m_new > m + 8.0f;
      const float m_use = need ? m_new : m;
      const float factor = fast_exp2(m - m_use);  // 0 on the first tile
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_tm + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(o_tm + c * 32, o);
        }
        tmem_st_wait();
      }
      m = m_use;
      float2 s4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) s4[k] = make_float2(0.f, 0.f);
      const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
      const float2 nm2 = make_float2(-m, -m);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = ffma2(make_float2(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])),
                                 sc2, nm2);
          const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          s4[i & 3] = fadd2(s4[i & 3], p);
          pk[i] = F16 ? pack_f16(p.x, p.y) : pack_bf16(p.x, p.y);
        }
        tmem_st16(s_tm + c * 16, pk);
        if ((c + 1) % (4 / kParts) == 0) {  // a part of the row's P is in TMEM: hand it over
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full(t, c / (4 / kParts)));
        }
      }
      const float rowsum = ((s4[0].x + s4[0].y) + (s4[1].x + s4[1].y)) + ((s4[2].x + s4[2].y) + (s4[3].x + s4[3].y));
      l = l * factor + rowsum;
    }
    const bool have_o = ok && n_kv > 0 && mbar_wait(o_full(t), 0, abort_flag, a.status, kStatusTimeoutEpilogue);
    if (have_o) {
      __syncwarp();
      tc_fence_after();
    }
    // (the split position is re-derived from the block index and the
    // arguments here rather than kept live through the softmax loop)
    const int pidx = SPLIT ? static_cast<int>(blockIdx.x) - a.full_units : -1;
    if (!SPLIT || pidx < 0) {
      if (have_o) {
        const float inv = 1.0f / l;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_tm + c * 32, o);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
          if (out_row) attn_store_row(out_row, c * 32, v, F16);
        }
      }
    } else if constexpr (SPLIT) {
      // A piece of a split unit: its unnormalised O and (m, l) go to the
      // workspace (column-major per tile, so a warp's 32 rows are one
      // 128-byte line per column), then it counts itself in. The last piece
      // to arrive merges all of them in piece order.
      const int ns = a.split;
      if (have_o) {
        float* po = a.part_o + (static_cast<size_t>(pidx) * 2 + t) * HD * 128 + r;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_tm + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(po + (c * 32 + i) * 128, __uint_as_float(o[i]));
        }
        __stcg(&a.part_ml[(static_cast<size_t>(pidx) * 2 + t) * 128 + r], make_float2(m, l));
      }
      // Every piece arrives once, also after a timeout (its status is set and
      // the merged rows are then not meaningful), so the count stays exact.
      volatile int* is_last = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);
      __threadfence();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const unsigned split_unit = static_cast<unsigned>(pidx / ns);
      if (threadIdx.x == 128) {
        const unsigned prev = atomicAdd(&a.counters[split_unit], 1u);
        const int last = prev == static_cast<unsigned>(ns - 1);
        if (last) a.counters[split_unit] = 0u;  // every piece has counted: ready for the next launch
        *is_last = last;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (*is_last) {
        __threadfence();
        const int first = static_cast<int>(split_unit) * ns;
        const float2* ml = a.part_ml + (static_cast<size_t>(first) * 2 + t) * 128 + r;
        float mx = -INFINITY;
        for (int i = 0; i < ns; ++i) mx = fmaxf(mx, __ldcg(ml + static_cast<size_t>(i) * 256).x);
        float sum = 0.f;
        for (int i = 0; i < ns; ++i) {
          const float2 p = __ldcg(ml + static_cast<size_t>(i) * 256);
          sum += fast_exp2(p.x - mx) * p.y;
        }
        const float inv = 1.0f / sum;
        const float* po = a.part_o + (static_cast<size_t>(first) * 2 + t) * HD * 128 + r;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float v[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = 0.f;
#pragma unroll 1
          for (int i = 0; i < ns; ++i) {
            const float w = fast_exp2(__ldcg(ml + static_cast<size_t>(i) * 256).x - mx);
            const float* src = po + static_cast<size_t>(i) * 2 * HD * 128 + c * 32 * 128;
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = fmaf(w, __ldcg(src + k * 128), v[k]);
          }
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] *= inv;
          if (out_row) attn_store_row(out_row, c * 32, v, F16);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace nd
