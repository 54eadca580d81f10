// Host side of the tcgen05 flash-attention kernel (attention_sm100.cuh).
#include <algorithm>
#include <climits>
#include <cmath>

#include "attention_sm100.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {

constexpr int64_t kAttnCounterBytes = 16384;  // one unsigned per split unit (at most 4096)

int64_t attn_piece_bytes(int hd) { return 256 * (8 + 4 * static_cast<int64_t>(hd)); }

// Sets the kernel's shared-memory limit and checks its register split, once
// per device.
template <int HD, bool SPLIT, bool F16>
int configure_attention() {
  static bool configured[64] = {};
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    auto kernel = attention_sm100_kernel<HD, SPLIT, F16>;
    int rc = check_register_split(reinterpret_cast<const void*>(kernel), kAttnThreads, kAttnRegsNeeded, "attention");
    if (rc) return rc;
    ND_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem<HD>::kLaunchBytes));
    configured[dev & 63] = true;
  }
  return ND_OK;
}

template <int HD, bool SPLIT, bool F16>
int launch_attention(dim3 grid, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const AttnArgs& g, cudaStream_t stream) {
  int rc = configure_attention<HD, SPLIT, F16>();
  if (rc) return rc;
  ND_CUDA(launch_pdl(attention_sm100_kernel<HD, SPLIT, F16>, grid, dim3(kAttnThreads), AttnSmem<HD>::kLaunchBytes, stream,
                     tq, tk, tv, g));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

// CTAs of the attention kernel resident at once on this device (one per SM:
// 512 TMEM columns and the 384 x 168 register file each); 0 if unknown.
template <int HD>
int attn_slots() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int& c = cached[dev & 63];
  if (!c) {
    if (configure_attention<HD, true, false>()) return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attention_sm100_kernel<HD, true, false>, kAttnThreads,
                                                      AttnSmem<HD>::kLaunchBytes) != cudaSuccess || per_sm <= 0)
      return 0;
    c = per_sm * sm_count();
  }
  return c;
}

// The split of the units past the last whole wave: each of the T tail units
// runs as s CTAs over a 1/s share of the keys, so the tail takes
// ceil(T s / slots) rounds of (n_kv / s + fixed) key-tile times instead of
// one round of (n_kv + fixed). The fixed costs (Q load, pipeline fill and
// drain; for pieces also the partial write and the merge) are counted in
// key tiles. Returns 1 (no split) unless the model gains 10 %, and for tails
// of more than half a wave: there the model's gain did not show (cfg3's
// 84-unit tail of 148: 1.00x measured for a predicted 1.03x), while the
// split kernel's extra registers cost its whole units ~3 %.
int choose_split(int64_t units, int slots, int n_kv, int64_t max_pieces) {
  if (slots <= 0) return 1;
  const int64_t tail = units % slots;
  if (tail == 0 || 2 * tail > slots) return 1;
  const double fixed = 1.5, merge = 1.0;
  const double base = n_kv + fixed;
  int best = 1;
  double best_cost = base;
  for (int s = 2; s <= kAttnMaxSplit && 2 * s <= n_kv && tail * s <= max_pieces; ++s) {
    const double rounds = static_cast<double>((tail * s + slots - 1) / slots);
    const double cost = rounds * (static_cast<double>(n_kv) / s + fixed + merge);
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best_cost < 0.9 * base ? best : 1;
}

}  // namespace

int64_t attention_workspace_bytes(int hd) {
  if (hd != 64 && hd != 128) return 0;
  return kAttnCounterBytes + 2LL * sm_count() * attn_piece_bytes(hd);
}

int attention(const nd_attention_args& a, cudaStream_t stream) {
  if (a.dtype == ND_F32) return attention_f32(a, stream);
  if (a.dtype != ND_BF16 && a.dtype != ND_F16) return fail(ND_ERR_INVALID, "attention: dtype must be bf16, f16 or f32");
  if (a.out_dtype != 0 && a.out_dtype != a.dtype) return fail(ND_ERR_INVALID, "attention: out_dtype must match a 16-bit dtype");
  if (a.head_dim != 128 && a.head_dim != 64) return fail(ND_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  const int hd = a.head_dim;
  if (a.heads <= 0 || a.batch <= 0 || a.q_rows <= 0 || a.kv_rows <= 0)
    return fail(ND_ERR_INVALID, "attention: empty shape");
  if (a.q_rows > INT_MAX / 4 || a.kv_rows > INT_MAX / 4 || a.batch * a.q_rows > INT_MAX / 2 ||
      a.batch * a.kv_rows > INT_MAX / 2)
    return fail(ND_ERR_INVALID, "attention: shape too large");
  const int64_t limit = a.key_limit <= 0 || a.key_limit > a.kv_rows ? a.kv_rows : a.key_limit;
  if (!a.q || !a.k || !a.v || !a.out) return fail(ND_ERR_INVALID, "attention: null operand");
  const int kvh = a.kv_heads > 0 ? a.kv_heads : a.heads;
  if (a.heads % kvh) return fail(ND_ERR_INVALID, "attention: kv_heads must divide heads");
  const int64_t width = static_cast<int64_t>(a.heads) * hd;
  const int64_t kv_width = static_cast<int64_t>(kvh) * hd;
  if (a.ldq < width || a.ldk < kv_width || a.ldv < kv_width || a.ldo < width)
    return fail(ND_ERR_INVALID, "attention: leading dimensions must cover heads (kv_heads) * head_dim");
  if ((a.ldo % 8) || (reinterpret_cast<uintptr_t>(a.out) & 15u))
    return fail(ND_ERR_INVALID, "attention: out must be 16-byte aligned with ldo % 8 == 0");
  if (a.causal && a.q_rows != a.kv_rows) return fail(ND_ERR_INVALID, "attention: causal needs q_rows == kv_rows");

  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, a.q, 2, a.batch * a.q_rows, width, a.ldq, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tk, a.k, 2, a.batch * a.kv_rows, kv_width, a.ldk, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tv, a.v, 2, a.batch * a.kv_rows, kv_width, a.ldv, 128, 64, true);
  if (rc) return rc;

  AttnArgs g{};
  g.q_rows = static_cast<int>(a.q_rows);
  g.kv_rows = static_cast<int>(a.kv_rows);
  g.key_limit = static_cast<int>(limit);
  g.causal = a.causal ? 1 : 0;
  g.kv_group = a.heads / kvh;
  const float scale = a.scale > 0.f ? a.scale : 1.0f / std::sqrt(static_cast<float>(hd));
  g.scale_log2 = scale * 1.4426950408889634f;
  g.out = a.out;
  g.ldo = a.ldo;
  g.out_f16 = a.dtype == ND_F16;
  g.idesc_s = make_idesc_f16(128, 128, a.dtype == ND_BF16);
  g.idesc_s64 = make_idesc_f16(128, 64, a.dtype == ND_BF16);
  g.idesc_pv = make_idesc_f16(128, hd, a.dtype == ND_BF16, false, true);
  g.status = device_status();
  if (!g.status) return fail(ND_ERR_CUDA, "attention: no device status word");

  const int64_t q_pairs = (a.q_rows + 255) / 256;
  const int64_t units = q_pairs * a.heads * a.batch;
  if (units > INT_MAX / 2) return fail(ND_ERR_INVALID, "attention: too many query tiles x heads x batch");
  g.q_pairs = static_cast<int>(q_pairs);
  g.heads = a.heads;
  g.full_units = static_cast<int>(units);
  g.split = 1;
  int64_t ctas = units;
  if (a.workspace && !a.causal) {
    if (reinterpret_cast<uintptr_t>(a.workspace) & 15u)
      return fail(ND_ERR_INVALID, "attention: workspace must be 16-byte aligned");
    const int64_t max_pieces = (a.workspace_bytes - kAttnCounterBytes) / attn_piece_bytes(hd);
    const int slots = hd == 128 ? attn_slots<128>() : attn_slots<64>();
    const int n_kv = static_cast<int>((limit + 127) / 128);
    const int split = max_pieces > 0 && slots > 0 ? choose_split(units, slots, n_kv, max_pieces) : 1;
    const int64_t tail = slots > 0 ? units % slots : 0;
    if (split > 1 && tail <= kAttnCounterBytes / 4) {
      g.full_units = static_cast<int>(units - tail);
      g.split = split;
      ctas = g.full_units + tail * split;
      uint8_t* ws = static_cast<uint8_t*>(a.workspace);
      g.counters = reinterpret_cast<unsigned*>(ws);
      g.part_ml = reinterpret_cast<float2*>(ws + kAttnCounterBytes);
      g.part_o = reinterpret_cast<float*>(ws + kAttnCounterBytes + max_pieces * 256 * 8);
    }
  }
  const bool f16 = g.out_f16 != 0;
  if (g.split > 1) {
    const dim3 grid(static_cast<unsigned>(ctas));
    if (hd == 128)
      return f16 ? launch_attention<128, true, true>(grid, tq, tk, tv, g, stream)
                 : launch_attention<128, true, false>(grid, tq, tk, tv, g, stream);
    return f16 ? launch_attention<64, true, true>(grid, tq, tk, tv, g, stream)
               : launch_attention<64, true, false>(grid, tq, tk, tv, g, stream);
  }
  const dim3 grid(static_cast<unsigned>(q_pairs), static_cast<unsigned>(a.heads), static_cast<unsigned>(a.batch));
  if (hd == 128)
    return f16 ? launch_attention<128, false, true>(grid, tq, tk, tv, g, stream)
               : launch_attention<128, false, false>(grid, tq, tk, tv, g, stream);
  return f16 ? launch_attention<64, false, true>(grid, tq, tk, tv, g, stream)
             : launch_attention<64, false, false>(grid, tq, tk, tv, g, stream);
}

}  // namespace nd
