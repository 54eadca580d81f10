// Host side of the tcgen05 GEMM: argument checks, tensor maps, tile-width
// choice and launch. The kernel itself is in gemm_sm100.cuh.
#include <algorithm>
#include <climits>
#include <cmath>
#include <string>

#include "gemm2_sm100.cuh"
#include "gemm2_w8_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_w8_sm100.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {

template <int BN, int STAGES, bool CONV = false>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                const GemmArgs& g, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  static bool configured[64] = {};
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    ND_CUDA(cudaFuncSetAttribute(gemm_sm100_kernel<BN, STAGES, CONV>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, L::kLaunchBytes));
    configured[dev & 63] = true;
  }
  const int num_m = (g.M + 127) / 128;
  const int num_n = (g.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int grid = std::min(tiles, sm_count());
  ND_CUDA(launch_pdl(gemm_sm100_kernel<BN, STAGES, CONV>, dim3(grid), dim3(192), L::kLaunchBytes, stream, ta, tb, tc, g));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

// The pair kernel (gemm2_sm100.cuh): clusters of two CTAs, as many pairs as
// fit on the GPU at once (cudaOccupancyMaxActiveClusters, looked up once per
// device), each looping over 256-row tiles.
template <int BN, int STAGES, bool CONV = false>
int launch_gemm2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& g,
                 cudaStream_t stream) {
  using L = Gemm2Smem<BN, STAGES>;
  auto kernel = gemm2_sm100_kernel<BN, STAGES, CONV>;
  static int max_pairs[64] = {};
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::kLaunchBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  if (!max_pairs[dev & 63]) {
    ND_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kLaunchBytes));
    cfg.gridDim = dim3(2 * sm_count());
    cfg.numAttrs = 1;
    int n = 0;
    ND_CUDA(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
    if (n <= 0) return fail(ND_ERR_UNSUPPORTED, "linear: no CTA pair fits on this GPU");
    max_pairs[dev & 63] = n;
  }
  const int tiles = ((g.M + 255) / 256) * ((g.N + BN - 1) / BN);
  cfg.gridDim = dim3(2 * std::min(tiles, max_pairs[dev & 63]));
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  ND_CUDA(cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, g));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

// The int8 pair kernel (gemm2_w8_sm100.cuh), launched like launch_gemm2.
template <int BN, int STAGES, int BSTAGES, bool F16>
int launch_gemm2_w8(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& tc, const GemmArgs& g,
                    cudaStream_t stream) {
  using L = Gemm2W8Smem<BN, STAGES, BSTAGES>;
  auto kernel = gemm2_w8_sm100_kernel<BN, STAGES, BSTAGES, F16>;
  static int max_pairs[64] = {};
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kW8Threads);
  cfg.dynamicSmemBytes = L::kLaunchBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  if (!max_pairs[dev & 63]) {
    int rc = check_register_split(reinterpret_cast<const void*>(kernel), kW8Threads, kW8RegsNeeded, "int8 linear");
    if (rc) return rc;
    ND_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kLaunchBytes));
    cfg.gridDim = dim3(2 * sm_count());
    cfg.numAttrs = 1;
    int n = 0;
    ND_CUDA(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
    if (n <= 0) return fail(ND_ERR_UNSUPPORTED, "linear: no CTA pair fits on this GPU");
    max_pairs[dev & 63] = n;
  }
  const int tiles = ((g.M + 255) / 256) * ((g.N + BN - 1) / BN);
  cfg.gridDim = dim3(2 * std::min(tiles, max_pairs[dev & 63]));
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  ND_CUDA(cudaLaunchKernelEx(&cfg, kernel, ta, tw, tc, g));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

// Tile width: 256 unless the grid of 256-wide tiles leaves most SMs idle
// (narrow outputs, few rows), or, for the linear layers, 256-wide tiles pad
// the output columns more than 128-wide ones do (N = 320, 640, 1920: the
// padding is computed and thrown away; the SDXL step's linear layers gained
// 0.9 ms). The convolutions keep 256: at K = 9 Cin a 128-wide tile doubles
// the A traffic per FLOP and measured slower (the SDXL step's convolutions
// 3.84 -> 4.00 ms). (A 192-wide variant filled the last wave better at
// N = 3072 but measured slower per tile on B200.)
int pick_bn(int64_t rows, int64_t n, bool force256, bool pad_aware = true) {
  if (force256) return 256;
  const int64_t tiles256 = ((rows + 127) / 128) * ((n + 255) / 256);
  if (n < 256 || tiles256 < sm_count()) return 128;
  if (!pad_aware) return 256;
  return (n + 255) / 256 * 256 > (n + 127) / 128 * 128 ? 128 : 256;
}

// Pair-tile width for the plain epilogues: 160 where 160-column tiles cut the
// rounds of pair tiles enough to pay (the SDXL widths 320 / 640 / 1280, whose
// 256-wide tiles pad or leave a near-empty last round and whose 128-wide ones
// double the rounds). The cost of one 256 x bn pair tile per 64-deep k block,
// per SM, is its MMA time (2 bn cycles) or, for narrow tiles, its operand
// loads (128 A rows + bn / 2 W rows of 128 B at about 85 B per cycle); a
// round of pair tiles is one per pair on the GPU. 160 must beat the width
// `bn` by 15 %: a partial last round costs less than the model says (the
// other SMs idle, the clock rises), which made 192-wide tiles at N = 3072
// measure even where this model gives them 6 %.
int pair_bn(int64_t rows, int64_t n, int bn) {
  if (n < 160) return bn;
  const int pairs = std::max(1, sm_count() / 2);
  auto cost = [&](int w) {
    const int64_t tiles = ((rows + 255) / 256) * ((n + w - 1) / w);
    const double per = std::max(2.0 * w, (128.0 + w / 2) * 1.5);
    return static_cast<double>((tiles + pairs - 1) / pairs) * per;
  };
  return cost(160) < 0.85 * cost(bn) ? 160 : bn;
}

// Whether a GEMM runs on CTA pairs (256 x bn tiles): enough rows for the 256-row
// tiles to fill the GPU, and no pair straddling two weight groups (the two
// CTAs of a pair multiply by one W tile).
bool use_pairs(const GemmArgs& g, int bn) {
  (void)bn;
  if (g.M < 1024) return false;
  if (g.group_split >= g.M || g.shared_weights || g.row_groups) return true;
  return g.group_split % 256 == 0;
}

template <int BN, int STAGES, bool F16>
int launch_gemm_w8(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& tc,
                   const GemmArgs& g, cudaStream_t stream) {
  using L = GemmW8Smem<BN, STAGES>;
  auto kernel = gemm_w8_sm100_kernel<BN, STAGES, F16>;
  static bool configured[64] = {};
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    int rc = check_register_split(reinterpret_cast<const void*>(kernel), kW8Threads, kW8RegsNeeded, "int8 linear");
    if (rc) return rc;
    ND_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kLaunchBytes));
    configured[dev & 63] = true;
  }
  const int tiles = ((g.M + 127) / 128) * ((g.N + BN - 1) / BN);
  const int grid = std::min(tiles, sm_count());
  ND_CUDA(launch_pdl(kernel, dim3(grid), dim3(kW8Threads), L::kLaunchBytes, stream, ta, tw, tc, g));
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace

namespace {

// fp32 compute on bf16 hi|lo pairs (ND_BF16X2): the same mainloop over three
// K segments, outputs as pairs (or fp32 for the attention's Q/K/V).
int linear_split(const nd_linear_args& a, cudaStream_t stream) {
  if (a.rows <= 0 || a.in_features <= 0 || a.out_features <= 0)
    return fail(ND_ERR_INVALID, "linear: empty shape");
  if (a.rows > INT_MAX || a.in_features > INT_MAX / 4 || a.out_features > INT_MAX / 4)
    return fail(ND_ERR_INVALID, "linear: shape too large");
  if (a.in_features % 64) return fail(ND_ERR_INVALID, "linear: bf16x2 operands need in_features % 64 == 0");
  if (a.weight_dtype != 0 && a.weight_dtype != ND_BF16X2)
    return fail(ND_ERR_INVALID, "linear: bf16x2 activations need bf16x2 weights");
  if (!a.x || !a.weight) return fail(ND_ERR_INVALID, "linear: null operand");
  if (a.ldx < 2 * a.in_features || a.ldx % 8) return fail(ND_ERR_INVALID, "linear: bf16x2 x needs ldx >= 2 * in_features, ldx % 8 == 0");
  const bool split = a.group_split < a.rows;
  const bool shared = a.shared_weights != 0;
  if (split && a.group_split <= 0) return fail(ND_ERR_INVALID, "linear: group_split must be positive");
  if (split && !shared && a.group_split % 128 != 0)
    return fail(ND_ERR_INVALID, "linear: group_split must be a multiple of 128 (or give shared_weights)");
  const int epi = a.epilogue;
  if (epi < 0 || epi > ND_EPI_GEGLU || epi == ND_EPI_ADD_STORE)
    return fail(ND_ERR_INVALID, "linear: unknown epilogue (ADD_STORE is not offered for bf16x2)");
  const bool swiglu = epi == ND_EPI_SWIGLU || epi == ND_EPI_GEGLU;
  if (swiglu && a.out_features % 128) return fail(ND_ERR_INVALID, "linear: SWIGLU / GEGLU need out_features % 128 == 0");
  const bool resid = epi == ND_EPI_RESIDUAL_GATE || epi == ND_EPI_RESIDUAL_ADD || epi == ND_EPI_STORE_F32;
  const bool qk = epi == ND_EPI_QK_NORM_ROPE;
  if (resid && (!a.residual || a.ldr < a.out_features || a.ldr % 4 != 0 || (reinterpret_cast<uintptr_t>(a.residual) & 15u)))
    return fail(ND_ERR_INVALID, "linear: residual epilogue needs a 16-byte aligned residual with ldr >= out_features, ldr % 4 == 0");
  if (qk && (!a.y || a.ldy < a.out_features || a.ldy % 4 != 0 || (reinterpret_cast<uintptr_t>(a.y) & 15u)))
    return fail(ND_ERR_INVALID, "linear: bf16x2 QK epilogue writes fp32 y: ldy >= out_features, ldy % 4 == 0, 16-byte aligned");
  if (!resid && !qk) {
    if (!a.y || a.ldy < 2 * a.out_features || a.ldy % 8 != 0 || (reinterpret_cast<uintptr_t>(a.y) & 15u))
      return fail(ND_ERR_INVALID, "linear: bf16x2 output needs a 16-byte aligned y with ldy >= 2 * out_features, ldy % 8 == 0");
    if (a.out_features % 32) return fail(ND_ERR_INVALID, "linear: bf16x2 output needs out_features % 32 == 0");
  }
  if (epi == ND_EPI_RESIDUAL_GATE && !a.gate) return fail(ND_ERR_INVALID, "linear: gate missing");
  const int64_t span = a.norm_span > 0 ? a.norm_span : a.qk_cols / 2;
  if (qk) {
    if (!a.qk_norm) return fail(ND_ERR_INVALID, "linear: qk epilogue needs qk_norm");
    if ((a.rope_cos == nullptr) != (a.rope_sin == nullptr))
      return fail(ND_ERR_INVALID, "linear: give both rope_cos and rope_sin, or neither");
    if (a.qk_cols <= 0 || a.qk_cols % 128 != 0 || a.qk_cols > a.out_features)
      return fail(ND_ERR_INVALID, "linear: qk_cols must be a positive multiple of 128, <= out_features");
    if (span <= 0 || span % 128 != 0 || a.qk_cols % span != 0)
      return fail(ND_ERR_INVALID, "linear: norm_span must be a multiple of 128 dividing qk_cols");
    if (a.out_features % 128 != 0) return fail(ND_ERR_INVALID, "linear: qk epilogue needs out_features % 128 == 0");
    if (a.rope_period < 0) return fail(ND_ERR_INVALID, "linear: rope_period must be >= 0");
  }
  if (a.bias && (reinterpret_cast<uintptr_t>(a.bias) & 15u))
    return fail(ND_ERR_INVALID, "linear: bias must be 16-byte aligned");
  if (a.out_features % 4 != 0 && (a.bias || a.gate))
    return fail(ND_ERR_INVALID, "linear: bias/gate need out_features % 4 == 0");

  const int groups = split && !shared ? 2 : 1;
  const int64_t K2 = 2 * a.in_features;
  CUtensorMap ta, tb, tc;
  int rc = make_tmap_2d(&ta, a.x, 2, a.rows, K2, a.ldx, 128, 64, true);
  if (rc) return rc;
  if (resid) rc = make_tmap_2d_typed(&tc, a.residual, ND_F32, a.rows, a.out_features, a.ldr, 32, 32, 128);
  else if (qk) rc = make_tmap_2d_typed(&tc, a.y, ND_F32, a.rows, a.out_features, a.ldy, 32, 32, 128);
  else rc = make_tmap_2d_typed(&tc, a.y, ND_BF16, a.rows, 2 * a.out_features, a.ldy, 32, 32, 64);
  if (rc) return rc;

  GemmArgs g{};
  g.M = static_cast<int>(a.rows);
  g.N = static_cast<int>(swiglu ? 2 * a.out_features : a.out_features);
  g.K = static_cast<int>(a.in_features);
  g.swiglu_half = swiglu ? static_cast<int>(a.out_features) : 0;
  g.shared_weights = shared ? 1 : 0;
  g.row_groups = shared && split ? 1 : 0;
  g.split_kb = static_cast<int>(a.in_features / 64);
  g.split_koff = static_cast<int>(a.in_features);
  g.out_kind = resid ? 0 : (qk ? 2 : 1);
  g.group_split = split ? static_cast<int>(a.group_split) : INT_MAX;
  g.epi = epi;
  g.out = a.y;
  g.ldo = a.ldy;
  g.resid = a.residual;
  g.ldr = a.ldr;
  g.bias = a.bias;
  g.bias_stride = static_cast<int>(swiglu ? 2 * a.out_features : a.out_features);
  g.gate = a.gate;
  g.gate_stride = static_cast<int>(a.gate_stride > 0 ? a.gate_stride : a.out_features);
  if (a.gate && (g.gate_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(a.gate) & 15u)))
    return fail(ND_ERR_INVALID, "linear: gate must be 16-byte aligned with gate_stride % 4 == 0");
  g.qk_norm = a.qk_norm;
  g.rope_cos = a.rope_cos;
  g.rope_sin = a.rope_sin;
  g.qk_cols = static_cast<int>(a.qk_cols);
  g.norm_span = static_cast<int>(span > 0 ? span : 128);
  g.norm_sets = static_cast<int>(a.qk_cols > 0 && span > 0 ? a.qk_cols / span : 1);
  g.rope_period = static_cast<int>(a.rope_period);
  g.head_dim = 128;
  g.norm_eps = a.eps;
  g.status = device_status();
  if (!g.status) return fail(ND_ERR_CUDA, "linear: no device status word");

  const int64_t n_all = g.N;
  const int bn = pick_bn(a.rows, n_all, qk);
  if (use_pairs(g, bn)) {
    g.idesc = make_idesc_f16(256, bn, true);
    rc = make_tmap_2d(&tb, a.weight, 2, groups * n_all, K2, K2, bn / 2, 64, true);
    if (rc) return rc;
    if (bn == 256) return launch_gemm2<256, 6>(ta, tb, tc, g, stream);
    return launch_gemm2<128, 8>(ta, tb, tc, g, stream);
  }
  g.idesc = make_idesc_f16(128, bn, true);
  rc = make_tmap_2d(&tb, a.weight, 2, groups * n_all, K2, K2, swiglu ? bn / 2 : bn, 64, true);
  if (rc) return rc;
  if (bn == 256) return launch_gemm<256, 4>(ta, tb, tc, g, stream);
  return launch_gemm<128, 6>(ta, tb, tc, g, stream);
}

}  // namespace

int linear(const nd_linear_args& a, cudaStream_t stream) {
  if (a.dtype == ND_BF16X2) return linear_split(a, stream);
  if (a.dtype != ND_BF16 && a.dtype != ND_F16) return fail(ND_ERR_INVALID, "linear: dtype must be bf16, f16 or bf16x2");
  if (a.rows <= 0 || a.in_features <= 0 || a.out_features <= 0)
    return fail(ND_ERR_INVALID, "linear: empty shape");
  if (a.rows > INT_MAX || a.in_features > INT_MAX || a.out_features > INT_MAX / 2)
    return fail(ND_ERR_INVALID, "linear: shape too large");
  if (a.in_features % 8 != 0) return fail(ND_ERR_INVALID, "linear: in_features must be a multiple of 8");
  const bool w8 = a.weight_dtype == ND_I8;
  if (a.weight_dtype != 0 && !w8 && a.weight_dtype != a.dtype)
    return fail(ND_ERR_INVALID, "linear: weight_dtype must be 0, the activation dtype or ND_I8");
  if (w8) {
    if (a.in_features % 16 != 0) return fail(ND_ERR_INVALID, "linear: int8 weights need in_features % 16 == 0");
    if (!a.scales) return fail(ND_ERR_INVALID, "linear: int8 weights need scales");
    if (a.scale_dtype != ND_F16 && a.scale_dtype != ND_F32)
      return fail(ND_ERR_INVALID, "linear: scale_dtype must be ND_F16 or ND_F32");
    if (a.quant_group < 0 || (a.quant_group > 0 && a.in_features % a.quant_group != 0))
      return fail(ND_ERR_INVALID, "linear: quant_group must divide in_features (or be 0: per channel)");
  }
  if (a.ldx < a.in_features || a.ldx % 8 != 0) return fail(ND_ERR_INVALID, "linear: ldx must be >= in_features and a multiple of 8");
  if (!a.x || !a.weight) return fail(ND_ERR_INVALID, "linear: null operand");
  const bool split = a.group_split < a.rows;
  const bool shared = a.shared_weights != 0;
  if (split && a.group_split <= 0) return fail(ND_ERR_INVALID, "linear: group_split must be positive");
  if (split && !shared && a.group_split % 128 != 0)
    return fail(ND_ERR_INVALID, "linear: group_split must be a multiple of 128 (or give shared_weights)");
  const int epi = a.epilogue;
  const bool resid = epi == ND_EPI_RESIDUAL_GATE || epi == ND_EPI_RESIDUAL_ADD || epi == ND_EPI_STORE_F32;
  if (epi < 0 || epi > ND_EPI_GEGLU) return fail(ND_ERR_INVALID, "linear: unknown epilogue");
  const bool swiglu = epi == ND_EPI_SWIGLU || epi == ND_EPI_GEGLU;
  if (swiglu && a.out_features % 128) return fail(ND_ERR_INVALID, "linear: SWIGLU / GEGLU need out_features % 128 == 0");
  if (epi == ND_EPI_ADD_STORE && (!a.addend || a.ld_add < a.out_features || a.ld_add % 8 != 0))
    return fail(ND_ERR_INVALID, "linear: ADD_STORE needs addend with ld_add >= out_features, ld_add % 8 == 0");
  if (resid && (!a.residual || a.ldr < a.out_features || a.ldr % 4 != 0))
    return fail(ND_ERR_INVALID, "linear: residual epilogue needs residual with ldr >= out_features, ldr % 4 == 0");
  if (!resid && (!a.y || a.ldy < a.out_features || a.ldy % 8 != 0))
    return fail(ND_ERR_INVALID, "linear: output needs y with ldy >= out_features, ldy % 8 == 0");
  if (epi == ND_EPI_RESIDUAL_GATE && !a.gate) return fail(ND_ERR_INVALID, "linear: gate missing");
  const int64_t span = a.norm_span > 0 ? a.norm_span : a.qk_cols / 2;
  if (epi == ND_EPI_QK_NORM_ROPE) {
    if (!a.qk_norm) return fail(ND_ERR_INVALID, "linear: qk epilogue needs qk_norm");
    if ((a.rope_cos == nullptr) != (a.rope_sin == nullptr))
      return fail(ND_ERR_INVALID, "linear: give both rope_cos and rope_sin, or neither");
    if (a.qk_cols <= 0 || a.qk_cols % 128 != 0 || a.qk_cols > a.out_features)
      return fail(ND_ERR_INVALID, "linear: qk_cols must be a positive multiple of 128, <= out_features");
    if (span <= 0 || span % 128 != 0 || a.qk_cols % span != 0)
      return fail(ND_ERR_INVALID, "linear: norm_span must be a multiple of 128 dividing qk_cols");
    if (a.out_features % 128 != 0) return fail(ND_ERR_INVALID, "linear: qk epilogue needs out_features % 128 == 0");
    if (a.rope_period < 0) return fail(ND_ERR_INVALID, "linear: rope_period must be >= 0");
  }
  if (a.bias && (reinterpret_cast<uintptr_t>(a.bias) & 15u))
    return fail(ND_ERR_INVALID, "linear: bias must be 16-byte aligned");
  if (a.out_features % 4 != 0 && (a.bias || a.gate))
    return fail(ND_ERR_INVALID, "linear: bias/gate need out_features % 4 == 0");

  const int groups = split && !shared ? 2 : 1;
  CUtensorMap ta, tb, tc;
  int rc = make_tmap_2d(&ta, a.x, 2, a.rows, a.in_features, a.ldx, 128, 64, true);
  if (rc) return rc;
  // The epilogue's TMA target: [32 x 32] chunks of the bf16/fp16 output
  // (64B swizzle) or of the fp32 residual / output (128B swizzle, float add).
  if (resid) {
    if (reinterpret_cast<uintptr_t>(a.residual) & 15u) return fail(ND_ERR_INVALID, "linear: residual must be 16-byte aligned");
    rc = make_tmap_2d_typed(&tc, a.residual, ND_F32, a.rows, a.out_features, a.ldr, 32, 32, 128);
  } else {
    if (reinterpret_cast<uintptr_t>(a.y) & 15u) return fail(ND_ERR_INVALID, "linear: y must be 16-byte aligned");
    rc = make_tmap_2d_typed(&tc, a.y, a.dtype, a.rows, a.out_features, a.ldy, 32, 32, 64);
  }
  if (rc) return rc;

  GemmArgs g{};
  g.M = static_cast<int>(a.rows);
  g.N = static_cast<int>(swiglu ? 2 * a.out_features : a.out_features);
  g.K = static_cast<int>(a.in_features);
  g.swiglu_half = swiglu ? static_cast<int>(a.out_features) : 0;
  g.shared_weights = shared ? 1 : 0;
  g.row_groups = shared && split ? 1 : 0;
  g.group_split = split ? static_cast<int>(a.group_split) : INT_MAX;
  g.epi = epi;
  g.out_f16 = a.dtype == ND_F16;
  g.out = a.y;
  g.ldo = a.ldy;
  g.resid = a.residual;
  g.ldr = a.ldr;
  g.bias = a.bias;
  g.bias_stride = static_cast<int>(swiglu ? 2 * a.out_features : a.out_features);
  g.gate = a.gate;
  g.gate_stride = static_cast<int>(a.gate_stride > 0 ? a.gate_stride : a.out_features);
  if (a.gate && (g.gate_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(a.gate) & 15u)))
    return fail(ND_ERR_INVALID, "linear: gate must be 16-byte aligned with gate_stride % 4 == 0");
  g.qk_norm = a.qk_norm;
  g.rope_cos = a.rope_cos;
  g.rope_sin = a.rope_sin;
  g.qk_cols = static_cast<int>(a.qk_cols);
  g.norm_span = static_cast<int>(span > 0 ? span : 128);
  g.norm_sets = static_cast<int>(a.qk_cols > 0 && span > 0 ? a.qk_cols / span : 1);
  g.rope_period = static_cast<int>(a.rope_period);
  g.addend = a.addend;
  g.ld_add = a.ld_add;
  g.head_dim = 128;
  g.norm_eps = a.eps;
  g.status = device_status();
  if (!g.status) return fail(ND_ERR_CUDA, "linear: no device status word");
  if (w8) {
    const int64_t group = a.quant_group > 0 ? a.quant_group : a.in_features;
    g.w8_scales = a.scales;
    g.w8_group = static_cast<int>(group);
    g.w8_scale_cols = static_cast<int>(a.in_features / group);
    g.w8_scale_f16 = a.scale_dtype == ND_F16;
  }

  // Tile width: pick_bn.
  const int64_t n_all = g.N;
  const int bn = pick_bn(a.rows, n_all, epi == ND_EPI_QK_NORM_ROPE);
  g.idesc = make_idesc_f16(128, bn, a.dtype == ND_BF16);
  if (w8) {
    if (bn == 256 && use_pairs(g, bn)) {
      // Each CTA of a pair loads and widens [bn / 2 rows x 64 bytes].
      g.idesc = make_idesc_f16(256, bn, a.dtype == ND_BF16);
      rc = make_tmap_2d_typed(&tb, a.weight, ND_I8, groups * n_all, a.in_features, a.in_features, bn / 2, 64, 0);
      if (rc) return rc;
      return g.out_f16 ? launch_gemm2_w8<256, 4, 4, true>(ta, tb, tc, g, stream)  // 4 raw + 4 widened slots
                       : launch_gemm2_w8<256, 4, 4, false>(ta, tb, tc, g, stream);
    }
    // Raw int8 tiles [bn rows x 64 bytes], unswizzled (the converters swizzle).
    rc = make_tmap_2d_typed(&tb, a.weight, ND_I8, groups * n_all, a.in_features, a.in_features,
                            swiglu ? bn / 2 : bn, 64, 0);
    if (rc) return rc;
    if (bn == 256)
      return g.out_f16 ? launch_gemm_w8<256, 4, true>(ta, tb, tc, g, stream)
                       : launch_gemm_w8<256, 4, false>(ta, tb, tc, g, stream);
    return g.out_f16 ? launch_gemm_w8<128, 6, true>(ta, tb, tc, g, stream)
                     : launch_gemm_w8<128, 6, false>(ta, tb, tc, g, stream);
  }
  if (use_pairs(g, bn)) {
    const int pbn = swiglu || epi == ND_EPI_QK_NORM_ROPE ? bn : pair_bn(a.rows, n_all, bn);
    g.idesc = make_idesc_f16(256, pbn, a.dtype == ND_BF16);
    rc = make_tmap_2d(&tb, a.weight, 2, groups * n_all, a.in_features, a.in_features, pbn / 2, 64, true);
    if (rc) return rc;
    if (pbn == 256) return launch_gemm2<256, 6>(ta, tb, tc, g, stream);
    if (pbn == 160) return launch_gemm2<160, 7>(ta, tb, tc, g, stream);
    return launch_gemm2<128, 8>(ta, tb, tc, g, stream);
  }
  rc = make_tmap_2d(&tb, a.weight, 2, groups * n_all, a.in_features, a.in_features, swiglu ? bn / 2 : bn, 64,
                    true);
  if (rc) return rc;
  if (bn == 256) return launch_gemm<256, 4>(ta, tb, tc, g, stream);
  return launch_gemm<128, 6>(ta, tb, tc, g, stream);
}

int conv2d(const nd_conv_args& c, cudaStream_t stream) {
  if (c.dtype != ND_F16 && c.dtype != ND_BF16) return fail(ND_ERR_INVALID, "conv2d: dtype must be f16 or bf16");
  if (c.batch <= 0 || c.height <= 0 || c.width <= 0 || c.in_channels <= 0 || c.out_channels <= 0)
    return fail(ND_ERR_INVALID, "conv2d: empty shape");
  if (c.in_channels % 8 || c.in_channels < 64)
    return fail(ND_ERR_UNSUPPORTED, "conv2d: in_channels must be a multiple of 8, at least 64");
  if (c.stride != 1 && c.stride != 2) return fail(ND_ERR_UNSUPPORTED, "conv2d: stride must be 1 or 2");
  const int ho = (c.height - 1) / c.stride + 1, wo = (c.width - 1) / c.stride + 1;
  if (wo <= 128 ? 128 % wo != 0 : wo % 128 != 0)
    return fail(ND_ERR_UNSUPPORTED, "conv2d: output width must divide 128 or be a multiple of 128");
  if ((static_cast<int64_t>(ho) * wo) % 128 != 0) return fail(ND_ERR_UNSUPPORTED, "conv2d: output pixels per image must be a multiple of 128");
  const int epi = c.epilogue;
  if (epi != ND_EPI_STORE && epi != ND_EPI_ADD_STORE && epi != ND_EPI_STORE_F32 && epi != ND_EPI_SILU)
    return fail(ND_ERR_INVALID, "conv2d: epilogue must be STORE, ADD_STORE, STORE_F32 or SILU");
  if (!c.x || !c.weight) return fail(ND_ERR_INVALID, "conv2d: null operand");
  if (epi == ND_EPI_STORE_F32 ? !c.y_f32 : !c.y) return fail(ND_ERR_INVALID, "conv2d: null output");
  if (epi == ND_EPI_ADD_STORE && !c.addend) return fail(ND_ERR_INVALID, "conv2d: ADD_STORE needs addend");
  if (epi != ND_EPI_STORE_F32 && c.out_channels % 8) return fail(ND_ERR_INVALID, "conv2d: out_channels % 8 for a 16-bit output");
  if (c.out_channels % 4) return fail(ND_ERR_INVALID, "conv2d: out_channels must be a multiple of 4");
  const int64_t M = static_cast<int64_t>(c.batch) * ho * wo;
  // Each tap's channels in chunks of 64; a last partial chunk reads past the
  // tensor's channel extent, which TMA fills with zeros, against zero rows of
  // the weight (stored with the channels padded to a multiple of 64).
  const int kpc = (c.in_channels + 63) / 64;
  const int64_t K = 9LL * kpc * 64;
  if (M > INT_MAX || K > INT_MAX) return fail(ND_ERR_INVALID, "conv2d: shape too large");

  CUtensorMap ta, tb, tc;
  const int64_t cin = c.in_channels;
  const int64_t dims[4] = {cin, c.width, c.height, c.batch};
  const int64_t strides[3] = {cin * 2, cin * c.width * 2, cin * c.width * c.height * 2};
  // A tile is 128 output pixels: 128 / wo whole rows, or (wide images) 128
  // pixels of one row. With a traversal stride s, TMA loads ceil(box / s)
  // elements along a dimension, so the box spans s x the output extent.
  const int tile_w = std::min(wo, 128);
  const int rows = 128 / tile_w;
  const int box[4] = {64, tile_w * c.stride, rows * c.stride, 1};
  const int es[4] = {1, c.stride, c.stride, 1};
  int rc = make_tmap_4d(&ta, c.x, c.dtype, dims, strides, box, es, 128);
  if (rc) return rc;
  if (epi == ND_EPI_STORE_F32) {
    rc = make_tmap_2d_typed(&tc, c.y_f32, ND_F32, M, c.out_channels, c.out_channels, 32, 32, 128);
  } else {
    rc = make_tmap_2d_typed(&tc, c.y, c.dtype, M, c.out_channels, c.out_channels, 32, 32, 64);
  }
  if (rc) return rc;

  GemmArgs g{};
  g.M = static_cast<int>(M);
  g.N = c.out_channels;
  g.K = static_cast<int>(K);
  g.epi = epi;
  g.out_f16 = c.dtype == ND_F16;
  g.out = c.y;
  g.ldo = c.out_channels;
  g.resid = c.y_f32;
  g.ldr = c.out_channels;
  g.bias = c.bias;
  g.bias_stride = static_cast<int>(c.bias_stride > 0 ? c.bias_stride : c.out_channels);
  g.group_split = c.per_batch_bias ? ho * wo : INT_MAX;
  g.periodic_groups = c.per_batch_bias ? 1 : 0;
  g.shared_weights = 1;
  g.addend = c.addend;
  g.ld_add = c.out_channels;
  g.conv_kpc = kpc;
  g.conv_hw = ho * wo;
  g.conv_w_out = wo;
  g.conv_stride = c.stride;
  g.head_dim = 128;
  g.status = device_status();
  if (!g.status) return fail(ND_ERR_CUDA, "conv2d: no device status word");
  const int bn = pick_bn(M, c.out_channels, false, false);
  // Pairs with 256- or 160-wide tiles (128-wide conv tiles stay on single
  // CTAs, as measured).
  const int pbn = use_pairs(g, 256) ? pair_bn(M, c.out_channels, 256) : 0;
  if (pbn == 160 || (pbn == 256 && bn == 256)) {
    g.idesc = make_idesc_f16(256, pbn, c.dtype == ND_BF16);
    rc = make_tmap_2d(&tb, c.weight, 2, c.out_channels, K, K, pbn / 2, 64, true);
    if (rc) return rc;
    if (pbn == 160) return launch_gemm2<160, 7, true>(ta, tb, tc, g, stream);
    return launch_gemm2<256, 6, true>(ta, tb, tc, g, stream);
  }
  g.idesc = make_idesc_f16(128, bn, c.dtype == ND_BF16);
  rc = make_tmap_2d(&tb, c.weight, 2, c.out_channels, K, K, bn, 64, true);
  if (rc) return rc;
  if (bn == 256) return launch_gemm<256, 4, true>(ta, tb, tc, g, stream);
  return launch_gemm<128, 6, true>(ta, tb, tc, g, stream);
}

int dequantize(const int8_t* q, const void* scales, int scale_dtype, int64_t quant_group, int64_t rows,
               int64_t cols, void* out, int out_dtype, cudaStream_t stream) {
  if (!q || !scales || !out) return fail(ND_ERR_INVALID, "dequantize: null operand");
  if (rows <= 0 || cols <= 0 || cols > INT_MAX) return fail(ND_ERR_INVALID, "dequantize: bad shape");
  if (scale_dtype != ND_F16 && scale_dtype != ND_F32) return fail(ND_ERR_INVALID, "dequantize: scale_dtype");
  if (out_dtype != ND_BF16 && out_dtype != ND_F16) return fail(ND_ERR_INVALID, "dequantize: out_dtype");
  const int64_t group = quant_group > 0 ? quant_group : cols;
  if (cols % group) return fail(ND_ERR_INVALID, "dequantize: quant_group must divide cols");
  const long long total = rows * cols;
  const unsigned grid = static_cast<unsigned>(std::min<long long>((total + 255) / 256, sm_count() * 16LL));
  dequant_w8_kernel<<<grid, 256, 0, stream>>>(q, scales, scale_dtype == ND_F16, static_cast<int>(group),
                                              static_cast<int>(cols / group), rows, static_cast<int>(cols),
                                              out, out_dtype == ND_F16);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd
