// The text towers, the step before the denoiser path, on the device:
//   Qwen3TextModel.Forward (Text/Qwen/Qwen3TextModel.cs:47-104): a Qwen3
//     decoder read as a text encoder (Anima's Qwen3-0.6B, and the language
//     model of Qwen-Image 2.1's Qwen3-VL-8B): pre-norm blocks of causal
//     grouped-query attention, a norm on every query and key head, rotary
//     positions, a SwiGLU feed-forward.
//   LlmAdapter.Forward (Models/Anima/LlmAdapter.cs:29-78): Anima's six-block
//     bridge from the Qwen3 hidden states to T5-shaped context: self- and
//     cross-attention with per-head norms and rotary positions (64-wide
//     heads), a GELU MLP, an output projection and a final norm.
// The reference runs both on the CPU (CpuMath) reading bf16 weights a row at
// a time; here the weights stay in HBM and each layer is a handful of the
// library's kernels: RMSNorm, the tcgen05 GEMM (fused head norm + RoPE for
// Qwen3's 128-wide heads, SwiGLU, residual adds), the flash attention with
// grouped-query heads. Calls run eagerly: their row count changes per prompt.
#include <cmath>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_common.cuh"
#include "nd_runtime.h"

namespace nd {

namespace {

// x[r, :] = table[ids[r], :] as fp32; table bf16 / f16 [vocab, width], or a
// bf16 hi|lo pair [vocab, 2 * width] (fp32 compute).
__global__ void embed_rows_kernel(const void* __restrict__ table, int tdt, const int32_t* __restrict__ ids,
                                  int rows, int width, float* __restrict__ x) {
  const long long n = static_cast<long long>(rows) * width;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / width), c = static_cast<int>(i - static_cast<long long>(r) * width);
    const long long id = ids[r];
    const uint16_t* t = static_cast<const uint16_t*>(table);
    float v;
    if (tdt == ND_BF16X2) {
      const uint16_t hi = t[id * 2 * width + c], lo = t[id * 2 * width + width + c];
      v = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&hi)) +
          __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&lo));
    } else {
      const uint16_t h = t[id * width + c];
      v = tdt == ND_F16 ? __half2float(*reinterpret_cast<const __half*>(&h))
                        : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&h));
    }
    x[i] = v;
  }
}

__device__ __forceinline__ float load_any(const void* p, long long i, int dt) {
  if (dt == ND_F32) return static_cast<const float*>(p)[i];
  const uint16_t h = static_cast<const uint16_t*>(p)[i];
  return dt == ND_F16 ? __half2float(*reinterpret_cast<const __half*>(&h))
                      : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&h));
}

__device__ __forceinline__ void store_any(void* p, long long i, int dt, float v) {
  if (dt == ND_F32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == ND_F16) {
    const __half h = __float2half_rn(v);
    static_cast<uint16_t*>(p)[i] = *reinterpret_cast<const uint16_t*>(&h);
  } else {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    static_cast<uint16_t*>(p)[i] = *reinterpret_cast<const uint16_t*>(&h);
  }
}

// One warp per (row, head): RMSNorm over the head's features times the
// stored weight, then rotate-half with the row's angles. Lane l holds the
// pairs (l + 32k, l + 32k + hd/2).
template <int HD>
__global__ void __launch_bounds__(256) head_norm_rope_kernel(void* __restrict__ x, int dt, long long ld, int rows,
                                                             int heads, const float* __restrict__ w,
                                                             const float* __restrict__ cs,
                                                             const float* __restrict__ sn, float eps) {
  constexpr int kHalf = HD / 2;
  constexpr int kPer = kHalf / 32;
  const long long item = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (item >= static_cast<long long>(rows) * heads) return;
  const int r = static_cast<int>(item / heads), h = static_cast<int>(item - static_cast<long long>(r) * heads);
  const long long base = r * ld + static_cast<long long>(h) * HD;
  float lo[kPer], hi[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = lane + 32 * k;
    lo[k] = load_any(x, base + i, dt);
    hi[k] = load_any(x, base + kHalf + i, dt);
    ss = fmaf(lo[k], lo[k], fmaf(hi[k], hi[k], ss));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float sc = rsqrtf(ss / HD + eps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = lane + 32 * k;
    const float l = lo[k] * sc * w[i], u = hi[k] * sc * w[kHalf + i];
    float c = 1.f, s = 0.f;
    if (cs) {
      c = cs[static_cast<long long>(r) * kHalf + i];
      s = sn[static_cast<long long>(r) * kHalf + i];
    }
    store_any(x, base + i, dt, l * c - u * s);
    store_any(x, base + kHalf + i, dt, u * c + l * s);
  }
}

// CpuMath.RopeTables (Tensors/CpuMath.cs:177-194): inverse frequencies in
// float as torch computes them, angle = position * frequency.
void rope_tables_1d(int rows, int dim, double theta, float* cos, float* sin) {
  const int half = dim / 2;
  for (int i = 0; i < half; ++i) {
    const float frequency = 1.0f / std::pow(static_cast<float>(theta), 2.0f * i / dim);
    for (int m = 0; m < rows; ++m) {
      const float angle = static_cast<float>(m) * frequency;
      cos[static_cast<int64_t>(m) * half + i] = std::cos(angle);
      sin[static_cast<int64_t>(m) * half + i] = std::sin(angle);
    }
  }
}

unsigned grid_for(long long n) {
  return static_cast<unsigned>(std::max<long long>(1, std::min<long long>((n + 255) / 256, sm_count() * 16LL)));
}

// Common plumbing of the two towers: ids / outputs, tables, op helpers.
struct TextTower : nd_denoiser {
  int W = 0, H = 0, HD = 128, NB = 0, F = 0, V = 0, maxR = 0;
  double theta = 1e6;
  int dt = ND_BF16, lt = ND_BF16, pw = 1;
  size_t qe = 2;
  bool f32 = false;
  float eps = 1e-6f;
  int rows = 1;  // rows of the staged call
  int32_t* ids_d = nullptr;
  float *x = nullptr, *out_d = nullptr, *cos_d = nullptr, *sin_d = nullptr;
  std::vector<float> cos_h, sin_h;

  int common_build(const char* who) {
    const nd_model_desc& d = desc;
    if (d.compute != ND_BF16 && d.compute != ND_F16 && d.compute != ND_F32)
      return fail(ND_ERR_UNSUPPORTED, std::string(who) + ": compute must be bf16, f16 or f32");
    if (d.weight_dtype != d.compute) return fail(ND_ERR_UNSUPPORTED, std::string(who) + ": weights are stored in the compute dtype");
    if (d.context_rows <= 0 || d.vocab <= 0 || d.width <= 0 || d.width % 128 || d.blocks <= 0 || d.mlp_width % 128)
      return fail(ND_ERR_INVALID, std::string(who) + ": bad shape (width and mlp_width multiples of 128)");
    dt = d.compute;
    f32 = dt == ND_F32;
    lt = f32 ? ND_BF16X2 : dt;
    pw = f32 ? 2 : 1;
    qe = f32 ? 4 : 2;
    W = d.width;
    H = d.heads;
    NB = d.blocks;
    F = d.mlp_width;
    V = d.vocab;
    maxR = d.context_rows;
    theta = d.rope_theta > 0 ? d.rope_theta : 1e6;
    eps = d.eps > 0 ? d.eps : 1e-6f;
    return ND_OK;
  }

  int64_t latent_elems() const override { return 0; }
  const float* output() const override { return out_d; }
  int check_cond(int, const nd_named_tensor*, StepInputs&) override {
    return fail(ND_ERR_INVALID, "a text tower runs through nd_text_encode, not predict");
  }
  int stage(const StepInputs&, cudaStream_t) override { return fail(ND_ERR_INVALID, "text tower: use nd_text_encode"); }

  int rms(cudaStream_t s, const float* in, void* y, int out_dtype, int64_t ldy, const float* w) {
    nd_rmsnorm_args a{};
    a.x = in;
    a.ldx = W;
    a.in_dtype = ND_F32;
    a.y = y;
    a.ldy = ldy;
    a.out_dtype = out_dtype;
    a.rows = rows;
    a.width = W;
    a.weight = w;
    a.eps = eps;
    return rmsnorm(a, s);
  }

  void weight_args(nd_linear_args& a, const Mat& m, int64_t row) const { a.weight = m.at(row, 2); }

  int lin(cudaStream_t s, const void* xin, int64_t r, int64_t k, const Mat& w, int64_t wrow, int64_t n, int epi,
          void* y, int64_t ldy, float* resid = nullptr, const float* bias = nullptr) {
    nd_linear_args a{};
    a.dtype = lt;
    a.epilogue = epi;
    a.rows = r;
    a.in_features = k;
    a.out_features = n;
    a.x = xin;
    a.ldx = k * pw;
    weight_args(a, w, wrow);
    a.bias = bias;
    a.group_split = r;
    a.y = y;
    a.ldy = ldy * pw;
    a.residual = resid;
    a.ldr = W;
    a.eps = eps;
    return linear(a, s);
  }

  int embed(cudaStream_t s, const Mat& table) {
    embed_rows_kernel<<<grid_for(static_cast<long long>(rows) * W), 256, 0, s>>>(table.w, lt, ids_d, rows, W, x);
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }

  // Validate and stage one call's ids (host), run it, copy [rows, W] out.
  int run(const int32_t* ids, int n, float* out) {
    if (n <= 0 || n > maxR) return fail(ND_ERR_INVALID, "text_encode: rows must be 1.." + std::to_string(maxR));
    for (int i = 0; i < n; ++i)
      if (ids[i] < 0 || ids[i] >= V) return fail(ND_ERR_INVALID, "text_encode: token id " + std::to_string(ids[i]) + " out of the vocabulary");
    cudaStream_t s = dev->stream;
    rows = n;
    ND_CUDA(cudaMemcpyAsync(ids_d, ids, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, s));
    ND_TRY_RC(forward(s));
    ND_CUDA(cudaMemcpyAsync(out, out_d, static_cast<size_t>(n) * W * 4, cudaMemcpyDeviceToHost, s));
    ND_CUDA(cudaStreamSynchronize(s));
    return check_device_status(s);
  }
};

#define ND_OP(cls, flops, expr) \
  do {                          \
    prof_begin(s);              \
    int rc_ = (expr);           \
    if (rc_) return rc_;        \
    prof_end(s, cls, flops, 0.0); \
  } while (0)

// ------------------------------------------------------------ Qwen3
struct Qwen3Text final : TextTower {
  int KV = 0, QW = 0, KW = 0, QKV = 0;
  bool final_norm = true;
  Mat emb, qkv_w, o_w, gu_w, down_w;
  float *ln1 = nullptr, *ln2 = nullptr, *qn = nullptr, *kn = nullptr, *sets = nullptr, *fnorm = nullptr;
  void *xn = nullptr, *qkv = nullptr, *att = nullptr, *hid = nullptr;

  int build() override {
    ND_TRY_RC(common_build("qwen3"));
    const nd_model_desc& d = desc;
    if (d.head_dim != 128 || H <= 0) return fail(ND_ERR_INVALID, "qwen3: head_dim must be 128");
    KV = d.kv_heads > 0 ? d.kv_heads : H;
    if (H % KV) return fail(ND_ERR_INVALID, "qwen3: kv_heads must divide heads");
    if (f32 && W % 64) return fail(ND_ERR_INVALID, "qwen3: fp32 compute needs width % 64 == 0");
    QW = H * 128;
    KW = KV * 128;
    QKV = QW + 2 * KW;
    auto Vv = [&](int64_t n) { return static_cast<float*>(alloc(static_cast<size_t>(n) * 4, true)); };
    emb = alloc_mat(V, W, V);
    qkv_w = alloc_mat(static_cast<int64_t>(NB) * QKV, W, QKV);
    o_w = alloc_mat(static_cast<int64_t>(NB) * W, QW, W);
    gu_w = alloc_mat(static_cast<int64_t>(NB) * 2 * F, W, F);
    down_w = alloc_mat(static_cast<int64_t>(NB) * W, F, W);
    ln1 = Vv(static_cast<int64_t>(NB) * W);
    ln2 = Vv(static_cast<int64_t>(NB) * W);
    qn = Vv(static_cast<int64_t>(NB) * 128);
    kn = Vv(static_cast<int64_t>(NB) * 128);
    sets = Vv(static_cast<int64_t>(NB) * (H + KV) * 128);
    fnorm = Vv(W);
    auto S = [&](size_t b) { return alloc(b, false); };
    ids_d = static_cast<int32_t*>(S(static_cast<size_t>(maxR) * 4));
    x = static_cast<float*>(S(static_cast<size_t>(maxR) * W * 4));
    out_d = static_cast<float*>(S(static_cast<size_t>(maxR) * W * 4));
    cos_d = static_cast<float*>(S(static_cast<size_t>(maxR) * 64 * 4));
    sin_d = static_cast<float*>(S(static_cast<size_t>(maxR) * 64 * 4));
    xn = S(static_cast<size_t>(maxR) * W * 2 * pw);
    qkv = S(static_cast<size_t>(maxR) * QKV * qe);
    att = S(static_cast<size_t>(maxR) * QW * 2 * pw);
    hid = S(static_cast<size_t>(maxR) * F * 2 * pw);
    if (alloc_failed) return fail(ND_ERR_OOM, "qwen3: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));
    // registry (the checkpoint's names)
    auto M_ = [&](const std::string& n, const Mat& m, int64_t row, int64_t r) {
      add_slot(n, kMatrix, r, m.cols, m.at(row, 2));
    };
    M_("model.embed_tokens.weight", emb, 0, V);
    add_slot("model.norm.weight", kVector, W, 1, fnorm);
    for (int l = 0; l < NB; ++l) {
      const std::string p = "model.layers." + std::to_string(l) + ".";
      const int64_t q0 = static_cast<int64_t>(l) * QKV;
      add_slot(p + "input_layernorm.weight", kVector, W, 1, ln1 + static_cast<int64_t>(l) * W);
      M_(p + "self_attn.q_proj.weight", qkv_w, q0, QW);
      M_(p + "self_attn.k_proj.weight", qkv_w, q0 + QW, KW);
      M_(p + "self_attn.v_proj.weight", qkv_w, q0 + QW + KW, KW);
      add_slot(p + "self_attn.q_norm.weight", kVector, 128, 1, qn + static_cast<int64_t>(l) * 128);
      add_slot(p + "self_attn.k_norm.weight", kVector, 128, 1, kn + static_cast<int64_t>(l) * 128);
      M_(p + "self_attn.o_proj.weight", o_w, static_cast<int64_t>(l) * W, W);
      add_slot(p + "post_attention_layernorm.weight", kVector, W, 1, ln2 + static_cast<int64_t>(l) * W);
      M_(p + "mlp.gate_proj.weight", gu_w, static_cast<int64_t>(l) * 2 * F, F);
      M_(p + "mlp.up_proj.weight", gu_w, static_cast<int64_t>(l) * 2 * F + F, F);
      M_(p + "mlp.down_proj.weight", down_w, static_cast<int64_t>(l) * W, W);
    }
    cos_h.resize(static_cast<size_t>(maxR) * 64);
    sin_h.resize(static_cast<size_t>(maxR) * 64);
    rope_tables_1d(maxR, 128, theta, cos_h.data(), sin_h.data());
    return ND_OK;
  }

  int prepare() override {
    cudaStream_t s = dev->stream;
    // the GEMM epilogue's norm weight per 128-column head: the layer's q_norm
    // for the H query heads, k_norm for the KV key heads
    for (int l = 0; l < NB; ++l)
      for (int h = 0; h < H + KV; ++h)
        ND_CUDA(cudaMemcpyAsync(sets + (static_cast<int64_t>(l) * (H + KV) + h) * 128,
                                (h < H ? qn : kn) + static_cast<int64_t>(l) * 128, 128 * 4,
                                cudaMemcpyDeviceToDevice, s));
    ND_CUDA(cudaMemcpyAsync(cos_d, cos_h.data(), cos_h.size() * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaMemcpyAsync(sin_d, sin_h.data(), sin_h.size() * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaStreamSynchronize(s));
    return ND_OK;
  }

  int encode(const int32_t* ids, int n, const float* src, int src_rows, int fn, float* out) override {
    if (src || src_rows) return fail(ND_ERR_INVALID, "qwen3: takes no source rows");
    final_norm = fn != 0;
    return run(ids, n, out);
  }

  int forward(cudaStream_t s) override {
    const double r = rows;
    ND_OP("embed", 0.0, embed(s, emb));
    for (int l = 0; l < NB; ++l) {
      ND_OP("rmsnorm", 0.0, rms(s, x, xn, lt, static_cast<int64_t>(W) * pw, ln1 + static_cast<int64_t>(l) * W));
      {
        nd_linear_args a{};
        a.dtype = lt;
        a.epilogue = ND_EPI_QK_NORM_ROPE;
        a.rows = rows;
        a.in_features = W;
        a.out_features = QKV;
        a.x = xn;
        a.ldx = static_cast<int64_t>(W) * pw;
        weight_args(a, qkv_w, static_cast<int64_t>(l) * QKV);
        a.group_split = rows;
        a.y = qkv;
        a.ldy = QKV;
        a.qk_norm = sets + static_cast<int64_t>(l) * (H + KV) * 128;
        a.norm_span = 128;
        a.rope_cos = cos_d;
        a.rope_sin = sin_d;
        a.qk_cols = QW + KW;
        a.eps = eps;
        ND_OP("gemm.qkv", 2.0 * r * QKV * W, linear(a, s));
      }
      {
        nd_attention_args a{};
        a.dtype = dt;
        a.out_dtype = f32 ? ND_BF16X2 : 0;
        a.heads = H;
        a.kv_heads = KV;
        a.head_dim = 128;
        a.batch = 1;
        a.q_rows = rows;
        a.kv_rows = rows;
        a.causal = 1;
        uint8_t* base = static_cast<uint8_t*>(qkv);
        a.q = base;
        a.k = base + static_cast<size_t>(QW) * qe;
        a.v = base + static_cast<size_t>(QW + KW) * qe;
        a.ldq = a.ldk = a.ldv = QKV;
        a.out = att;
        a.ldo = static_cast<int64_t>(QW) * pw;
        ND_OP("attention", 2.0 * r * r * QW, attention(a, s));
      }
      ND_OP("gemm.out", 2.0 * r * W * QW,
            lin(s, att, rows, QW, o_w, static_cast<int64_t>(l) * W, W, ND_EPI_RESIDUAL_ADD, nullptr, 0, x));
      ND_OP("rmsnorm", 0.0, rms(s, x, xn, lt, static_cast<int64_t>(W) * pw, ln2 + static_cast<int64_t>(l) * W));
      ND_OP("gemm.up", 4.0 * r * F * W,
            lin(s, xn, rows, W, gu_w, static_cast<int64_t>(l) * 2 * F, F, ND_EPI_SWIGLU, hid, F));
      ND_OP("gemm.down", 2.0 * r * W * F,
            lin(s, hid, rows, F, down_w, static_cast<int64_t>(l) * W, W, ND_EPI_RESIDUAL_ADD, nullptr, 0, x));
    }
    if (final_norm) {
      ND_OP("rmsnorm", 0.0, rms(s, x, out_d, ND_F32, W, fnorm));
    } else {
      ND_CUDA(cudaMemcpyAsync(out_d, x, static_cast<size_t>(rows) * W * 4, cudaMemcpyDeviceToDevice, s));
    }
    return ND_OK;
  }
};

// ------------------------------------------------------------ LLM adapter
struct LlmAdapter final : TextTower {
  int maxS = 0, srows = 0;
  Mat emb, sqkv_w, so_w, cq_w, ckv_w, co_w, m0_w, m2_w, out_w;
  float *nsa = nullptr, *nca = nullptr, *nml = nullptr, *sqn = nullptr, *skn = nullptr, *cqn = nullptr,
        *ckn = nullptr, *m0_b = nullptr, *m2_b = nullptr, *out_b = nullptr, *fnorm = nullptr;
  float *src32 = nullptr, *y32 = nullptr;
  void *xn = nullptr, *qkv = nullptr, *qc = nullptr, *kvc = nullptr, *att = nullptr, *hid = nullptr,
       *srcn = nullptr;

  int build() override {
    ND_TRY_RC(common_build("llm adapter"));
    const nd_model_desc& d = desc;
    HD = d.head_dim > 0 ? d.head_dim : 64;
    if ((HD != 64 && HD != 128) || H * HD != W) return fail(ND_ERR_INVALID, "llm adapter: heads x head_dim (64 or 128) must be the width");
    if (f32) return fail(ND_ERR_UNSUPPORTED, "llm adapter: compute must be bf16 or f16");
    maxS = d.source_rows;
    if (maxS <= 0) return fail(ND_ERR_INVALID, "llm adapter: source_rows must be positive");
    theta = d.rope_theta > 0 ? d.rope_theta : 1e4;
    auto Vv = [&](int64_t n) { return static_cast<float*>(alloc(static_cast<size_t>(n) * 4, true)); };
    const int64_t WW = static_cast<int64_t>(W);
    emb = alloc_mat(V, W, V);
    sqkv_w = alloc_mat(NB * 3 * WW, W, W);
    so_w = alloc_mat(NB * WW, W, W);
    cq_w = alloc_mat(NB * WW, W, W);
    ckv_w = alloc_mat(NB * 2 * WW, W, W);
    co_w = alloc_mat(NB * WW, W, W);
    m0_w = alloc_mat(static_cast<int64_t>(NB) * F, W, F);
    m2_w = alloc_mat(NB * WW, F, W);
    out_w = alloc_mat(WW, W, W);
    nsa = Vv(NB * WW);
    nca = Vv(NB * WW);
    nml = Vv(NB * WW);
    sqn = Vv(static_cast<int64_t>(NB) * HD);
    skn = Vv(static_cast<int64_t>(NB) * HD);
    cqn = Vv(static_cast<int64_t>(NB) * HD);
    ckn = Vv(static_cast<int64_t>(NB) * HD);
    m0_b = Vv(static_cast<int64_t>(NB) * F);
    m2_b = Vv(NB * WW);
    out_b = Vv(WW);
    fnorm = Vv(WW);
    auto S = [&](size_t b) { return alloc(b, false); };
    const int tr = std::max(maxR, maxS);
    ids_d = static_cast<int32_t*>(S(static_cast<size_t>(maxR) * 4));
    x = static_cast<float*>(S(static_cast<size_t>(maxR) * W * 4));
    out_d = static_cast<float*>(S(static_cast<size_t>(maxR) * W * 4));
    y32 = static_cast<float*>(S(static_cast<size_t>(maxR) * W * 4));
    src32 = static_cast<float*>(S(static_cast<size_t>(maxS) * W * 4));
    cos_d = static_cast<float*>(S(static_cast<size_t>(tr) * (HD / 2) * 4));
    sin_d = static_cast<float*>(S(static_cast<size_t>(tr) * (HD / 2) * 4));
    xn = S(static_cast<size_t>(maxR) * W * 2);
    qkv = S(static_cast<size_t>(maxR) * 3 * W * 2);
    qc = S(static_cast<size_t>(maxR) * W * 2);
    kvc = S(static_cast<size_t>(maxS) * 2 * W * 2);
    att = S(static_cast<size_t>(maxR) * W * 2);
    hid = S(static_cast<size_t>(maxR) * F * 2);
    srcn = S(static_cast<size_t>(maxS) * W * 2);
    if (alloc_failed) return fail(ND_ERR_OOM, "llm adapter: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));
    auto M_ = [&](const std::string& n, const Mat& m, int64_t row, int64_t r) {
      add_slot(n, kMatrix, r, m.cols, m.at(row, 2));
    };
    M_("embed.weight", emb, 0, V);
    M_("out_proj.weight", out_w, 0, W);
    add_slot("out_proj.bias", kVector, W, 1, out_b, false);
    add_slot("norm.weight", kVector, W, 1, fnorm);
    for (int b = 0; b < NB; ++b) {
      const std::string p = "blocks." + std::to_string(b) + ".";
      const int64_t bw = b * WW;
      add_slot(p + "norm_self_attn.weight", kVector, W, 1, nsa + bw);
      add_slot(p + "norm_cross_attn.weight", kVector, W, 1, nca + bw);
      add_slot(p + "norm_mlp.weight", kVector, W, 1, nml + bw);
      M_(p + "self_attn.q_proj.weight", sqkv_w, 3 * bw, W);
      M_(p + "self_attn.k_proj.weight", sqkv_w, 3 * bw + W, W);
      M_(p + "self_attn.v_proj.weight", sqkv_w, 3 * bw + 2 * W, W);
      M_(p + "self_attn.o_proj.weight", so_w, bw, W);
      add_slot(p + "self_attn.q_norm.weight", kVector, HD, 1, sqn + static_cast<int64_t>(b) * HD);
      add_slot(p + "self_attn.k_norm.weight", kVector, HD, 1, skn + static_cast<int64_t>(b) * HD);
      M_(p + "cross_attn.q_proj.weight", cq_w, bw, W);
      M_(p + "cross_attn.k_proj.weight", ckv_w, 2 * bw, W);
      M_(p + "cross_attn.v_proj.weight", ckv_w, 2 * bw + W, W);
      M_(p + "cross_attn.o_proj.weight", co_w, bw, W);
      add_slot(p + "cross_attn.q_norm.weight", kVector, HD, 1, cqn + static_cast<int64_t>(b) * HD);
      add_slot(p + "cross_attn.k_norm.weight", kVector, HD, 1, ckn + static_cast<int64_t>(b) * HD);
      M_(p + "mlp.0.weight", m0_w, static_cast<int64_t>(b) * F, F);
      add_slot(p + "mlp.0.bias", kVector, F, 1, m0_b + static_cast<int64_t>(b) * F, false);
      M_(p + "mlp.2.weight", m2_w, bw, W);
      add_slot(p + "mlp.2.bias", kVector, W, 1, m2_b + bw, false);
    }
    cos_h.resize(static_cast<size_t>(tr) * (HD / 2));
    sin_h.resize(static_cast<size_t>(tr) * (HD / 2));
    rope_tables_1d(tr, HD, theta, cos_h.data(), sin_h.data());
    srows = 1;
    return ND_OK;
  }

  int prepare() override {
    cudaStream_t s = dev->stream;
    ND_CUDA(cudaMemcpyAsync(cos_d, cos_h.data(), cos_h.size() * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaMemcpyAsync(sin_d, sin_h.data(), sin_h.size() * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaStreamSynchronize(s));
    return ND_OK;
  }

  int encode(const int32_t* ids, int n, const float* src, int src_rows, int, float* out) override {
    if (!src || src_rows <= 0 || src_rows > maxS)
      return fail(ND_ERR_INVALID, "llm adapter: needs 1.." + std::to_string(maxS) + " source rows");
    srows = src_rows;
    ND_CUDA(cudaMemcpyAsync(src32, src, static_cast<size_t>(src_rows) * W * 4, cudaMemcpyHostToDevice, dev->stream));
    return run(ids, n, out);
  }

  int head_norm(cudaStream_t s, void* t, int64_t ld, int r, const float* w) {
    const long long warps = static_cast<long long>(r) * H;
    const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
    if (HD == 64)
      head_norm_rope_kernel<64><<<grid, 256, 0, s>>>(t, dt, ld, r, H, w, cos_d, sin_d, eps);
    else
      head_norm_rope_kernel<128><<<grid, 256, 0, s>>>(t, dt, ld, r, H, w, cos_d, sin_d, eps);
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }

  int attend(cudaStream_t s, const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int kv_rows) {
    nd_attention_args a{};
    a.dtype = dt;
    a.heads = H;
    a.head_dim = HD;
    a.batch = 1;
    a.q_rows = rows;
    a.kv_rows = kv_rows;
    a.q = q;
    a.ldq = ldq;
    a.k = k;
    a.v = v;
    a.ldk = a.ldv = ldkv;
    a.out = att;
    a.ldo = W;
    return attention(a, s);
  }

  int forward(cudaStream_t s) override {
    const double r = rows, sr = srows;
    const int64_t WW = W;
    ND_OP("embed", 0.0, embed(s, emb));
    // the Qwen3 rows in the compute type, for the cross-attention's keys / values
    ND_OP("embed", 0.0, convert(src32, ND_F32, srcn, dt, static_cast<int64_t>(srows) * W, s));
    for (int b = 0; b < NB; ++b) {
      const int64_t bw = b * WW;
      // self-attention over the T5 sequence, unmasked
      ND_OP("rmsnorm", 0.0, rms(s, x, xn, dt, W, nsa + bw));
      ND_OP("gemm.qkv", 2.0 * r * 3 * W * W, lin(s, xn, rows, W, sqkv_w, 3 * bw, 3 * WW, ND_EPI_STORE, qkv, 3 * WW));
      ND_OP("headnorm", 0.0, head_norm(s, qkv, 3 * WW, rows, sqn + static_cast<int64_t>(b) * HD));
      ND_OP("headnorm", 0.0, head_norm(s, static_cast<uint16_t*>(qkv) + W, 3 * WW, rows, skn + static_cast<int64_t>(b) * HD));
      ND_OP("attention", 4.0 * r * r * W,
            attend(s, qkv, 3 * WW, static_cast<uint16_t*>(qkv) + W, static_cast<uint16_t*>(qkv) + 2 * W, 3 * WW, rows));
      ND_OP("gemm.out", 2.0 * r * W * W, lin(s, att, rows, W, so_w, bw, W, ND_EPI_RESIDUAL_ADD, nullptr, 0, x));
      // cross-attention into the Qwen3 rows, keys placed by their own positions
      ND_OP("rmsnorm", 0.0, rms(s, x, xn, dt, W, nca + bw));
      ND_OP("gemm.qkv", 2.0 * r * W * W, lin(s, xn, rows, W, cq_w, bw, W, ND_EPI_STORE, qc, W));
      ND_OP("gemm.qkv", 2.0 * sr * 2 * W * W, lin(s, srcn, srows, W, ckv_w, 2 * bw, 2 * WW, ND_EPI_STORE, kvc, 2 * WW));
      ND_OP("headnorm", 0.0, head_norm(s, qc, W, rows, cqn + static_cast<int64_t>(b) * HD));
      ND_OP("headnorm", 0.0, head_norm(s, kvc, 2 * WW, srows, ckn + static_cast<int64_t>(b) * HD));
      ND_OP("attention", 4.0 * r * sr * W, attend(s, qc, W, kvc, static_cast<uint16_t*>(kvc) + W, 2 * WW, srows));
      ND_OP("gemm.out", 2.0 * r * W * W, lin(s, att, rows, W, co_w, bw, W, ND_EPI_RESIDUAL_ADD, nullptr, 0, x));
      // GELU MLP
      ND_OP("rmsnorm", 0.0, rms(s, x, xn, dt, W, nml + bw));
      ND_OP("gemm.up", 2.0 * r * F * W,
            lin(s, xn, rows, W, m0_w, static_cast<int64_t>(b) * F, F, ND_EPI_GELU_ERF, hid, F, nullptr,
                m0_b + static_cast<int64_t>(b) * F));
      ND_OP("gemm.down", 2.0 * r * W * F,
            lin(s, hid, rows, F, m2_w, bw, W, ND_EPI_RESIDUAL_ADD, nullptr, 0, x, m2_b + bw));
    }
    // out_proj + bias, then the final norm
    ND_OP("embed", 0.0, convert(x, ND_F32, xn, dt, static_cast<int64_t>(rows) * W, s));
    ND_OP("gemm.out", 2.0 * r * W * W, lin(s, xn, rows, W, out_w, 0, W, ND_EPI_STORE_F32, nullptr, 0, y32, out_b));
    ND_OP("rmsnorm", 0.0, rms(s, y32, out_d, ND_F32, W, fnorm));
    return ND_OK;
  }
};

#undef ND_OP

}  // namespace

nd_denoiser* make_qwen3_text() { return new Qwen3Text(); }
nd_denoiser* make_llm_adapter() { return new LlmAdapter(); }

int head_norm_rope(void* x, int dtype, int64_t ld, int64_t rows, int heads, int head_dim, const float* weight,
                   const float* cos, const float* sin, float eps, cudaStream_t s) {
  if (dtype != ND_F32 && dtype != ND_F16 && dtype != ND_BF16) return fail(ND_ERR_INVALID, "head_norm_rope: dtype");
  if (head_dim != 64 && head_dim != 128) return fail(ND_ERR_UNSUPPORTED, "head_norm_rope: head_dim must be 64 or 128");
  if (!x || !weight || rows <= 0 || heads <= 0 || ld < static_cast<int64_t>(heads) * head_dim)
    return fail(ND_ERR_INVALID, "head_norm_rope: bad arguments");
  if ((cos == nullptr) != (sin == nullptr)) return fail(ND_ERR_INVALID, "head_norm_rope: give both cos and sin");
  const long long threads = rows * heads * 32;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  if (head_dim == 64)
    head_norm_rope_kernel<64><<<grid, 256, 0, s>>>(x, dtype, ld, static_cast<int>(rows), heads, weight, cos, sin, eps);
  else
    head_norm_rope_kernel<128><<<grid, 256, 0, s>>>(x, dtype, ld, static_cast<int>(rows), heads, weight, cos, sin, eps);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd

extern "C" int nd_op_head_norm_rope(void* x, int dtype, int64_t ld, int64_t rows, int heads, int head_dim,
                                    const float* weight, const float* cos, const float* sin, float eps,
                                    void* stream) {
  return nd::head_norm_rope(x, dtype, ld, rows, heads, head_dim, weight, cos, sin, eps,
                            static_cast<cudaStream_t>(stream));
}
