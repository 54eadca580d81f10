// The Anima (Cosmos-Predict2 2B) DiT denoiser step: AnimaDit
// (Models/Anima/AnimaDit.cs) on the library's kernels.
//
// Per step (AnimaDit.Build, :360-404): 2x2 patches -> x_embedder (the first
// 64 of its 68 columns: the padding-mask channel is zero, :250-260);
// sinusoid(sigma, width) -> RMSNorm = temb, and Linear-SiLU-Linear = the
// shared adaLN term `lora` [3D]; then the blocks; then the final layer
// LN x (1 + scale) + shift -> Linear -> unpatchify.
// Per block (AnimaDit.Block, :295-358), every residual gated in fp32:
//   self-attention   Modulate -> fused QKV GEMM with head RMSNorm + 3-D RoPE
//                    in the epilogue -> flash attention -> gated out GEMM
//   cross-attention  Modulate -> Q GEMM (+ head norm) ; K|V GEMM over the text
//                    context (+ head norm on K) -> attention -> gated out GEMM
//   MLP              Modulate -> exact-GELU GEMM -> gated down GEMM
// The low-rank adaLN of every block (Modulation, :270-291) is one GEMV over
// all blocks' first factors and one grouped GEMV per block for the second.
// Batch items (CFG branches) are stacked by rows; they share the timestep.
#include <cmath>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_runtime.h"

namespace nd {

namespace {

// AnimaDit.RopeTables (Models/Anima/AnimaDit.cs:149-188): 22 still temporal
// pairs (a single frame), then 21 row and 21 column pairs at the NTK-scaled
// spatial base 10000 * 4^(42/40), frequencies in float.
void anima_rope_tables(int rows, int columns, int head_dim, float* cos, float* sin) {
  const int spatial = head_dim / 6 * 2;
  const int temporal = head_dim - 2 * spatial;
  const int pairs = head_dim / 2;
  const double ntk = std::pow(4.0, spatial / static_cast<double>(spatial - 2));
  const float theta = static_cast<float>(10000.0 * ntk);
  std::vector<float> sf(spatial / 2);
  for (int k = 0; k < spatial / 2; ++k) sf[k] = 1.0f / std::pow(theta, 2.0f * k / spatial);
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < columns; ++j) {
      const int64_t off = static_cast<int64_t>(i * columns + j) * pairs;
      for (int d = 0; d < temporal / 2; ++d) {
        cos[off + d] = 1.f;
        sin[off + d] = 0.f;
      }
      for (int k = 0; k < spatial / 2; ++k) {
        const float ra = i * sf[k], ca = j * sf[k];
        cos[off + temporal / 2 + k] = std::cos(ra);
        sin[off + temporal / 2 + k] = std::sin(ra);
        cos[off + temporal / 2 + spatial / 2 + k] = std::cos(ca);
        sin[off + temporal / 2 + spatial / 2 + k] = std::sin(ca);
      }
    }
}

// Transformer.Sinusoid (Graph/Transformer.cs:20-32) of the level itself
// (AnimaDit.Predict, :124-134: Cosmos embeds sigma as it is).
void sinusoid(double sigma, int width, float* out) {
  const float time = static_cast<float>(sigma);
  const int half = width / 2;
  for (int i = 0; i < half; ++i) {
    const float frequency = std::exp(-std::log(10000.0f) * i / half);
    const float angle = time * frequency;
    out[i] = std::cos(angle);
    out[half + i] = std::sin(angle);
  }
}

constexpr int kLatentChannels = 16;
constexpr int kEmbedCols = 68;  // (16 latent + 1 padding-mask channel) x 2 x 2

struct Anima final : nd_denoiser {
  int D = 0, H = 0, F = 0, NB = 0, R = 0, ctx = 0, cw = 0, Hl = 0, Wl = 0, P = 2, B = 1;
  int T = 0, cin = 0;
  int dt = ND_BF16;
  // fp32 compute: GEMM operands as bf16 hi|lo pairs (lt = ND_BF16X2, pair
  // buffers twice as wide), Q/K/V and the attention in fp32.
  bool f32 = false;
  int lt = ND_BF16;
  int pw = 1;      // columns per logical column in GEMM-operand buffers (2: pairs)
  size_t qe = 2;   // bytes per element of the Q/K/V buffers
  float eps = 1e-6f;
  Mat x_emb, t1, t2, mod1, mod2, sqkv, so, cq, ckv, co, fc1, fc2, fmod1, fmod2, flin;
  float *t_norm = nullptr, *snorm = nullptr, *cqnorm = nullptr, *cknorm = nullptr;
  // inputs
  float *in_latent = nullptr, *in_ctx = nullptr, *in_tsin = nullptr, *in_cos = nullptr, *in_sin = nullptr;
  std::vector<float> def_cos, def_sin;
  bool default_rope = true;
  float* tsin = nullptr;  // pinned
  // scratch
  float *x = nullptr, *temb = nullptr, *th = nullptr, *lora = nullptr, *h1 = nullptr, *mods = nullptr;
  float *fh = nullptr, *fmod = nullptr, *out_tok = nullptr, *out_latent = nullptr;
  void *xn = nullptr, *qkv = nullptr, *attn = nullptr, *cqb = nullptr, *kvb = nullptr, *ctxb = nullptr;
  void *hid = nullptr, *tok_in = nullptr;

  int build() override {
    const nd_model_desc& d = desc;
    if (d.compute != ND_BF16 && d.compute != ND_F16 && d.compute != ND_F32)
      return fail(ND_ERR_UNSUPPORTED, "anima: compute must be bf16, f16 or f32");
    if (d.weight_dtype != d.compute && !(d.weight_dtype == ND_I8 && d.compute != ND_F32))
      return fail(ND_ERR_UNSUPPORTED, "anima: weights must be stored in the compute dtype (or int8 with 16-bit compute)");
    if (d.weight_dtype == ND_I8 && d.quant_scale_dtype != ND_F16 && d.quant_scale_dtype != ND_F32)
      return fail(ND_ERR_INVALID, "anima: int8 weights need quant_scale_dtype ND_F16 or ND_F32");
    if (d.head_dim != 128 || d.heads * 128 != d.width) return fail(ND_ERR_INVALID, "anima: width must be heads x 128");
    if (d.blocks <= 0 || d.mlp_width <= 0 || d.mlp_width % 8) return fail(ND_ERR_INVALID, "anima: bad blocks / mlp_width");
    if (d.adaln_rank <= 0 || d.adaln_rank % 16) return fail(ND_ERR_INVALID, "anima: adaln_rank must be a positive multiple of 16");
    if (d.context_rows <= 0 || d.context_width <= 0 || d.context_width % 16)
      return fail(ND_ERR_INVALID, "anima: context width must be a multiple of 16");
    if (d.latent_channels != kLatentChannels || d.patch != 2)
      return fail(ND_ERR_INVALID, "anima: latent must have 16 channels in 2x2 patches");
    if (d.latent_height % 2 || d.latent_width % 2) return fail(ND_ERR_INVALID, "anima: latent does not divide into patches");
    if (d.batch < 1 || d.batch > 4) return fail(ND_ERR_INVALID, "anima: batch must be 1..4");
    if (d.time_width != 0 && d.time_width != d.width) return fail(ND_ERR_INVALID, "anima: time_width is the width");
    dt = d.compute;
    f32 = dt == ND_F32;
    lt = f32 ? ND_BF16X2 : dt;
    pw = f32 ? 2 : 1;
    qe = f32 ? 4 : 2;
    D = d.width;
    H = d.heads;
    F = d.mlp_width;
    NB = d.blocks;
    R = d.adaln_rank;
    ctx = d.context_rows;
    cw = d.context_width;
    Hl = d.latent_height;
    Wl = d.latent_width;
    B = d.batch;
    T = (Hl / P) * (Wl / P);
    cin = kLatentChannels * P * P;
    eps = d.eps > 0 ? d.eps : 1e-6f;
    const int64_t M = static_cast<int64_t>(B) * T;

    auto V = [&](int64_t n) { return static_cast<float*>(alloc(static_cast<size_t>(n) * 4, true)); };
    x_emb = alloc_mat(D, cin, D);
    t1 = alloc_mat(D, D, D);
    t2 = alloc_mat(3LL * D, D, 3LL * D);
    t_norm = V(D);
    mod1 = alloc_mat(static_cast<int64_t>(NB) * 3 * R, D, R);
    mod2 = alloc_mat(static_cast<int64_t>(NB) * 3 * 3 * D, R, 3LL * D);
    sqkv = alloc_mat(static_cast<int64_t>(NB) * 3 * D, D, D);
    so = alloc_mat(static_cast<int64_t>(NB) * D, D, D);
    snorm = V(static_cast<int64_t>(NB) * 2 * 128);
    cq = alloc_mat(static_cast<int64_t>(NB) * D, D, D);
    ckv = alloc_mat(static_cast<int64_t>(NB) * 2 * D, cw, D);
    co = alloc_mat(static_cast<int64_t>(NB) * D, D, D);
    cqnorm = V(static_cast<int64_t>(NB) * 128);
    cknorm = V(static_cast<int64_t>(NB) * 128);
    fc1 = alloc_mat(static_cast<int64_t>(NB) * F, D, F);
    fc2 = alloc_mat(static_cast<int64_t>(NB) * D, F, D);
    fmod1 = alloc_mat(R, D, R);
    fmod2 = alloc_mat(2LL * D, R, 2LL * D);
    flin = alloc_mat(cin, D, cin);

    auto S = [&](size_t bytes) { return alloc(bytes, false); };
    const size_t e = 2;
    in_latent = static_cast<float*>(S(static_cast<size_t>(B) * kLatentChannels * Hl * Wl * 4));
    in_ctx = static_cast<float*>(S(static_cast<size_t>(B) * ctx * cw * 4));
    in_tsin = static_cast<float*>(S(static_cast<size_t>(D) * 4));
    in_cos = static_cast<float*>(S(static_cast<size_t>(T) * 64 * 4));
    in_sin = static_cast<float*>(S(static_cast<size_t>(T) * 64 * 4));
    x = static_cast<float*>(S(static_cast<size_t>(M) * D * 4));
    temb = static_cast<float*>(S(static_cast<size_t>(D) * 4));
    th = static_cast<float*>(S(static_cast<size_t>(D) * 4));
    lora = static_cast<float*>(S(static_cast<size_t>(3) * D * 4));
    h1 = static_cast<float*>(S(static_cast<size_t>(NB) * 3 * R * 4));
    mods = static_cast<float*>(S(static_cast<size_t>(NB) * 9 * D * 4));
    fh = static_cast<float*>(S(static_cast<size_t>(R) * 4));
    fmod = static_cast<float*>(S(static_cast<size_t>(2) * D * 4));
    out_tok = static_cast<float*>(S(static_cast<size_t>(M) * cin * 4));
    out_latent = static_cast<float*>(S(static_cast<size_t>(B) * kLatentChannels * Hl * Wl * 4));
    xn = S(static_cast<size_t>(M) * D * e * pw);
    qkv = S(static_cast<size_t>(M) * 3 * D * qe);
    attn = S(static_cast<size_t>(M) * D * e * pw);
    cqb = S(static_cast<size_t>(M) * D * qe);
    kvb = S(static_cast<size_t>(B) * ctx * 2 * D * qe);
    ctxb = S(static_cast<size_t>(B) * ctx * cw * e * pw);
    hid = S(static_cast<size_t>(M) * F * e * pw);
    tok_in = S(static_cast<size_t>(M) * cin * e * pw);
    tsin = static_cast<float*>(pinned(static_cast<size_t>(D) * 4));
    if (desc.compute != ND_F32) alloc_attn_workspace(128);
    if (alloc_failed) return fail(ND_ERR_OOM, "anima: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));

    // ---- registry (Anima / Cosmos-Predict2 tensor names)
    auto M_ = [&](const std::string& name, const Mat& m, int64_t row, int64_t rows) {
      const int64_t sc = m.q8 ? m.cols / qgroup(m.cols) : 0;
      add_slot(name, kMatrix, rows, m.cols, m.at(row, 2), true, m.q8 ? m.scales_at(row, sc, qf16()) : nullptr);
    };
    M_("x_embedder.proj.1.weight", x_emb, 0, D);
    slots.back().src_cols = kEmbedCols;
    M_("t_embedder.1.linear_1.weight", t1, 0, D);
    M_("t_embedder.1.linear_2.weight", t2, 0, 3LL * D);
    add_slot("t_embedding_norm.weight", kVector, D, 1, t_norm);
    const char* subs[3] = {"adaln_modulation_self_attn", "adaln_modulation_cross_attn", "adaln_modulation_mlp"};
    for (int b = 0; b < NB; ++b) {
      const std::string p = "blocks." + std::to_string(b) + ".";
      for (int j = 0; j < 3; ++j) {
        M_(p + subs[j] + ".1.weight", mod1, (static_cast<int64_t>(b) * 3 + j) * R, R);
        M_(p + subs[j] + ".2.weight", mod2, (static_cast<int64_t>(b) * 3 + j) * 3 * D, 3LL * D);
      }
      const int64_t bD = static_cast<int64_t>(b) * D;
      M_(p + "self_attn.q_proj.weight", sqkv, 3 * bD, D);
      M_(p + "self_attn.k_proj.weight", sqkv, 3 * bD + D, D);
      M_(p + "self_attn.v_proj.weight", sqkv, 3 * bD + 2 * D, D);
      M_(p + "self_attn.output_proj.weight", so, bD, D);
      add_slot(p + "self_attn.q_norm.weight", kVector, 128, 1, snorm + b * 256);
      add_slot(p + "self_attn.k_norm.weight", kVector, 128, 1, snorm + b * 256 + 128);
      M_(p + "cross_attn.q_proj.weight", cq, bD, D);
      M_(p + "cross_attn.k_proj.weight", ckv, 2 * bD, D);
      M_(p + "cross_attn.v_proj.weight", ckv, 2 * bD + D, D);
      M_(p + "cross_attn.output_proj.weight", co, bD, D);
      add_slot(p + "cross_attn.q_norm.weight", kVector, 128, 1, cqnorm + b * 128);
      add_slot(p + "cross_attn.k_norm.weight", kVector, 128, 1, cknorm + b * 128);
      M_(p + "mlp.layer1.weight", fc1, static_cast<int64_t>(b) * F, F);
      M_(p + "mlp.layer2.weight", fc2, bD, D);
    }
    M_("final_layer.adaln_modulation.1.weight", fmod1, 0, R);
    M_("final_layer.adaln_modulation.2.weight", fmod2, 0, 2LL * D);
    M_("final_layer.linear.weight", flin, 0, cin);

    def_cos.resize(static_cast<size_t>(T) * 64);
    def_sin.resize(static_cast<size_t>(T) * 64);
    anima_rope_tables(Hl / P, Wl / P, 128, def_cos.data(), def_sin.data());
    return ND_OK;
  }

  int prepare() override {
    cudaStream_t s = dev->stream;
    ND_CUDA(cudaMemcpyAsync(in_cos, def_cos.data(), def_cos.size() * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaMemcpyAsync(in_sin, def_sin.data(), def_sin.size() * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaStreamSynchronize(s));
    default_rope = true;
    return ND_OK;
  }

  int64_t latent_elems() const override { return static_cast<int64_t>(B) * kLatentChannels * Hl * Wl; }
  const float* output() const override { return out_latent; }

  int check_cond(int n, const nd_named_tensor* cond, StepInputs& in) override {
    for (int i = 0; i < n; ++i) {
      const nd_named_tensor& t = cond[i];
      if (!t.name || !t.data) return fail(ND_ERR_INVALID, "predict: conditioning entry without name or data");
      int64_t elems = 1;
      for (int r = 0; r < t.rank; ++r) elems *= t.shape[r];
      const std::string name = t.name;
      if (name == "context") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(B) * ctx * cw)
          return fail(ND_ERR_INVALID, "predict: context must be f32 [" + std::to_string(B) + ", " +
                                          std::to_string(ctx) + ", " + std::to_string(cw) + "]");
        in.context = static_cast<const float*>(t.data);
      } else if (name == "cos" || name == "sin") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(T) * 64)
          return fail(ND_ERR_INVALID, "predict: " + name + " must be f32 [" + std::to_string(T) + ", 64]");
        (name == "cos" ? in.cos : in.sin) = static_cast<const float*>(t.data);
      } else {
        return fail(ND_ERR_INVALID, "predict: unknown conditioning " + name);
      }
    }
    if (!in.context) return fail(ND_ERR_INVALID, "predict: conditioning needs \"context\"");
    if ((in.cos == nullptr) != (in.sin == nullptr)) return fail(ND_ERR_INVALID, "predict: give both cos and sin");
    return ND_OK;
  }

  int stage(const StepInputs& in, cudaStream_t s) override {
    const cudaMemcpyKind k = in.device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    ND_CUDA(cudaMemcpyAsync(in_latent, in.latent, static_cast<size_t>(latent_elems()) * 4, k, s));
    ND_CUDA(cudaMemcpyAsync(in_ctx, in.context, static_cast<size_t>(B) * ctx * cw * 4, k, s));
    ND_CUDA(cudaEventSynchronize(staged));
    sinusoid(in.sigma, D, tsin);
    ND_CUDA(cudaMemcpyAsync(in_tsin, tsin, static_cast<size_t>(D) * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaEventRecord(staged, s));
    if (in.cos) {
      ND_CUDA(cudaMemcpyAsync(in_cos, in.cos, static_cast<size_t>(T) * 64 * 4, k, s));
      ND_CUDA(cudaMemcpyAsync(in_sin, in.sin, static_cast<size_t>(T) * 64 * 4, k, s));
      default_rope = false;
    } else if (!default_rope) {
      ND_CUDA(cudaMemcpyAsync(in_cos, def_cos.data(), def_cos.size() * 4, cudaMemcpyHostToDevice, s));
      ND_CUDA(cudaMemcpyAsync(in_sin, def_sin.data(), def_sin.size() * 4, cudaMemcpyHostToDevice, s));
      default_rope = true;
    }
    return ND_OK;
  }

  void weight_args(nd_linear_args& a, const Mat& m, int64_t row) const {
    a.weight = m.at(row, 2);
    if (m.q8) {
      a.weight_dtype = ND_I8;
      a.scales = m.scales_at(row, m.cols / qgroup(m.cols), qf16());
      a.scale_dtype = desc.quant_scale_dtype;
      a.quant_group = desc.quant_group;
    }
  }

  nd_linear_args lin_args(const void* xin, int64_t rows, int64_t k, const Mat& w, int64_t wrow, int64_t n,
                          int epi) const {
    nd_linear_args a{};
    a.dtype = lt;
    a.epilogue = epi;
    a.rows = rows;
    a.in_features = k;
    a.out_features = n;
    a.x = xin;
    a.ldx = k * pw;
    weight_args(a, w, wrow);
    a.group_split = rows;
    a.eps = eps;
    return a;
  }

  int gv(cudaStream_t s, const Mat& w, int64_t row, int64_t n, int64_t k, const float* xin, bool pre_silu,
         int act, float* y, int64_t x_rows_per_vec = 0, const float* bias = nullptr, int64_t bias_period = 0) {
    nd_gemv_args g{};
    g.w = w.at(row, 2);
    g.w_dtype = w.q8 ? ND_I8 : lt;
    g.n = n;
    g.k = k;
    g.x = xin;
    g.batch = 1;
    g.pre_silu = pre_silu ? 1 : 0;
    g.act = act;
    g.y = y;
    g.bias = bias;
    g.bias_period = bias_period;
    g.x_rows_per_vec = x_rows_per_vec;
    if (w.q8) {
      g.scales = w.scales_at(row, w.cols / qgroup(w.cols), qf16());
      g.scale_dtype = desc.quant_scale_dtype;
      g.quant_group = desc.quant_group;
    }
    return gemv(g, s);
  }

  int mod(cudaStream_t s, const float* shift, const float* scale, int64_t rows) {
    nd_modulate_args m{};
    m.x = x;
    m.ldx = D;
    m.y = xn;
    m.ldy = static_cast<int64_t>(D) * pw;
    m.out_dtype = lt;
    m.rows = rows;
    m.width = D;
    m.shift = shift;
    m.scale = scale;
    m.vec_stride = D;
    m.group_split = rows;
    m.eps = eps;
    return modulate(m, s);
  }

  int attend(cudaStream_t s, const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv,
             int q_rows, int kv_rows) {
    nd_attention_args a{};
    a.dtype = dt;
    a.out_dtype = f32 ? ND_BF16X2 : 0;
    a.heads = H;
    a.head_dim = 128;
    a.batch = B;
    a.q_rows = q_rows;
    a.kv_rows = kv_rows;
    a.q = q;
    a.ldq = ldq;
    a.k = k;
    a.ldk = ldkv;
    a.v = v;
    a.ldv = ldkv;
    a.out = attn;
    a.ldo = static_cast<int64_t>(D) * pw;
    use_attn_workspace(a);
    return attention(a, s);
  }

#define ND_OP(cls, flops, bytes, expr) \
  do {                                 \
    prof_begin(s);                     \
    int rc_ = (expr);                  \
    if (rc_) return rc_;               \
    prof_end(s, cls, flops, bytes);    \
  } while (0)

  static double gf(double m, double n, double k) { return 2.0 * m * n * k; }

  int block(cudaStream_t s, int b) {
    const int64_t M = static_cast<int64_t>(B) * T;
    const int64_t bD = static_cast<int64_t>(b) * D;
    const float* mv = mods + static_cast<int64_t>(b) * 9 * D;  // self | cross | mlp, each shift scale gate
    const double mD = static_cast<double>(M) * D;
    const size_t e = qe;
    // ---- self-attention
    ND_OP("modulate", 0.0, mD * 6, mod(s, mv, mv + D, M));
    {
      nd_linear_args a = lin_args(xn, M, D, sqkv, 3 * bD, 3LL * D, ND_EPI_QK_NORM_ROPE);
      a.y = qkv;
      a.ldy = 3LL * D;
      a.qk_norm = snorm + b * 256;
      a.qk_cols = 2LL * D;
      a.norm_span = D;
      a.rope_cos = in_cos;
      a.rope_sin = in_sin;
      a.rope_period = T;
      ND_OP("gemm.qkv", gf(M, 3.0 * D, D), 0.0, linear(a, s));
    }
    ND_OP("attention", 4.0 * B * T * static_cast<double>(T) * D, 0.0,
          attend(s, qkv, 3LL * D, static_cast<uint8_t*>(qkv) + D * e, static_cast<uint8_t*>(qkv) + 2 * D * e,
                 3LL * D, T, T));
    {
      nd_linear_args a = lin_args(attn, M, D, so, bD, D, ND_EPI_RESIDUAL_GATE);
      a.residual = x;
      a.ldr = D;
      a.gate = mv + 2 * D;
      ND_OP("gemm.out", gf(M, D, D), 0.0, linear(a, s));
    }
    // ---- cross-attention to the text context
    ND_OP("modulate", 0.0, mD * 6, mod(s, mv + 3 * D, mv + 4 * D, M));
    {
      nd_linear_args a = lin_args(xn, M, D, cq, bD, D, ND_EPI_QK_NORM_ROPE);
      a.y = cqb;
      a.ldy = D;
      a.qk_norm = cqnorm + b * 128;
      a.qk_cols = D;
      a.norm_span = D;
      ND_OP("gemm.cross_q", gf(M, D, D), 0.0, linear(a, s));
    }
    {
      nd_linear_args a = lin_args(ctxb, static_cast<int64_t>(B) * ctx, cw, ckv, 2 * bD, 2LL * D, ND_EPI_QK_NORM_ROPE);
      a.y = kvb;
      a.ldy = 2LL * D;
      a.qk_norm = cknorm + b * 128;
      a.qk_cols = D;
      a.norm_span = D;
      ND_OP("gemm.cross_kv", gf(static_cast<double>(B) * ctx, 2.0 * D, cw), 0.0, linear(a, s));
    }
    ND_OP("attention", 4.0 * B * T * static_cast<double>(ctx) * D, 0.0,
          attend(s, cqb, D, kvb, static_cast<uint8_t*>(kvb) + D * e, 2LL * D, T, ctx));
    {
      nd_linear_args a = lin_args(attn, M, D, co, bD, D, ND_EPI_RESIDUAL_GATE);
      a.residual = x;
      a.ldr = D;
      a.gate = mv + 5 * D;
      ND_OP("gemm.out", gf(M, D, D), 0.0, linear(a, s));
    }
    // ---- MLP (exact GELU, DmlOps.ActivationGelu / CpuMath.Gelu)
    ND_OP("modulate", 0.0, mD * 6, mod(s, mv + 6 * D, mv + 7 * D, M));
    {
      nd_linear_args a = lin_args(xn, M, D, fc1, static_cast<int64_t>(b) * F, F, ND_EPI_GELU_ERF);
      a.y = hid;
      a.ldy = static_cast<int64_t>(F) * pw;
      ND_OP("gemm.up", gf(M, F, D), 0.0, linear(a, s));
    }
    {
      nd_linear_args a = lin_args(hid, M, F, fc2, bD, D, ND_EPI_RESIDUAL_GATE);
      a.residual = x;
      a.ldr = D;
      a.gate = mv + 8 * D;
      ND_OP("gemm.down", gf(M, D, F), 0.0, linear(a, s));
    }
    return ND_OK;
  }

  int forward(cudaStream_t s) override {
    const int64_t M = static_cast<int64_t>(B) * T;
    const double dD = D;
    ND_OP("embed", 0.0, 0.0, patchify(in_latent, tok_in, lt, B, kLatentChannels, Hl, Wl, P, cin * pw, s));
    {
      nd_linear_args a = lin_args(tok_in, M, cin, x_emb, 0, D, ND_EPI_STORE_F32);
      a.residual = x;
      a.ldr = D;
      ND_OP("embed", gf(M, D, cin), 0.0, linear(a, s));
    }
    if (f32) {
      ND_OP("embed", 0.0, 0.0, convert_cols(in_ctx, ND_F32, cw, ctxb, ND_BF16X2, static_cast<int64_t>(B) * ctx, cw, s));
    } else {
      ND_OP("embed", 0.0, 0.0, convert(in_ctx, ND_F32, ctxb, dt, static_cast<int64_t>(B) * ctx * cw, s));
    }
    // time: temb = RMSNorm(sinusoid); lora = Linear(SiLU(Linear(sinusoid)))
    {
      nd_rmsnorm_args r{};
      r.x = in_tsin;
      r.ldx = D;
      r.in_dtype = ND_F32;
      r.y = temb;
      r.ldy = D;
      r.out_dtype = ND_F32;
      r.rows = 1;
      r.width = D;
      r.weight = t_norm;
      r.eps = eps;
      ND_OP("gemv", 0.0, 0.0, rmsnorm(r, s));
    }
    ND_OP("gemv", 2.0 * dD * dD, dD * dD * 2, gv(s, t1, 0, D, D, in_tsin, false, 1, th));
    ND_OP("gemv", 6.0 * dD * dD, 3 * dD * dD * 2, gv(s, t2, 0, 3LL * D, D, th, false, 0, lora));
    // every block's low-rank adaLN: first factors in one pass, second per block
    ND_OP("gemv", 2.0 * NB * 3 * R * dD, NB * 3.0 * R * dD * 2,
          gv(s, mod1, 0, static_cast<int64_t>(NB) * 3 * R, D, temb, true, 0, h1));
    for (int b = 0; b < NB; ++b) {
      ND_OP("gemv", 2.0 * 9 * dD * R, 9.0 * dD * R * 2,
            gv(s, mod2, static_cast<int64_t>(b) * 9 * D, 9LL * D, R, h1 + static_cast<int64_t>(b) * 3 * R, false, 0,
               mods + static_cast<int64_t>(b) * 9 * D, 3LL * D, lora, 3LL * D));
    }
    for (int b = 0; b < NB; ++b) {
      int rc = block(s, b);
      if (rc) return rc;
    }
    // final layer: LN x (1 + scale) + shift -> Linear
    ND_OP("gemv", 2.0 * R * dD, R * dD * 2, gv(s, fmod1, 0, R, D, temb, true, 0, fh));
    ND_OP("gemv", 4.0 * dD * R, 2 * dD * R * 2, gv(s, fmod2, 0, 2LL * D, R, fh, false, 0, fmod, 0, lora, 0));
    ND_OP("modulate", 0.0, static_cast<double>(M) * D * 6, mod(s, fmod, fmod + D, M));
    {
      nd_linear_args a = lin_args(xn, M, D, flin, 0, cin, ND_EPI_STORE_F32);
      a.residual = out_tok;
      a.ldr = cin;
      ND_OP("embed", gf(M, cin, D), 0.0, linear(a, s));
    }
    ND_OP("embed", 0.0, 0.0, unpatchify(out_tok, cin, out_latent, B, kLatentChannels, Hl, Wl, P, s));
    return ND_OK;
  }
#undef ND_OP
};

}  // namespace

nd_denoiser* make_anima() { return new Anima(); }

}  // namespace nd
