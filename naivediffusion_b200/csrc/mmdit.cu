// The Qwen-Image-style dual-stream DiT (MMDiT) denoiser step: the benchmark
// configuration the headline number is quoted on (60 blocks x 3072, 24 heads,
// GELU-tanh MLP 12288, 16-channel latent patchified 2x2, 3584-wide text).
//
// The reference implements only the single-stream Qwen-Image 2.1
// (Models/QwenImage/QwenImageDit.cs); the dual-stream block here is composed
// from the same primitives in the same order (QwenImageDit.Block,
// :309-425): per stream Modulate -> Q/K/V with head RMSNorm -> rotate-half
// RoPE over the joint sequence -> joint attention -> gated residual ->
// Modulate -> GELU-tanh MLP -> gated residual. Tensor names follow the
// dual-stream Qwen-Image checkpoint layout (img_* / txt_* streams).
//
// Sequence layout in HBM: one [image rows; text rows] activation matrix
// (QwenImageDit's order, image first), so each projection of both streams is
// ONE GEMM launch with two weight groups split at the first text row.
// Weights are packed per kind across blocks: qkv [blocks][2][3D][D],
// out [blocks][2][D][D], up [blocks][2][F][D], down [blocks][2][D][F],
// modulation [blocks][2][6D][D] (one GEMV pass for every block's vectors).
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_runtime.h"

namespace nd {

namespace {

// QwenImageDit.RopeTables (Models/QwenImage/QwenImageDit.cs:189-240): rows
// for the image cells in row-major order, then `context_rows` text rows;
// 64 pair columns over the axes 16/56/56 at 10000^(-2k/axis). Image cell
// (i, j) sits at (text_len, i - ceil(h/2), j - ceil(w/2)); text token p at (p, p, p).
void qwen_rope_tables(int rows, int columns, int text_len, int context_rows, float* cos,
                      float* sin) {
  const int axes[3] = {16, 56, 56};
  double freq[64];
  int p = 0;
  for (int a = 0; a < 3; ++a)
    for (int k = 0; k < axes[a] / 2; ++k) freq[p++] = 1.0 / std::pow(10000.0, 2.0 * k / axes[a]);
  auto fill = [&](int token, double a0, double a1, double a2) {
    const double pos[3] = {a0, a1, a2};
    int pr = 0;
    for (int a = 0; a < 3; ++a)
      for (int k = 0; k < axes[a] / 2; ++k, ++pr) {
        const double ang = pos[a] * freq[pr];
        cos[static_cast<int64_t>(token) * 64 + pr] = static_cast<float>(std::cos(ang));
        sin[static_cast<int64_t>(token) * 64 + pr] = static_cast<float>(std::sin(ang));
      }
  };
  const int r0 = rows - rows / 2, c0 = columns - columns / 2;
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < columns; ++j) fill(i * columns + j, text_len, i - r0, j - c0);
  for (int t = 0; t < context_rows; ++t) fill(rows * columns + t, t, t, t);
}

// Transformer.Sinusoid (Graph/Transformer.cs:20-32) of QwenImageDit.TimeEmbedding
// (:178-179): half cosines then half sines of (float)(sigma * 1000) * 10000^(-i/half).
void sinusoid(double sigma, int width, float* out) {
  const float time = static_cast<float>(sigma * 1000.0);
  const int half = width / 2;
  for (int i = 0; i < half; ++i) {
    const float frequency = std::exp(-std::log(10000.0f) * i / half);
    const float angle = time * frequency;
    out[i] = std::cos(angle);
    out[half + i] = std::sin(angle);
  }
}

struct MMDiT final : nd_denoiser {
  int D = 0, H = 0, F = 0, NB = 0, ctx = 0, cw = 0, C = 0, Hl = 0, Wl = 0, P = 0, tw = 0, cin = 0;
  int n_img = 0, M = 0;
  int dt = ND_BF16;
  // fp32 compute: GEMM operands as bf16 hi|lo pairs (lt = ND_BF16X2, pair
  // buffers twice as wide), Q/K/V and the attention in fp32.
  bool f32 = false;
  int lt = ND_BF16;
  int pw = 1;     // columns per logical column in GEMM-operand buffers
  size_t qe = 2;  // bytes per element of the Q/K/V buffer
  float eps = 1e-6f;
  // weights (compute dtype or int8 + scales) and vectors (fp32)
  Mat img_in_w, txt_in_w, t1_w, t2_w, mod_w, qkv_w, out_w, up_w, down_w, norm_out_w, proj_out_w;
  float *img_in_b = nullptr, *txt_norm = nullptr, *txt_in_b = nullptr, *t1_b = nullptr, *t2_b = nullptr;
  float *mod_b = nullptr, *qkv_b = nullptr, *out_b = nullptr, *up_b = nullptr, *down_b = nullptr;
  float *qk_norm = nullptr, *norm_out_b = nullptr, *proj_out_b = nullptr;
  // inputs
  float *in_latent = nullptr, *in_ctx = nullptr, *in_tsin = nullptr, *in_cos = nullptr, *in_sin = nullptr;
  int key_limit = 0;
  bool default_rope = true;
  std::vector<float> def_cos, def_sin;
  float* tsin = nullptr;  // pinned
  // scratch
  float *x = nullptr, *temb_h = nullptr, *temb = nullptr, *mods = nullptr, *fmod = nullptr;
  float *out_tok = nullptr, *out_latent = nullptr;
  void *xn = nullptr, *qkv = nullptr, *attn = nullptr, *hid = nullptr, *tok_in = nullptr, *ctx_n = nullptr;

  size_t esz() const { return 2; }

  int build() override {
    const nd_model_desc& d = desc;
    if (d.batch != 1) return fail(ND_ERR_UNSUPPORTED, "mmdit: batch must be 1 (shard images across devices)");
    if (d.compute != ND_BF16 && d.compute != ND_F16 && d.compute != ND_F32)
      return fail(ND_ERR_UNSUPPORTED, "mmdit: compute must be bf16, f16 or f32");
    if (d.weight_dtype != d.compute && !(d.weight_dtype == ND_I8 && d.compute != ND_F32))
      return fail(ND_ERR_UNSUPPORTED, "mmdit: weights must be stored in the compute dtype (or int8 with 16-bit compute)");
    if (d.weight_dtype == ND_I8) {
      if (d.quant_scale_dtype != ND_F16 && d.quant_scale_dtype != ND_F32)
        return fail(ND_ERR_INVALID, "mmdit: int8 weights need quant_scale_dtype ND_F16 or ND_F32");
      if (d.quant_group < 0 || (d.quant_group > 0 && d.quant_group % 16))
        return fail(ND_ERR_INVALID, "mmdit: quant_group must be 0 (per channel) or a multiple of 16");
    }
    if (d.head_dim != 128 || d.heads * 128 != d.width) return fail(ND_ERR_INVALID, "mmdit: width must be heads x 128");
    if (d.width % 256) return fail(ND_ERR_UNSUPPORTED, "mmdit: width must be a multiple of 256");
    if (d.blocks <= 0 || d.mlp_width <= 0 || d.mlp_width % 8) return fail(ND_ERR_INVALID, "mmdit: bad blocks / mlp_width");
    if (d.context_rows <= 0 || d.context_width <= 0 || d.context_width % 8 || d.context_width > 4096)
      return fail(ND_ERR_INVALID, "mmdit: context width must be a multiple of 8 up to 4096");
    if (d.patch <= 0 || d.latent_height % d.patch || d.latent_width % d.patch)
      return fail(ND_ERR_INVALID, "mmdit: latent does not divide into patches");
    if (d.time_width <= 0 || d.time_width % 8) return fail(ND_ERR_INVALID, "mmdit: time_width must be a multiple of 8");
    dt = d.compute;
    f32 = dt == ND_F32;
    lt = f32 ? ND_BF16X2 : dt;
    pw = f32 ? 2 : 1;
    qe = f32 ? 4 : 2;
    D = d.width;
    H = d.heads;
    F = d.mlp_width;
    NB = d.blocks;
    ctx = d.context_rows;
    cw = d.context_width;
    C = d.latent_channels;
    Hl = d.latent_height;
    Wl = d.latent_width;
    P = d.patch;
    tw = d.time_width;
    cin = C * P * P;
    if (cin % 8) return fail(ND_ERR_INVALID, "mmdit: channels x patch^2 must be a multiple of 8");
    if (f32 && (cin % 64 || cw % 64 || F % 64))
      return fail(ND_ERR_UNSUPPORTED, "mmdit: fp32 compute needs channels x patch^2, context width and mlp width % 64 == 0");
    n_img = (Hl / P) * (Wl / P);
    if (n_img % 128) return fail(ND_ERR_UNSUPPORTED, "mmdit: image tokens must be a multiple of 128");
    M = n_img + ctx;
    eps = d.eps > 0 ? d.eps : 1e-6f;
    const int64_t DD = static_cast<int64_t>(D) * D;

    // ---- weights
    auto V = [&](int64_t elems) { return static_cast<float*>(alloc(static_cast<size_t>(elems) * 4, true)); };
    img_in_w = alloc_mat(D, cin, D);
    img_in_b = V(D);
    txt_norm = V(cw);
    txt_in_w = alloc_mat(D, cw, D);
    txt_in_b = V(D);
    t1_w = alloc_mat(D, tw, D);
    t1_b = V(D);
    t2_w = alloc_mat(D, D, D);
    t2_b = V(D);
    mod_w = alloc_mat(static_cast<int64_t>(NB) * 2 * 6 * D, D, 6 * D);
    mod_b = V(static_cast<int64_t>(NB) * 2 * 6 * D);
    qkv_w = alloc_mat(static_cast<int64_t>(NB) * 2 * 3 * D, D, D);
    qkv_b = V(static_cast<int64_t>(NB) * 2 * 3 * D);
    out_w = alloc_mat(static_cast<int64_t>(NB) * 2 * D, D, D);
    out_b = V(static_cast<int64_t>(NB) * 2 * D);
    up_w = alloc_mat(static_cast<int64_t>(NB) * 2 * F, D, F);
    up_b = V(static_cast<int64_t>(NB) * 2 * F);
    down_w = alloc_mat(static_cast<int64_t>(NB) * 2 * D, F, D);
    down_b = V(static_cast<int64_t>(NB) * 2 * D);
    qk_norm = V(static_cast<int64_t>(NB) * 2 * 2 * 128);
    norm_out_w = alloc_mat(2 * D, D, 2 * D);
    norm_out_b = V(2 * D);
    proj_out_w = alloc_mat(cin, D, cin);
    proj_out_b = V(cin);
    // ---- inputs and scratch
    auto S = [&](size_t bytes) { return alloc(bytes, false); };
    in_latent = static_cast<float*>(S(static_cast<size_t>(C) * Hl * Wl * 4));
    in_ctx = static_cast<float*>(S(static_cast<size_t>(ctx) * cw * 4));
    in_tsin = static_cast<float*>(S(static_cast<size_t>(tw) * 4));
    in_cos = static_cast<float*>(S(static_cast<size_t>(M) * 64 * 4));
    in_sin = static_cast<float*>(S(static_cast<size_t>(M) * 64 * 4));
    x = static_cast<float*>(S(static_cast<size_t>(M) * D * 4));
    temb_h = static_cast<float*>(S(static_cast<size_t>(D) * 4));
    temb = static_cast<float*>(S(static_cast<size_t>(D) * 4));
    mods = static_cast<float*>(S(static_cast<size_t>(NB) * 2 * 6 * D * 4));
    fmod = static_cast<float*>(S(static_cast<size_t>(2) * D * 4));
    out_tok = static_cast<float*>(S(static_cast<size_t>(n_img) * cin * 4));
    out_latent = static_cast<float*>(S(static_cast<size_t>(C) * Hl * Wl * 4));
    xn = S(static_cast<size_t>(M) * D * esz() * pw);
    qkv = S(static_cast<size_t>(M) * 3 * D * qe);
    attn = S(static_cast<size_t>(M) * D * esz() * pw);
    hid = S(static_cast<size_t>(M) * F * esz() * pw);
    tok_in = S(static_cast<size_t>(n_img) * cin * esz() * pw);
    ctx_n = S(static_cast<size_t>(ctx) * cw * esz() * pw);
    tsin = static_cast<float*>(pinned(static_cast<size_t>(tw) * 4));
    if (desc.compute != ND_F32) alloc_attn_workspace(128);
    if (alloc_failed) return fail(ND_ERR_OOM, "mmdit: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));

    // ---- registry (dual-stream Qwen-Image tensor names)
    auto M_ = [&](const std::string& name, const Mat& m, int64_t row, int64_t rows) {
      const int64_t sc = m.q8 ? m.cols / qgroup(m.cols) : 0;
      add_slot(name, kMatrix, rows, m.cols, m.at(row, 2), true, m.q8 ? m.scales_at(row, sc, qf16()) : nullptr);
    };
    M_("img_in.weight", img_in_w, 0, D);
    add_slot("img_in.bias", kVector, D, 1, img_in_b, false);
    add_slot("txt_norm.weight", kVector, cw, 1, txt_norm);
    M_("txt_in.weight", txt_in_w, 0, D);
    add_slot("txt_in.bias", kVector, D, 1, txt_in_b, false);
    M_("time_text_embed.timestep_embedder.linear_1.weight", t1_w, 0, D);
    add_slot("time_text_embed.timestep_embedder.linear_1.bias", kVector, D, 1, t1_b, false);
    M_("time_text_embed.timestep_embedder.linear_2.weight", t2_w, 0, D);
    add_slot("time_text_embed.timestep_embedder.linear_2.bias", kVector, D, 1, t2_b, false);
    M_("norm_out.linear.weight", norm_out_w, 0, 2 * D);
    add_slot("norm_out.linear.bias", kVector, 2 * D, 1, norm_out_b, false);
    M_("proj_out.weight", proj_out_w, 0, cin);
    add_slot("proj_out.bias", kVector, cin, 1, proj_out_b, false);
    const char* stream_mod[2] = {"img_mod.1", "txt_mod.1"};
    const char* proj[2][3] = {{"attn.to_q", "attn.to_k", "attn.to_v"},
                              {"attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"}};
    const char* norms[2][2] = {{"attn.norm_q", "attn.norm_k"}, {"attn.norm_added_q", "attn.norm_added_k"}};
    const char* outs[2] = {"attn.to_out.0", "attn.to_add_out"};
    const char* ups[2] = {"img_mlp.net.0.proj", "txt_mlp.net.0.proj"};
    const char* downs[2] = {"img_mlp.net.2", "txt_mlp.net.2"};
    for (int b = 0; b < NB; ++b) {
      const std::string pre = "transformer_blocks." + std::to_string(b) + ".";
      for (int s = 0; s < 2; ++s) {
        const int64_t g = static_cast<int64_t>(b) * 2 + s;
        M_(pre + stream_mod[s] + ".weight", mod_w, g * 6 * D, 6 * D);
        add_slot(pre + stream_mod[s] + ".bias", kVector, 6 * D, 1, mod_b + g * 6 * D, false);
        for (int j = 0; j < 3; ++j) {
          M_(pre + proj[s][j] + ".weight", qkv_w, (g * 3 + j) * D, D);
          add_slot(pre + proj[s][j] + ".bias", kVector, D, 1, qkv_b + (g * 3 + j) * D, false);
        }
        for (int j = 0; j < 2; ++j)
          add_slot(pre + norms[s][j] + ".weight", kVector, 128, 1, qk_norm + (g * 2 + j) * 128);
        M_(pre + outs[s] + ".weight", out_w, g * D, D);
        add_slot(pre + outs[s] + ".bias", kVector, D, 1, out_b + g * D, false);
        M_(pre + ups[s] + ".weight", up_w, g * F, F);
        add_slot(pre + ups[s] + ".bias", kVector, F, 1, up_b + g * F, false);
        M_(pre + downs[s] + ".weight", down_w, g * D, D);
        add_slot(pre + downs[s] + ".bias", kVector, D, 1, down_b + g * D, false);
      }
    }
    def_cos.resize(static_cast<size_t>(M) * 64);
    def_sin.resize(static_cast<size_t>(M) * 64);
    qwen_rope_tables(Hl / P, Wl / P, ctx, ctx, def_cos.data(), def_sin.data());
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

  int64_t latent_elems() const override { return static_cast<int64_t>(C) * Hl * Wl; }
  const float* output() const override { return out_latent; }

  int check_cond(int n, const nd_named_tensor* cond, StepInputs& in) override {
    for (int i = 0; i < n; ++i) {
      const nd_named_tensor& t = cond[i];
      if (!t.name || !t.data) return fail(ND_ERR_INVALID, "predict: conditioning entry without name or data");
      int64_t elems = 1;
      for (int r = 0; r < t.rank; ++r) elems *= t.shape[r];
      const std::string name = t.name;
      if (name == "context") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(ctx) * cw)
          return fail(ND_ERR_INVALID, "predict: context must be f32 [1, " + std::to_string(ctx) + ", " + std::to_string(cw) + "]");
        in.context = static_cast<const float*>(t.data);
      } else if (name == "cos" || name == "sin") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(M) * 64)
          return fail(ND_ERR_INVALID, "predict: " + name + " must be f32 [" + std::to_string(M) + ", 64]");
        (name == "cos" ? in.cos : in.sin) = static_cast<const float*>(t.data);
      } else if (name == "key_length") {
        if (t.dtype != ND_I32 || elems != 1 || in.device)
          return fail(ND_ERR_INVALID, "predict: key_length must be one host i32");
        const int k = *static_cast<const int32_t*>(t.data);
        if (k < 1 || k > M) return fail(ND_ERR_INVALID, "predict: key_length out of range");
        in.key_limit = k == M ? 0 : k;
      } else if (name == "text_mask") {
        // Qwen-Image 2.1's causal text table: the dual-stream block attends
        // jointly and takes no table.
        continue;
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
    ND_CUDA(cudaMemcpyAsync(in_ctx, in.context, static_cast<size_t>(ctx) * cw * 4, k, s));
    // The pinned sinusoid buffer is reused: wait until the previous call's
    // copy out of it has run before overwriting it.
    ND_CUDA(cudaEventSynchronize(staged));
    sinusoid(in.sigma, tw, tsin);
    ND_CUDA(cudaMemcpyAsync(in_tsin, tsin, static_cast<size_t>(tw) * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaEventRecord(staged, s));
    if (in.cos) {
      ND_CUDA(cudaMemcpyAsync(in_cos, in.cos, static_cast<size_t>(M) * 64 * 4, k, s));
      ND_CUDA(cudaMemcpyAsync(in_sin, in.sin, static_cast<size_t>(M) * 64 * 4, k, s));
      default_rope = false;
    } else if (!default_rope) {
      ND_CUDA(cudaMemcpyAsync(in_cos, def_cos.data(), def_cos.size() * 4, cudaMemcpyHostToDevice, s));
      ND_CUDA(cudaMemcpyAsync(in_sin, def_sin.data(), def_sin.size() * 4, cudaMemcpyHostToDevice, s));
      default_rope = true;
    }
    key_limit = in.key_limit;
    return ND_OK;
  }

  // Point a GEMM at rows [row, ...) of a matrix kind (int8 or compute dtype).
  void weight_args(nd_linear_args& a, const Mat& m, int64_t row) const {
    a.weight = m.at(row, 2);
    if (m.q8) {
      a.weight_dtype = ND_I8;
      a.scales = m.scales_at(row, m.cols / qgroup(m.cols), qf16());
      a.scale_dtype = desc.quant_scale_dtype;
      a.quant_group = desc.quant_group;
    }
  }

  int lin(cudaStream_t s, const void* xin, int64_t rows, int64_t k, int64_t ldx, const Mat& w, int64_t wrow,
          const float* b, int64_t n, int epi, void* y, int64_t ldy, float* resid, int64_t ldr,
          const float* gate, int64_t gate_stride, int64_t split) {
    nd_linear_args a{};
    a.dtype = lt;
    a.epilogue = epi;
    a.rows = rows;
    a.in_features = k;
    a.out_features = n;
    a.x = xin;
    a.ldx = ldx * pw;  // pairs: hi then lo columns
    weight_args(a, w, wrow);
    a.bias = b;
    a.group_split = split;
    a.y = y;
    a.ldy = ldy * pw;
    a.residual = resid;
    a.ldr = ldr;
    a.gate = gate;
    a.gate_stride = gate_stride;
    a.eps = eps;
    return linear(a, s);
  }

  int mod(cudaStream_t s, const float* shift, const float* scale, int64_t rows, int64_t split) {
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
    m.vec_stride = 6 * D;
    m.group_split = split;
    m.eps = eps;
    return modulate(m, s);
  }

  int gv(cudaStream_t s, const Mat& w, int64_t n, int64_t k, const float* xin, const float* b,
         bool pre_silu, int act, float* y) {
    nd_gemv_args g{};
    g.w = w.w;
    g.w_dtype = w.q8 ? ND_I8 : lt;
    g.n = n;
    g.k = k;
    g.x = xin;
    g.batch = 1;
    g.pre_silu = pre_silu ? 1 : 0;
    g.bias = b;
    g.act = act;
    g.y = y;
    if (w.q8) {
      g.scales = w.scales;
      g.scale_dtype = desc.quant_scale_dtype;
      g.quant_group = desc.quant_group;
    }
    return gemv(g, s);
  }

#define ND_OP(cls, flops, bytes, expr) \
  do {                                 \
    prof_begin(s);                     \
    int rc_ = (expr);                  \
    if (rc_) return rc_;               \
    prof_end(s, cls, flops, bytes);    \
  } while (0)

  // Algorithmic work of the ops (1 MAC = 2 FLOP; bytes = each operand read
  // once and each result written once).
  double gemm_flops(double m, double n, double k) const { return 2.0 * m * n * k; }
  double gemm_bytes(double m, double n, double k, double out_bytes) const {
    return 2.0 * (m * k + n * k) + out_bytes;
  }

  int block(cudaStream_t s, int b) {
    const int64_t g0 = static_cast<int64_t>(b) * 2;
    const float* mv = mods + g0 * 6 * D;  // [2][6D]: shift1 scale1 gate1 shift2 scale2 gate2
    const double mD = static_cast<double>(M) * D;
    const double mod_bytes = mD * (4.0 + 2.0);
    const double keys = key_limit > 0 ? key_limit : M;
    ND_OP("modulate", 0.0, mod_bytes, mod(s, mv, mv + D, M, n_img));
    {
      nd_linear_args a{};
      a.dtype = lt;
      a.epilogue = ND_EPI_QK_NORM_ROPE;
      a.rows = M;
      a.in_features = D;
      a.out_features = 3 * D;
      a.x = xn;
      a.ldx = static_cast<int64_t>(D) * pw;
      weight_args(a, qkv_w, g0 * 3 * D);
      a.bias = qkv_b + g0 * 3 * D;
      a.group_split = n_img;
      a.y = qkv;
      a.ldy = 3 * D;
      a.qk_norm = qk_norm + g0 * 2 * 128;
      a.rope_cos = in_cos;
      a.rope_sin = in_sin;
      a.qk_cols = 2 * D;
      a.eps = eps;
      ND_OP("gemm.qkv", gemm_flops(M, 3.0 * D, D), gemm_bytes(M, 6.0 * D, D, mD * 3 * 2), linear(a, s));
    }
    {
      nd_attention_args a{};
      a.dtype = dt;
      a.out_dtype = f32 ? ND_BF16X2 : 0;
      a.heads = H;
      a.head_dim = 128;
      a.batch = 1;
      a.q_rows = M;
      a.kv_rows = M;
      a.key_limit = key_limit;
      a.q = qkv;
      a.ldq = 3 * D;
      a.k = static_cast<uint8_t*>(qkv) + static_cast<size_t>(D) * qe;
      a.ldk = 3 * D;
      a.v = static_cast<uint8_t*>(qkv) + static_cast<size_t>(2 * D) * qe;
      a.ldv = 3 * D;
      a.out = attn;
      a.ldo = static_cast<int64_t>(D) * pw;
      use_attn_workspace(a);
      ND_OP("attention", 4.0 * M * keys * D, mD * 2 * 4, attention(a, s));
    }
    ND_OP("gemm.out", gemm_flops(M, D, D), gemm_bytes(M, 2.0 * D, D, mD * 8),
          lin(s, attn, M, D, D, out_w, g0 * D, out_b + g0 * D, D, ND_EPI_RESIDUAL_GATE, nullptr, 0,
              x, D, mv + 2 * D, 6 * D, n_img));
    ND_OP("modulate", 0.0, mod_bytes, mod(s, mv + 3 * D, mv + 4 * D, M, n_img));
    ND_OP("gemm.up", gemm_flops(M, F, D), gemm_bytes(M, 2.0 * F, D, static_cast<double>(M) * F * 2),
          lin(s, xn, M, D, D, up_w, g0 * F, up_b + g0 * F, F,
              ND_EPI_GELU_TANH, hid, F, nullptr, 0, nullptr, 0, n_img));
    ND_OP("gemm.down", gemm_flops(M, D, F), gemm_bytes(M, 2.0 * D, F, mD * 8),
          lin(s, hid, M, F, F, down_w, g0 * D, down_b + g0 * D, D,
              ND_EPI_RESIDUAL_GATE, nullptr, 0, x, D, mv + 5 * D, 6 * D, n_img));
    return ND_OK;
  }

  int forward(cudaStream_t s) override {
    const double ni = n_img, dD = D;
    // embeddings: image patches and text rows into one fp32 sequence
    ND_OP("embed", 0.0, ni * cin * 6.0, patchify(in_latent, tok_in, lt, 1, C, Hl, Wl, P, cin * pw, s));
    ND_OP("embed", gemm_flops(ni, dD, cin), gemm_bytes(ni, dD, cin, ni * dD * 4),
          lin(s, tok_in, n_img, cin, cin, img_in_w, 0, img_in_b, D, ND_EPI_STORE_F32, nullptr, 0, x, D,
              nullptr, 0, n_img));
    {
      nd_rmsnorm_args r{};
      r.x = in_ctx;
      r.ldx = cw;
      r.in_dtype = ND_F32;
      r.y = ctx_n;
      r.ldy = static_cast<int64_t>(cw) * pw;
      r.out_dtype = lt;
      r.rows = ctx;
      r.width = cw;
      r.weight = txt_norm;
      r.plus_one = 0;
      r.eps = eps;
      ND_OP("embed", 0.0, static_cast<double>(ctx) * cw * 6.0, rmsnorm(r, s));
    }
    ND_OP("embed", gemm_flops(ctx, dD, cw), gemm_bytes(ctx, dD, cw, ctx * dD * 4),
          lin(s, ctx_n, ctx, cw, cw, txt_in_w, 0, txt_in_b, D, ND_EPI_STORE_F32, nullptr, 0,
              x + static_cast<int64_t>(n_img) * D, D, nullptr, 0, ctx));
    // time embedding -> every block's modulation vectors in one GEMV pass
    ND_OP("gemv", 2.0 * dD * tw, dD * tw * 2, gv(s, t1_w, D, tw, in_tsin, t1_b, false, 1, temb_h));
    ND_OP("gemv", 2.0 * dD * dD, dD * dD * 2, gv(s, t2_w, D, D, temb_h, t2_b, false, 0, temb));
    const double mod_rows = static_cast<double>(NB) * 2 * 6 * D;
    ND_OP("gemv", 2.0 * mod_rows * dD, mod_rows * dD * 2,
          gv(s, mod_w, static_cast<int64_t>(NB) * 2 * 6 * D, D, temb, mod_b, true, 0, mods));
    for (int b = 0; b < NB; ++b) {
      int rc = block(s, b);
      if (rc) return rc;
    }
    // final layer over the image rows: LN * (1 + scale) + shift -> proj_out
    ND_OP("gemv", 2.0 * 2 * dD * dD, 2 * dD * dD * 2, gv(s, norm_out_w, 2 * D, D, temb, norm_out_b, true, 0, fmod));
    {
      nd_modulate_args m{};
      m.x = x;
      m.ldx = D;
      m.y = xn;
      m.ldy = static_cast<int64_t>(D) * pw;
      m.out_dtype = lt;
      m.rows = n_img;
      m.width = D;
      m.scale = fmod;
      m.shift = fmod + D;
      m.vec_stride = D;
      m.group_split = n_img;
      m.eps = eps;
      ND_OP("modulate", 0.0, ni * dD * 6.0, modulate(m, s));
    }
    ND_OP("embed", gemm_flops(ni, cin, dD), gemm_bytes(ni, cin, dD, ni * cin * 4),
          lin(s, xn, n_img, D, D, proj_out_w, 0, proj_out_b, cin, ND_EPI_STORE_F32, nullptr, 0, out_tok, cin,
              nullptr, 0, n_img));
    ND_OP("embed", 0.0, ni * cin * 8.0, unpatchify(out_tok, cin, out_latent, 1, C, Hl, Wl, P, s));
    return ND_OK;
  }
#undef ND_OP
};

}  // namespace

nd_denoiser* make_mmdit() { return new MMDiT(); }

}  // namespace nd
