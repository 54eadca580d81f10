// Qwen-Image 2.1's single-stream DiT (QwenImageDit, Models/QwenImage/
// QwenImageDit.cs): the reference's own Qwen-Image model. One [image rows;
// text rows] activation matrix (the reference's order) goes through every
// block with ONE weight set; the rows differ only in the modulation they
// read (the noise level's row for image rows, time zero's for text rows,
// :292-302) and in what they attend to (image queries over every visible
// key, text queries causally over the text keys, :329-374).
//
// Per block (:406-425):
//   modulate(x, scale_attn)           LayerNorm * (1 + scale), no shift
//   QKV GEMM, head RMSNorm + RoPE     rotate-half on pairs-to-halves weights
//   attention (image) + attention (text, causal)
//   out GEMM, x += tanh(gate_attn) * . (gate chosen per row)
//   modulate(x, scale_mlp)
//   gate_up GEMM with the SwiGLU epilogue (silu(gate) * up in the epilogue)
//   down GEMM, x += tanh(gate_mlp) * .
// The modulation is one [4 * width] vector per time row for the whole model
// (modulation.1 over SiLU(temb)); its gates pass through tanh (:486-495).
// None of the model's linear layers has a bias.
//
// Weights packed per kind across blocks: qkv [blocks][3D][D] (to_q / to_k
// rows permuted pairs -> halves per head on upload), out [blocks][D][D],
// gate_up [blocks][2F][D] (the fused file tensor, or gate_layer and proj in
// its two halves), down [blocks][D][F].
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_runtime.h"

namespace nd {

namespace {

// QwenImageDit.RopeTables (Models/QwenImage/QwenImageDit.cs:189-240): image
// cells first (frame = the branch's real text length, grid centred), then the
// context rows at (p, p, p); 64 pair columns over the axes 16 / 56 / 56.
void rope_tables(int rows, int columns, int text_len, int context_rows, float* cos, float* sin) {
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

// Transformer.Sinusoid (Graph/Transformer.cs:20-32) of
// QwenImageDit.TimeEmbedding (:178-179): t * 1000, half cosines then half sines.
void sinusoid(double time, int width, float* out) {
  const float t = static_cast<float>(time * 1000.0);
  const int half = width / 2;
  for (int i = 0; i < half; ++i) {
    const float frequency = std::exp(-std::log(10000.0f) * i / half);
    const float angle = t * frequency;
    out[i] = std::cos(angle);
    out[half + i] = std::sin(angle);
  }
}

struct QwenImage final : nd_denoiser {
  int D = 0, H = 0, F = 0, NB = 0, R = 0, cw = 0, C = 0, Hl = 0, Wl = 0, tw = 0;
  int n_img = 0, M = 0;
  int dt = ND_BF16;
  bool f32 = false;
  int lt = ND_BF16;
  int pw = 1;     // columns per logical column in GEMM-operand buffers (2: hi|lo pairs)
  size_t qe = 2;  // bytes per element of Q/K/V
  float eps = 1e-6f;
  Mat img_in_w, txt1_w, txt2_w, t1_w, t2_w, mod_w, qkv_w, out_w, gu_w, down_w, norm_out_w, proj_out_w;
  float *txt_norm = nullptr, *qk_norm = nullptr;
  // inputs
  float *in_latent = nullptr, *in_ctx = nullptr, *in_tsin = nullptr, *in_cos = nullptr, *in_sin = nullptr;
  int real = 0;           // real text rows of the staged call
  int default_real = -1;  // text length the default tables on the device were made for (-1: none)
  std::vector<float> def_cos, def_sin;
  float* tsin = nullptr;  // pinned [2][tw]
  // scratch
  float *x = nullptr, *temb_h = nullptr, *temb = nullptr, *mods = nullptr, *fscale = nullptr;
  float *out_tok = nullptr, *out_latent = nullptr;
  void *xn = nullptr, *qkv = nullptr, *attn = nullptr, *hid = nullptr, *tok_in = nullptr, *ctx_n = nullptr;

  int build() override {
    const nd_model_desc& d = desc;
    if (d.batch != 1) return fail(ND_ERR_UNSUPPORTED, "qwen_image: batch must be 1 (run branches as separate calls or devices)");
    if (d.compute != ND_BF16 && d.compute != ND_F16 && d.compute != ND_F32)
      return fail(ND_ERR_UNSUPPORTED, "qwen_image: compute must be bf16, f16 or f32");
    if (d.weight_dtype != d.compute && !(d.weight_dtype == ND_I8 && d.compute != ND_F32))
      return fail(ND_ERR_UNSUPPORTED, "qwen_image: weights must be stored in the compute dtype (or int8 with 16-bit compute)");
    if (d.weight_dtype == ND_I8) {
      if (d.quant_scale_dtype != ND_F16 && d.quant_scale_dtype != ND_F32)
        return fail(ND_ERR_INVALID, "qwen_image: int8 weights need quant_scale_dtype ND_F16 or ND_F32");
      if (d.quant_group < 0 || (d.quant_group > 0 && d.quant_group % 16))
        return fail(ND_ERR_INVALID, "qwen_image: quant_group must be 0 (per channel) or a multiple of 16");
    }
    if (d.head_dim != 128 || d.heads * 128 != d.width)
      return fail(ND_ERR_INVALID, "qwen_image: width must be heads x 128 (the rotary axes take 128 features)");
    if (d.blocks <= 0 || d.mlp_width <= 0 || d.mlp_width % 128)
      return fail(ND_ERR_INVALID, "qwen_image: mlp_width must be a positive multiple of 128");
    if (d.context_rows <= 0 || d.context_width <= 0 || d.context_width % 64)
      return fail(ND_ERR_INVALID, "qwen_image: context width must be a multiple of 64");
    if (d.patch != 1 && d.patch != 0) return fail(ND_ERR_INVALID, "qwen_image: patch is 1");
    if (d.latent_channels <= 0 || d.latent_channels % 64)
      return fail(ND_ERR_INVALID, "qwen_image: latent channels must be a multiple of 64 (64 for Qwen-Image 2.1)");
    if (d.time_width <= 0 || d.time_width % 64) return fail(ND_ERR_INVALID, "qwen_image: time_width must be a multiple of 64");
    dt = d.compute;
    f32 = dt == ND_F32;
    lt = f32 ? ND_BF16X2 : dt;
    pw = f32 ? 2 : 1;
    qe = f32 ? 4 : 2;
    D = d.width;
    H = d.heads;
    F = d.mlp_width;
    NB = d.blocks;
    R = d.context_rows;
    cw = d.context_width;
    C = d.latent_channels;
    Hl = d.latent_height;
    Wl = d.latent_width;
    tw = d.time_width;
    if (Hl <= 0 || Wl <= 0) return fail(ND_ERR_INVALID, "qwen_image: empty latent");
    n_img = Hl * Wl;
    M = n_img + R;
    real = R;
    eps = d.eps > 0 ? d.eps : 1e-6f;

    // ---- weights (no biases anywhere)
    img_in_w = alloc_mat(D, C, D);
    txt_norm = static_cast<float*>(alloc(static_cast<size_t>(cw) * 4, true));
    txt1_w = alloc_mat(D, cw, D);
    txt2_w = alloc_mat(D, D, D);
    t1_w = alloc_mat(D, tw, D);
    t2_w = alloc_mat(D, D, D);
    mod_w = alloc_mat(4LL * D, D, D);
    qkv_w = alloc_mat(static_cast<int64_t>(NB) * 3 * D, D, D);
    out_w = alloc_mat(static_cast<int64_t>(NB) * D, D, D);
    gu_w = alloc_mat(static_cast<int64_t>(NB) * 2 * F, D, F);
    down_w = alloc_mat(static_cast<int64_t>(NB) * D, F, D);
    qk_norm = static_cast<float*>(alloc(static_cast<size_t>(NB) * 2 * 128 * 4, true));
    norm_out_w = alloc_mat(D, D, D);
    proj_out_w = alloc_mat(C, D, C);
    // ---- inputs and scratch
    auto S = [&](size_t bytes) { return alloc(bytes, false); };
    in_latent = static_cast<float*>(S(static_cast<size_t>(C) * n_img * 4));
    in_ctx = static_cast<float*>(S(static_cast<size_t>(R) * cw * 4));
    in_tsin = static_cast<float*>(S(static_cast<size_t>(2) * tw * 4));
    in_cos = static_cast<float*>(S(static_cast<size_t>(M) * 64 * 4));
    in_sin = static_cast<float*>(S(static_cast<size_t>(M) * 64 * 4));
    x = static_cast<float*>(S(static_cast<size_t>(M) * D * 4));
    temb_h = static_cast<float*>(S(static_cast<size_t>(2) * D * 4));
    temb = static_cast<float*>(S(static_cast<size_t>(2) * D * 4));
    mods = static_cast<float*>(S(static_cast<size_t>(4) * 2 * D * 4));
    fscale = static_cast<float*>(S(static_cast<size_t>(D) * 4));
    out_tok = static_cast<float*>(S(static_cast<size_t>(n_img) * C * 4));
    out_latent = static_cast<float*>(S(static_cast<size_t>(C) * n_img * 4));
    xn = S(static_cast<size_t>(M) * D * 2 * pw);
    qkv = S(static_cast<size_t>(M) * 3 * D * qe);
    attn = S(static_cast<size_t>(M) * D * 2 * pw);
    hid = S(static_cast<size_t>(M) * (F > D ? F : D) * 2 * pw);
    tok_in = S(static_cast<size_t>(n_img) * C * 2 * pw);
    ctx_n = S(static_cast<size_t>(R) * cw * 2 * pw);
    tsin = static_cast<float*>(pinned(static_cast<size_t>(2) * tw * 4));
    if (desc.compute != ND_F32) alloc_attn_workspace(128);
    if (alloc_failed) return fail(ND_ERR_OOM, "qwen_image: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));

    // ---- registry (QwenImageCheckpoint / QwenImageDit tensor names)
    auto M_ = [&](const std::string& name, const Mat& m, int64_t row, int64_t rows, bool required = true,
                  int head_perm = 0) {
      const int64_t sc = m.q8 ? m.cols / qgroup(m.cols) : 0;
      add_slot(name, kMatrix, rows, m.cols, m.at(row, 2), required, m.q8 ? m.scales_at(row, sc, qf16()) : nullptr);
      slots.back().head_perm = head_perm;
    };
    M_("img_in.weight", img_in_w, 0, D);
    add_slot("txt_in.text_norm.weight", kVector, cw, 1, txt_norm);
    M_("txt_in.in_layer.weight", txt1_w, 0, D);
    M_("txt_in.out_layer.weight", txt2_w, 0, D);
    M_("time_text_embed.timestep_embedder.linear_1.weight", t1_w, 0, D);
    M_("time_text_embed.timestep_embedder.linear_2.weight", t2_w, 0, D);
    M_("modulation.1.weight", mod_w, 0, 4LL * D);
    M_("norm_out.linear.weight", norm_out_w, 0, D);
    M_("proj_out.weight", proj_out_w, 0, C);
    for (int b = 0; b < NB; ++b) {
      const std::string pre = "transformer_blocks." + std::to_string(b) + ".";
      const int64_t q0 = static_cast<int64_t>(b) * 3 * D;
      M_(pre + "attn.to_q.weight", qkv_w, q0, D, true, 128);
      M_(pre + "attn.to_k.weight", qkv_w, q0 + D, D, true, 128);
      M_(pre + "attn.to_v.weight", qkv_w, q0 + 2 * D, D);
      add_slot(pre + "attn.norm_q.weight", kVector, 128, 1, qk_norm + (static_cast<int64_t>(b) * 2) * 128);
      slots.back().head_perm = 128;
      add_slot(pre + "attn.norm_k.weight", kVector, 128, 1, qk_norm + (static_cast<int64_t>(b) * 2 + 1) * 128);
      slots.back().head_perm = 128;
      M_(pre + "attn.to_out.0.weight", out_w, static_cast<int64_t>(b) * D, D);
      // the feed-forward's two projections: fused as one file tensor, or
      // separate (QwenImageCheckpoint.FusedGateUp / GateProjection / UpProjection)
      const int64_t g0 = static_cast<int64_t>(b) * 2 * F;
      M_(pre + "img_mlp.gate_up.weight", gu_w, g0, 2LL * F, false);
      M_(pre + "img_mlp.gate_layer.weight", gu_w, g0, F, false);
      M_(pre + "img_mlp.proj.weight", gu_w, g0 + F, F, false);
      M_(pre + "img_mlp.out.weight", down_w, static_cast<int64_t>(b) * D, D);
    }
    def_cos.resize(static_cast<size_t>(M) * 64);
    def_sin.resize(static_cast<size_t>(M) * 64);
    return ND_OK;
  }

  int prepare() override {
    // Every block needs its feed-forward: the fused tensor or both halves.
    for (int b = 0; b < NB; ++b) {
      const std::string pre = "transformer_blocks." + std::to_string(b) + ".img_mlp.";
      auto is_set = [&](const std::string& n) { return slots[index.at(pre + n)].set; };
      if (!is_set("gate_up.weight") && !(is_set("gate_layer.weight") && is_set("proj.weight")))
        return fail(ND_ERR_MISSING_WEIGHT, "qwen_image: " + pre + "gate_up.weight (or gate_layer + proj) not set");
    }
    default_real = -1;
    return ND_OK;
  }

  int64_t latent_elems() const override { return static_cast<int64_t>(C) * n_img; }
  const float* output() const override { return out_latent; }

  int check_cond(int n, const nd_named_tensor* cond, StepInputs& in) override {
    const int32_t* mask = nullptr;
    for (int i = 0; i < n; ++i) {
      const nd_named_tensor& t = cond[i];
      if (!t.name || !t.data) return fail(ND_ERR_INVALID, "predict: conditioning entry without name or data");
      int64_t elems = 1;
      for (int r = 0; r < t.rank; ++r) elems *= t.shape[r];
      const std::string name = t.name;
      if (name == "context") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(R) * cw)
          return fail(ND_ERR_INVALID, "predict: context must be f32 [1, " + std::to_string(R) + ", " + std::to_string(cw) + "]");
        in.context = static_cast<const float*>(t.data);
      } else if (name == "cos" || name == "sin") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(M) * 64)
          return fail(ND_ERR_INVALID, "predict: " + name + " must be f32 [" + std::to_string(M) + ", 64]");
        (name == "cos" ? in.cos : in.sin) = static_cast<const float*>(t.data);
      } else if (name == "key_length") {
        if (t.dtype != ND_I32 || elems != 1 || in.device)
          return fail(ND_ERR_INVALID, "predict: key_length must be one host i32");
        const int k = *static_cast<const int32_t*>(t.data);
        if (k <= n_img || k > M)
          return fail(ND_ERR_INVALID, "predict: key_length must be image tokens + 1 .. image tokens + rows");
        in.key_limit = k == M ? 0 : k;
      } else if (name == "text_mask") {
        if (t.dtype != ND_I32 || elems != static_cast<int64_t>(R) * R)
          return fail(ND_ERR_INVALID, "predict: text_mask must be i32 [" + std::to_string(R) + ", " + std::to_string(R) + "]");
        if (!in.device) mask = static_cast<const int32_t*>(t.data);
      } else {
        return fail(ND_ERR_INVALID, "predict: unknown conditioning " + name);
      }
    }
    if (!in.context) return fail(ND_ERR_INVALID, "predict: conditioning needs \"context\"");
    if ((in.cos == nullptr) != (in.sin == nullptr)) return fail(ND_ERR_INVALID, "predict: give both cos and sin");
    if (mask) {
      // QwenImageConditioning.CausalTable (Models/QwenImage/QwenImageConditioner.cs:66-78):
      // the one table the text attention's causal + key-count masks express.
      const int rl = in.key_limit > 0 ? in.key_limit - n_img : R;
      for (int i = 0; i < R; ++i)
        for (int j = 0; j < R; ++j)
          if ((mask[static_cast<int64_t>(i) * R + j] != 0) != (j <= i && j < rl))
            return fail(ND_ERR_INVALID, "predict: text_mask is not the causal table over " + std::to_string(rl) +
                                            " real rows (row " + std::to_string(i) + ", key " + std::to_string(j) + ")");
    }
    return ND_OK;
  }

  int stage(const StepInputs& in, cudaStream_t s) override {
    const cudaMemcpyKind k = in.device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    ND_CUDA(cudaMemcpyAsync(in_latent, in.latent, static_cast<size_t>(latent_elems()) * 4, k, s));
    ND_CUDA(cudaMemcpyAsync(in_ctx, in.context, static_cast<size_t>(R) * cw * 4, k, s));
    // The pinned buffers are reused: wait for the previous call's copies out of them.
    ND_CUDA(cudaEventSynchronize(staged));
    sinusoid(in.sigma, tw, tsin);
    sinusoid(0.0, tw, tsin + tw);
    ND_CUDA(cudaMemcpyAsync(in_tsin, tsin, static_cast<size_t>(2) * tw * 4, cudaMemcpyHostToDevice, s));
    real = in.key_limit > 0 ? in.key_limit - n_img : R;
    if (in.cos) {
      ND_CUDA(cudaMemcpyAsync(in_cos, in.cos, static_cast<size_t>(M) * 64 * 4, k, s));
      ND_CUDA(cudaMemcpyAsync(in_sin, in.sin, static_cast<size_t>(M) * 64 * 4, k, s));
      default_real = -1;
    } else if (default_real != real) {
      // the conditioner's tables: image rows placed after this branch's real text
      rope_tables(Hl, Wl, real, R, def_cos.data(), def_sin.data());
      ND_CUDA(cudaMemcpyAsync(in_cos, def_cos.data(), def_cos.size() * 4, cudaMemcpyHostToDevice, s));
      ND_CUDA(cudaMemcpyAsync(in_sin, def_sin.data(), def_sin.size() * 4, cudaMemcpyHostToDevice, s));
      ND_CUDA(cudaStreamSynchronize(s));  // def_* are rewritten by the next change
      default_real = real;
    }
    ND_CUDA(cudaEventRecord(staged, s));
    return ND_OK;
  }

  void weight_args(nd_linear_args& a, const Mat& w, int64_t row) const {
    a.weight = w.at(row, 2);
    if (w.q8) {
      a.weight_dtype = ND_I8;
      a.scales = w.scales_at(row, w.cols / qgroup(w.cols), qf16());
      a.scale_dtype = desc.quant_scale_dtype;
      a.quant_group = desc.quant_group;
    }
  }

  // One GEMM over `rows` rows of xin; gate (RESIDUAL_GATE) is [2][D] chosen per row.
  int lin(cudaStream_t s, const void* xin, int64_t rows, int64_t k, const Mat& w, int64_t wrow, int64_t n,
          int epi, void* y, int64_t ldy, float* resid, const float* gate, int64_t ldr = 0) {
    nd_linear_args a{};
    a.dtype = lt;
    a.epilogue = epi;
    a.rows = rows;
    a.in_features = k;
    a.out_features = n;
    a.x = xin;
    a.ldx = k * pw;
    weight_args(a, w, wrow);
    a.group_split = gate ? n_img : rows;
    a.shared_weights = 1;
    a.y = y;
    a.ldy = ldy * pw;
    a.residual = resid;
    a.ldr = ldr > 0 ? ldr : D;
    a.gate = gate;
    a.gate_stride = D;
    a.eps = eps;
    return linear(a, s);
  }

  int mod(cudaStream_t s, const float* scale, int64_t rows) {
    nd_modulate_args m{};
    m.x = x;
    m.ldx = D;
    m.y = xn;
    m.ldy = static_cast<int64_t>(D) * pw;
    m.out_dtype = lt;
    m.rows = rows;
    m.width = D;
    m.shift = nullptr;
    m.scale = scale;
    m.vec_stride = D;
    m.group_split = n_img;
    m.eps = eps;
    return modulate(m, s);
  }

  int gv(cudaStream_t s, const Mat& w, int64_t wrow, int64_t n, int64_t k, const float* xin, int batch,
         bool pre_silu, int act, float* y) {
    nd_gemv_args g{};
    g.w = w.at(wrow, 2);
    g.w_dtype = w.q8 ? ND_I8 : lt;
    g.n = n;
    g.k = k;
    g.x = xin;
    g.batch = batch;
    g.pre_silu = pre_silu ? 1 : 0;
    g.act = act;
    g.y = y;
    if (w.q8) {
      g.scales = w.scales_at(wrow, w.cols / qgroup(w.cols), qf16());
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

  double gemm_flops(double m, double n, double k) const { return 2.0 * m * n * k; }
  double gemm_bytes(double m, double n, double k, double out_bytes) const {
    return 2.0 * (m * k + n * k) + out_bytes;
  }

  int attend(cudaStream_t s, int64_t q_row0, int64_t q_rows, int64_t kv_row0, int64_t kv_rows, int64_t key_limit,
             bool causal) {
    nd_attention_args a{};
    a.dtype = dt;
    a.out_dtype = f32 ? ND_BF16X2 : 0;
    a.heads = H;
    a.head_dim = 128;
    a.batch = 1;
    a.q_rows = q_rows;
    a.kv_rows = kv_rows;
    a.key_limit = key_limit;
    a.causal = causal ? 1 : 0;
    const size_t row_bytes = static_cast<size_t>(3) * D * qe;
    uint8_t* base = static_cast<uint8_t*>(qkv);
    a.q = base + q_row0 * row_bytes;
    a.ldq = 3 * D;
    a.k = base + kv_row0 * row_bytes + static_cast<size_t>(D) * qe;
    a.ldk = 3 * D;
    a.v = base + kv_row0 * row_bytes + static_cast<size_t>(2 * D) * qe;
    a.ldv = 3 * D;
    a.out = static_cast<uint8_t*>(attn) + q_row0 * static_cast<size_t>(D) * 2 * pw;
    a.ldo = static_cast<int64_t>(D) * pw;
    use_attn_workspace(a);
    return attention(a, s);
  }

  int block(cudaStream_t s, int b) {
    const double mD = static_cast<double>(M) * D;
    const double mod_bytes = mD * (4.0 + 2.0);
    const float* scale_attn = mods;
    const float* gate_attn = mods + 2 * D;
    const float* scale_mlp = mods + 4 * D;
    const float* gate_mlp = mods + 6 * D;
    ND_OP("modulate", 0.0, mod_bytes, mod(s, scale_attn, M));
    {
      nd_linear_args a{};
      a.dtype = lt;
      a.epilogue = ND_EPI_QK_NORM_ROPE;
      a.rows = M;
      a.in_features = D;
      a.out_features = 3 * D;
      a.x = xn;
      a.ldx = static_cast<int64_t>(D) * pw;
      weight_args(a, qkv_w, static_cast<int64_t>(b) * 3 * D);
      a.group_split = M;
      a.y = qkv;
      a.ldy = 3 * D;
      a.qk_norm = qk_norm + static_cast<int64_t>(b) * 2 * 128;
      a.rope_cos = in_cos;
      a.rope_sin = in_sin;
      a.qk_cols = 2 * D;
      a.eps = eps;
      ND_OP("gemm.qkv", gemm_flops(M, 3.0 * D, D), gemm_bytes(M, 3.0 * D, D, mD * 3 * 2), linear(a, s));
    }
    // image rows over every visible key; text rows causally over the real text
    const double keys = static_cast<double>(n_img) + real;
    ND_OP("attention", 4.0 * n_img * keys * D, (static_cast<double>(n_img) * 2 + keys * 2) * D * 2,
          attend(s, 0, n_img, 0, M, real < R ? n_img + real : 0, false));
    ND_OP("attention", 2.0 * R * real * D, static_cast<double>(R) * D * 2 * 4,
          attend(s, n_img, R, n_img, R, real < R ? real : 0, true));
    ND_OP("gemm.out", gemm_flops(M, D, D), gemm_bytes(M, D, D, mD * 8),
          lin(s, attn, M, D, out_w, static_cast<int64_t>(b) * D, D, ND_EPI_RESIDUAL_GATE, nullptr, 0, x, gate_attn));
    ND_OP("modulate", 0.0, mod_bytes, mod(s, scale_mlp, M));
    ND_OP("gemm.up", gemm_flops(M, 2.0 * F, D), gemm_bytes(M, 2.0 * F, D, static_cast<double>(M) * F * 2),
          lin(s, xn, M, D, gu_w, static_cast<int64_t>(b) * 2 * F, F, ND_EPI_SWIGLU, hid, F, nullptr, nullptr));
    ND_OP("gemm.down", gemm_flops(M, D, F), gemm_bytes(M, D, F, mD * 8),
          lin(s, hid, M, F, down_w, static_cast<int64_t>(b) * D, D, ND_EPI_RESIDUAL_GATE, nullptr, 0, x, gate_mlp));
    return ND_OK;
  }

  int forward(cudaStream_t s) override {
    const double ni = n_img, dD = D;
    // embeddings: the latent's cells and the text rows into one fp32 sequence
    ND_OP("embed", 0.0, ni * C * 6.0, patchify(in_latent, tok_in, lt, 1, C, Hl, Wl, 1, C * pw, s));
    ND_OP("embed", gemm_flops(ni, dD, C), gemm_bytes(ni, dD, C, ni * dD * 4),
          lin(s, tok_in, n_img, C, img_in_w, 0, D, ND_EPI_STORE_F32, nullptr, 0, x, nullptr));
    {
      nd_rmsnorm_args r{};
      r.x = in_ctx;
      r.ldx = cw;
      r.in_dtype = ND_F32;
      r.y = ctx_n;
      r.ldy = static_cast<int64_t>(cw) * pw;
      r.out_dtype = lt;
      r.rows = R;
      r.width = cw;
      r.weight = txt_norm;
      r.plus_one = 1;  // the stored scale is the weight less one (:463-469)
      r.eps = eps;
      ND_OP("embed", 0.0, static_cast<double>(R) * cw * 6.0, rmsnorm(r, s));
    }
    ND_OP("embed", gemm_flops(R, dD, cw), gemm_bytes(R, dD, cw, R * dD * 2),
          lin(s, ctx_n, R, cw, txt1_w, 0, D, ND_EPI_GELU_TANH, hid, D, nullptr, nullptr));
    ND_OP("embed", gemm_flops(R, dD, dD), gemm_bytes(R, dD, dD, R * dD * 4),
          lin(s, hid, R, D, txt2_w, 0, D, ND_EPI_STORE_F32, nullptr, 0, x + static_cast<int64_t>(n_img) * D, nullptr));
    // the two times (noise level, zero) -> temb [2, D] -> the shared modulation
    ND_OP("gemv", 2.0 * 2 * dD * tw, dD * tw * 2, gv(s, t1_w, 0, D, tw, in_tsin, 2, false, 1, temb_h));
    ND_OP("gemv", 2.0 * 2 * dD * dD, dD * dD * 2, gv(s, t2_w, 0, D, D, temb_h, 2, false, 0, temb));
    for (int c = 0; c < 4; ++c)  // [chunk][time row][D]; the gates (chunks 1, 3) through tanh
      ND_OP("gemv", 2.0 * 2 * dD * dD, dD * dD * 2,
            gv(s, mod_w, static_cast<int64_t>(c) * D, D, D, temb, 2, true, c & 1 ? 2 : 0, mods + c * 2 * D));
    for (int b = 0; b < NB; ++b) {
      int rc = block(s, b);
      if (rc) return rc;
    }
    // final layer over the image rows: LayerNorm * (1 + scale) -> proj_out (:497-505)
    ND_OP("gemv", 2.0 * dD * dD, dD * dD * 2, gv(s, norm_out_w, 0, D, D, temb, 1, true, 0, fscale));
    {
      nd_modulate_args m{};
      m.x = x;
      m.ldx = D;
      m.y = xn;
      m.ldy = static_cast<int64_t>(D) * pw;
      m.out_dtype = lt;
      m.rows = n_img;
      m.width = D;
      m.scale = fscale;
      m.shift = nullptr;
      m.vec_stride = D;
      m.group_split = n_img;
      m.eps = eps;
      ND_OP("modulate", 0.0, ni * dD * 6.0, modulate(m, s));
    }
    ND_OP("embed", gemm_flops(ni, C, dD), gemm_bytes(ni, C, dD, ni * C * 4),
          lin(s, xn, n_img, D, proj_out_w, 0, C, ND_EPI_STORE_F32, nullptr, 0, out_tok, nullptr, C));
    ND_OP("embed", 0.0, ni * C * 8.0, unpatchify(out_tok, C, out_latent, 1, C, Hl, Wl, 1, s));
    return ND_OK;
  }
#undef ND_OP
};

}  // namespace

nd_denoiser* make_qwen_image() { return new QwenImage(); }

}  // namespace nd
