// The SDXL UNet denoiser step: UNetModel (Models/Sdxl/UNetModel.cs) on the
// library's kernels, NHWC activations in fp16 (or bf16).
//
// Per step (UNetModel.Build, :333-437): time and add embeddings (Linear-SiLU-
// Linear each, summed), conv_in, levels going down (ResBlocks, Transformer2D
// where the level has depth, stride-2 downsample), the mid block, levels going
// up (each unit first joins the newest skip connection), GroupNorm + SiLU,
// conv_out. A ResBlock (:230-254) is GroupNorm+SiLU -> conv3x3 (+ the time
// projection, folded into conv1's per-image bias) -> GroupNorm+SiLU ->
// conv3x3 + shortcut (1x1 conv when the width changes), the add fused in the
// conv's epilogue. A Transformer2D (:279-301) is GroupNorm -> proj_in -> blocks
// (LayerNorm -> self-attention; LayerNorm -> cross-attention to the 77 text
// rows; LayerNorm -> GEGLU feed-forward; every residual an fp32 reduce-add
// into the token stream) -> proj_out + the image residual.
//
// Limits of this implementation: latent sides such that every level's width
// divides 128 and each image's pixels per level are a multiple of 128 (the
// implicit-GEMM conv's tiles), weights stored fp16/bf16.
#include <cmath>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_runtime.h"

namespace nd {

namespace {

constexpr int kGroups = 32;
constexpr float kResEps = 1e-5f;    // ResBlock GroupNorm
constexpr float kT2dEps = 1e-6f;    // Transformer2D GroupNorm
constexpr float kLnEps = 1e-5f;     // nn.LayerNorm in the transformer blocks
constexpr int kTembWidth = 1280;

struct ResUnit {
  int cin = 0, cout = 0;
  float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr, *c1b = nullptr, *c2b = nullptr,
        *scb = nullptr, *tpb = nullptr;
  void *c1w = nullptr, *c2w = nullptr, *scw = nullptr;
  int64_t tp_off = 0;  // row offset in the stacked time projections
};

struct TBlock {
  float *n1w, *n1b, *n2w, *n2b, *n3w, *n3b, *o1b, *o2b, *f1b, *f2b;
  void *qkv, *o1, *q2, *kv2, *o2, *f1, *f2;
  int64_t kv_col;  // this block's K columns in the step's merged context K/V (V follows at + C)
};

struct T2d {
  int C = 0;
  float *nw = nullptr, *nb = nullptr, *pib = nullptr, *pob = nullptr;
  void *pin = nullptr, *pout = nullptr;
  std::vector<TBlock> blocks;
};

// UNetModel.TimestepEmbedding (Models/Sdxl/UNetModel.cs:171-188): cosines
// then sines of t * 10000^(-i/half), angles in double.
void timestep_embedding(double t, int dim, float* out) {
  const int half = dim / 2;
  for (int i = 0; i < half; ++i) {
    const double frequency = std::exp(-std::log(10000.0) * i / half);
    const double angle = t * frequency;
    out[i] = static_cast<float>(std::cos(angle));
    out[half + i] = static_cast<float>(std::sin(angle));
  }
}

struct Unet final : nd_denoiser {
  int B = 1, H0 = 0, W0 = 0, C0 = 320, L = 3, R = 2, ctx = 77, cw = 2048, aw = 2816, tw = 320, cinp = 64;
  int mult[4] = {1, 2, 4, 0}, depth[4] = {0, 2, 10, 0};
  int dt = ND_F16;
  size_t e = 2;
  // embeddings
  void *cin_w = nullptr, *cout_w = nullptr, *t1w = nullptr, *t2w = nullptr, *a1w = nullptr, *a2w = nullptr, *tproj = nullptr;
  float *cin_b = nullptr, *cout_b = nullptr, *t1b = nullptr, *t2b = nullptr, *a1b = nullptr, *a2b = nullptr,
        *tproj_b = nullptr, *tproj_bc = nullptr, *onw = nullptr, *onb = nullptr;
  int64_t tproj_rows = 0;
  std::vector<std::vector<ResUnit>> down_res, up_res;
  std::vector<std::vector<T2d>> down_t2d, up_t2d;
  std::vector<void*> down_w, up_w;
  std::vector<float*> down_b, up_b;
  ResUnit mid_res[2];
  T2d mid_t2d;
  // inputs
  float *in_latent = nullptr, *in_tsin = nullptr, *in_add = nullptr, *in_ctx = nullptr;
  float* tsin = nullptr;  // pinned [B][tw]
  // activations
  std::vector<void*> skips;
  std::vector<int> skip_c;
  void *xin = nullptr, *X0 = nullptr, *X1 = nullptr, *H1 = nullptr, *H2 = nullptr, *SC = nullptr, *CAT = nullptr,
       *UPB = nullptr, *A16 = nullptr, *QKV = nullptr, *ATT = nullptr, *Q2 = nullptr, *KV2 = nullptr,
       *FFG = nullptr, *CTX16 = nullptr;
  void* kv_all = nullptr;    // [kv_rows, cw]: every block's attn2 to_k then to_v rows
  int64_t kv_rows = 0, kv_next = 0;
  float *TOK = nullptr, *te1 = nullptr, *te = nullptr, *ae1 = nullptr, *ae = nullptr, *temb = nullptr,
        *rbias = nullptr, *out_nhwc = nullptr, *out_latent = nullptr;
  void* gn_scratch = nullptr;
  size_t gn_scratch_bytes = 0;

  int level_c(int l) const { return C0 * mult[l]; }
  int level_h(int l) const { return H0 >> l; }
  int level_w(int l) const { return W0 >> l; }

  float* V(int64_t n) { return static_cast<float*>(alloc(static_cast<size_t>(n) * 4, true)); }
  void* Wt(int64_t n) { return alloc(static_cast<size_t>(n) * e, true); }

  void conv_slot(const std::string& name, int cout, int cin, void*& w, float*& b, int cin_pad = 0) {
    const int cp = cin_pad ? cin_pad : cin;
    w = Wt(static_cast<int64_t>(cout) * 9 * cp);
    b = V(cout);
    add_slot(name + ".weight", kConv3x3, cout, 9LL * cp, w);
    slots.back().conv_cin = cin;
    add_slot(name + ".bias", kVector, cout, 1, b, false);
  }

  ResUnit make_res(const std::string& p, int cin, int cout) {
    ResUnit r;
    r.cin = cin;
    r.cout = cout;
    r.n1w = V(cin);
    r.n1b = V(cin);
    add_slot(p + ".norm1.weight", kVector, cin, 1, r.n1w);
    add_slot(p + ".norm1.bias", kVector, cin, 1, r.n1b, false);
    conv_slot(p + ".conv1", cout, cin, r.c1w, r.c1b);
    r.tp_off = tproj_rows;
    tproj_rows += cout;
    r.n2w = V(cout);
    r.n2b = V(cout);
    add_slot(p + ".norm2.weight", kVector, cout, 1, r.n2w);
    add_slot(p + ".norm2.bias", kVector, cout, 1, r.n2b, false);
    conv_slot(p + ".conv2", cout, cout, r.c2w, r.c2b);
    if (cin != cout) {
      r.scw = Wt(static_cast<int64_t>(cout) * cin);
      r.scb = V(cout);
      add_slot(p + ".conv_shortcut.weight", kMatrix, cout, cin, r.scw);
      add_slot(p + ".conv_shortcut.bias", kVector, cout, 1, r.scb, false);
    }
    return r;
  }

  T2d make_t2d(const std::string& p, int C, int dep) {
    T2d t;
    t.C = C;
    t.nw = V(C);
    t.nb = V(C);
    add_slot(p + ".norm.weight", kVector, C, 1, t.nw);
    add_slot(p + ".norm.bias", kVector, C, 1, t.nb, false);
    t.pin = Wt(static_cast<int64_t>(C) * C);
    t.pib = V(C);
    add_slot(p + ".proj_in.weight", kMatrix, C, C, t.pin);
    add_slot(p + ".proj_in.bias", kVector, C, 1, t.pib, false);
    for (int j = 0; j < dep; ++j) {
      const std::string q = p + ".transformer_blocks." + std::to_string(j);
      TBlock b{};
      const int64_t CC = static_cast<int64_t>(C) * C;
      b.n1w = V(C); b.n1b = V(C); b.n2w = V(C); b.n2b = V(C); b.n3w = V(C); b.n3b = V(C);
      add_slot(q + ".norm1.weight", kVector, C, 1, b.n1w);
      add_slot(q + ".norm1.bias", kVector, C, 1, b.n1b, false);
      add_slot(q + ".norm2.weight", kVector, C, 1, b.n2w);
      add_slot(q + ".norm2.bias", kVector, C, 1, b.n2b, false);
      add_slot(q + ".norm3.weight", kVector, C, 1, b.n3w);
      add_slot(q + ".norm3.bias", kVector, C, 1, b.n3b, false);
      b.qkv = Wt(3 * CC);
      add_slot(q + ".attn1.to_q.weight", kMatrix, C, C, b.qkv);
      add_slot(q + ".attn1.to_k.weight", kMatrix, C, C, static_cast<uint8_t*>(b.qkv) + CC * e);
      add_slot(q + ".attn1.to_v.weight", kMatrix, C, C, static_cast<uint8_t*>(b.qkv) + 2 * CC * e);
      b.o1 = Wt(CC);
      b.o1b = V(C);
      add_slot(q + ".attn1.to_out.0.weight", kMatrix, C, C, b.o1);
      add_slot(q + ".attn1.to_out.0.bias", kVector, C, 1, b.o1b, false);
      b.q2 = Wt(CC);
      add_slot(q + ".attn2.to_q.weight", kMatrix, C, C, b.q2);
      // every block's context K/V weights in one matrix: one GEMM per step
      b.kv_col = kv_next;
      b.kv2 = static_cast<uint8_t*>(kv_all) + kv_next * cw * e;
      kv_next += 2LL * C;
      add_slot(q + ".attn2.to_k.weight", kMatrix, C, cw, b.kv2);
      add_slot(q + ".attn2.to_v.weight", kMatrix, C, cw, static_cast<uint8_t*>(b.kv2) + static_cast<int64_t>(C) * cw * e);
      b.o2 = Wt(CC);
      b.o2b = V(C);
      add_slot(q + ".attn2.to_out.0.weight", kMatrix, C, C, b.o2);
      add_slot(q + ".attn2.to_out.0.bias", kVector, C, 1, b.o2b, false);
      b.f1 = Wt(8 * CC);
      b.f1b = V(8LL * C);
      add_slot(q + ".ff.net.0.proj.weight", kMatrix, 8LL * C, C, b.f1);
      add_slot(q + ".ff.net.0.proj.bias", kVector, 8LL * C, 1, b.f1b, false);
      b.f2 = Wt(4 * CC);
      b.f2b = V(C);
      add_slot(q + ".ff.net.2.weight", kMatrix, C, 4LL * C, b.f2);
      add_slot(q + ".ff.net.2.bias", kVector, C, 1, b.f2b, false);
      t.blocks.push_back(b);
    }
    t.pout = Wt(static_cast<int64_t>(C) * C);
    t.pob = V(C);
    add_slot(p + ".proj_out.weight", kMatrix, C, C, t.pout);
    add_slot(p + ".proj_out.bias", kVector, C, 1, t.pob, false);
    return t;
  }

  int build() override {
    const nd_model_desc& d = desc;
    if (d.compute != ND_F16 && d.compute != ND_BF16) return fail(ND_ERR_UNSUPPORTED, "sdxl: compute must be fp16 or bf16");
    if (d.weight_dtype != d.compute) return fail(ND_ERR_UNSUPPORTED, "sdxl: weights must be stored in the compute dtype");
    if (d.batch < 1 || d.batch > 4) return fail(ND_ERR_INVALID, "sdxl: batch must be 1..4");
    if (d.head_dim != 0 && d.head_dim != 64) return fail(ND_ERR_UNSUPPORTED, "sdxl: heads are 64 wide");
    dt = d.compute;
    B = d.batch;
    C0 = d.width > 0 ? d.width : 320;
    H0 = d.latent_height;
    W0 = d.latent_width;
    ctx = d.context_rows > 0 ? d.context_rows : 77;
    cw = d.context_width > 0 ? d.context_width : 2048;
    aw = d.add_width > 0 ? d.add_width : 2816;
    tw = d.time_width > 0 ? d.time_width : C0;
    if (d.unet_levels > 0) {
      if (d.unet_levels > 4) return fail(ND_ERR_INVALID, "sdxl: at most 4 levels");
      L = d.unet_levels;
      for (int l = 0; l < L; ++l) {
        mult[l] = d.unet_mult[l];
        depth[l] = d.unet_depth[l];
      }
      R = d.unet_resnets > 0 ? d.unet_resnets : 2;
    }
    if (d.latent_channels != 4) return fail(ND_ERR_INVALID, "sdxl: the latent has 4 channels");
    if (C0 % 64 || aw % 8 || cw % 8 || tw % 8) return fail(ND_ERR_INVALID, "sdxl: widths must be multiples of 64 / 8");
    for (int l = 0; l < L; ++l) {
      if (mult[l] <= 0) return fail(ND_ERR_INVALID, "sdxl: level multipliers must be positive");
      const int h = level_h(l), w = level_w(l);
      if ((H0 >> l) << l != H0 || (W0 >> l) << l != W0 || w > 128 || 128 % w != 0 || (h * w) % 128 != 0)
        return fail(ND_ERR_UNSUPPORTED, "sdxl: every level's width must divide 128 and its pixels be a multiple of 128");
    }
    e = 2;
    const int64_t px0 = static_cast<int64_t>(B) * H0 * W0;

    // ---- weights (diffusers' SDXL UNet tensor names)
    conv_slot("conv_in", C0, d.latent_channels, cin_w, cin_b, cinp);
    t1w = Wt(static_cast<int64_t>(kTembWidth) * tw);
    t1b = V(kTembWidth);
    t2w = Wt(static_cast<int64_t>(kTembWidth) * kTembWidth);
    t2b = V(kTembWidth);
    a1w = Wt(static_cast<int64_t>(kTembWidth) * aw);
    a1b = V(kTembWidth);
    a2w = Wt(static_cast<int64_t>(kTembWidth) * kTembWidth);
    a2b = V(kTembWidth);
    add_slot("time_embedding.linear_1.weight", kMatrix, kTembWidth, tw, t1w);
    add_slot("time_embedding.linear_1.bias", kVector, kTembWidth, 1, t1b, false);
    add_slot("time_embedding.linear_2.weight", kMatrix, kTembWidth, kTembWidth, t2w);
    add_slot("time_embedding.linear_2.bias", kVector, kTembWidth, 1, t2b, false);
    add_slot("add_embedding.linear_1.weight", kMatrix, kTembWidth, aw, a1w);
    add_slot("add_embedding.linear_1.bias", kVector, kTembWidth, 1, a1b, false);
    add_slot("add_embedding.linear_2.weight", kMatrix, kTembWidth, kTembWidth, a2w);
    add_slot("add_embedding.linear_2.bias", kVector, kTembWidth, 1, a2b, false);

    // the context K/V rows of every transformer block (2C each), in build order
    kv_rows = 0;
    for (int l = 0; l < L; ++l)
      if (depth[l] > 0) kv_rows += static_cast<int64_t>(R) * depth[l] * 2 * level_c(l);
    kv_rows += static_cast<int64_t>(depth[L - 1] > 0 ? depth[L - 1] : 1) * 2 * level_c(L - 1);
    for (int l = 0; l < L; ++l)
      if (depth[l] > 0) kv_rows += static_cast<int64_t>(R + 1) * depth[l] * 2 * level_c(l);
    kv_all = Wt(kv_rows * cw);
    kv_next = 0;

    std::vector<int> chans, levels;  // channels and level of every skip, in push order
    chans.push_back(C0);
    levels.push_back(0);
    int c = C0;
    down_res.resize(L);
    down_t2d.resize(L);
    for (int l = 0; l < L; ++l) {
      const std::string p = "down_blocks." + std::to_string(l);
      const int co = level_c(l);
      for (int i = 0; i < R; ++i) {
        down_res[l].push_back(make_res(p + ".resnets." + std::to_string(i), c, co));
        c = co;
        if (depth[l] > 0) down_t2d[l].push_back(make_t2d(p + ".attentions." + std::to_string(i), co, depth[l]));
        chans.push_back(co);
        levels.push_back(l);
      }
      if (l != L - 1) {
        void* w;
        float* b;
        conv_slot(p + ".downsamplers.0.conv", co, co, w, b);
        down_w.push_back(w);
        down_b.push_back(b);
        chans.push_back(co);
        levels.push_back(l + 1);
      }
    }
    mid_res[0] = make_res("mid_block.resnets.0", c, c);
    mid_t2d = make_t2d("mid_block.attentions.0", c, depth[L - 1] > 0 ? depth[L - 1] : 1);
    mid_res[1] = make_res("mid_block.resnets.1", c, c);
    up_res.resize(L);
    up_t2d.resize(L);
    std::vector<int> stack = chans;
    for (int i = 0; i < L; ++i) {
      const int l = L - 1 - i;
      const std::string p = "up_blocks." + std::to_string(i);
      const int co = level_c(l);
      for (int j = 0; j < R + 1; ++j) {
        const int skip = stack.back();
        stack.pop_back();
        up_res[l].push_back(make_res(p + ".resnets." + std::to_string(j), c + skip, co));
        c = co;
        if (depth[l] > 0) up_t2d[l].push_back(make_t2d(p + ".attentions." + std::to_string(j), co, depth[l]));
      }
      if (i != L - 1) {
        void* w;
        float* b;
        conv_slot(p + ".upsamplers.0.conv", co, co, w, b);
        up_w.push_back(w);
        up_b.push_back(b);
      }
    }
    onw = V(c);
    onb = V(c);
    add_slot("conv_norm_out.weight", kVector, c, 1, onw);
    add_slot("conv_norm_out.bias", kVector, c, 1, onb, false);
    conv_slot("conv_out", d.latent_channels, c, cout_w, cout_b);

    // every ResBlock's time projection, stacked for one GEMV per step
    tproj = Wt(tproj_rows * kTembWidth);
    tproj_b = V(tproj_rows);
    tproj_bc = V(tproj_rows);
    auto register_tproj = [&](const std::string& p, const ResUnit& r) {
      add_slot(p + ".time_emb_proj.weight", kMatrix, r.cout, kTembWidth,
               static_cast<uint8_t*>(tproj) + r.tp_off * kTembWidth * e);
      add_slot(p + ".time_emb_proj.bias", kVector, r.cout, 1, tproj_b + r.tp_off, false);
    };
    for (int l = 0; l < L; ++l)
      for (int i = 0; i < R; ++i) register_tproj("down_blocks." + std::to_string(l) + ".resnets." + std::to_string(i), down_res[l][i]);
    register_tproj("mid_block.resnets.0", mid_res[0]);
    register_tproj("mid_block.resnets.1", mid_res[1]);
    for (int i = 0; i < L; ++i)
      for (int j = 0; j < R + 1; ++j)
        register_tproj("up_blocks." + std::to_string(i) + ".resnets." + std::to_string(j), up_res[L - 1 - i][j]);

    // ---- inputs, skips and work buffers
    auto S = [&](size_t bytes) { return alloc(bytes, false); };
    in_latent = static_cast<float*>(S(static_cast<size_t>(B) * 4 * H0 * W0 * 4));
    in_tsin = static_cast<float*>(S(static_cast<size_t>(B) * tw * 4));
    in_add = static_cast<float*>(S(static_cast<size_t>(B) * aw * 4));
    in_ctx = static_cast<float*>(S(static_cast<size_t>(B) * ctx * cw * 4));
    tsin = static_cast<float*>(pinned(static_cast<size_t>(B) * tw * 4));
    for (size_t k = 0; k < chans.size(); ++k) {
      skips.push_back(S(static_cast<size_t>(B) * level_h(levels[k]) * level_w(levels[k]) * chans[k] * e));
      skip_c.push_back(chans[k]);
    }
    int64_t max_act = 0;  // elements of the largest NHWC activation (incl. concat)
    int64_t max_tok = 0, max_ff = 0, max_qkv = 0;
    for (int l = 0; l < L; ++l) {
      const int64_t px = static_cast<int64_t>(B) * level_h(l) * level_w(l);
      max_act = std::max<int64_t>(max_act, px * (level_c(l) + (l + 1 < L ? level_c(l + 1) : level_c(l)) + level_c(l)));
      max_act = std::max<int64_t>(max_act, px * 4LL * level_c(l));
      if (depth[l] > 0 || l == L - 1) {
        max_tok = std::max<int64_t>(max_tok, px * level_c(l));
        max_qkv = std::max<int64_t>(max_qkv, px * 3LL * level_c(l));
        max_ff = std::max<int64_t>(max_ff, px * 8LL * level_c(l));
      }
    }
    xin = S(static_cast<size_t>(px0) * cinp * e);
    X0 = S(max_act * e);
    X1 = S(max_act * e);
    H1 = S(max_act * e);
    H2 = S(max_act * e);
    SC = S(max_act * e);
    CAT = S(max_act * e);
    UPB = S(max_act * e);
    A16 = S(max_tok * e);
    TOK = static_cast<float*>(S(max_tok * 4));
    QKV = S(max_qkv * e);
    ATT = S(max_tok * e);
    Q2 = S(max_tok * e);
    if (kv_next != kv_rows) return fail(ND_ERR_INVALID, "sdxl: context K/V row count mismatch");
    KV2 = S(static_cast<size_t>(B) * ctx * kv_rows * e);
    FFG = S(max_ff / 2 * e);  // the GEGLU GEMM writes h * gelu(g) directly
    CTX16 = S(static_cast<size_t>(B) * ctx * cw * e);
    te1 = static_cast<float*>(S(static_cast<size_t>(B) * kTembWidth * 4));
    te = static_cast<float*>(S(static_cast<size_t>(B) * kTembWidth * 4));
    ae1 = static_cast<float*>(S(static_cast<size_t>(B) * kTembWidth * 4));
    ae = static_cast<float*>(S(static_cast<size_t>(B) * kTembWidth * 4));
    temb = static_cast<float*>(S(static_cast<size_t>(B) * kTembWidth * 4));
    rbias = static_cast<float*>(S(static_cast<size_t>(B) * tproj_rows * 4));
    out_nhwc = static_cast<float*>(S(static_cast<size_t>(px0) * 4 * 4));
    out_latent = static_cast<float*>(S(static_cast<size_t>(px0) * 4 * 4));
    size_t gsz = 0;
    for (int l = 0; l < L; ++l)
      gsz = std::max(gsz, group_norm_scratch(B, level_h(l) * level_w(l), static_cast<int>(max_act / (static_cast<int64_t>(B) * level_h(l) * level_w(l))), kGroups));
    gn_scratch_bytes = gsz;
    gn_scratch = S(gsz);
    if (desc.compute != ND_F32) alloc_attn_workspace(64);
    if (alloc_failed) return fail(ND_ERR_OOM, "sdxl: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));
    return ND_OK;
  }

  int prepare() override {
    // conv1's bias joins the time projection's: one per-image bias vector.
    cudaStream_t s = dev->stream;
    ND_CUDA(cudaMemcpyAsync(tproj_bc, tproj_b, static_cast<size_t>(tproj_rows) * 4, cudaMemcpyDeviceToDevice, s));
    auto fold = [&](const ResUnit& r) -> int { return add_vectors(tproj_bc + r.tp_off, r.c1b, r.cout, s); };
    for (int l = 0; l < L; ++l)
      for (auto& r : down_res[l]) ND_TRY_RC(fold(r));
    ND_TRY_RC(fold(mid_res[0]));
    ND_TRY_RC(fold(mid_res[1]));
    for (int l = 0; l < L; ++l)
      for (auto& r : up_res[l]) ND_TRY_RC(fold(r));
    ND_CUDA(cudaStreamSynchronize(s));
    return ND_OK;
  }

  int64_t latent_elems() const override { return static_cast<int64_t>(B) * 4 * H0 * W0; }
  const float* output() const override { return out_latent; }

  int check_cond(int n, const nd_named_tensor* cond, StepInputs& in) override {
    const float* add = nullptr;
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
      } else if (name == "add") {
        if (t.dtype != ND_F32 || elems != static_cast<int64_t>(B) * aw)
          return fail(ND_ERR_INVALID, "predict: add must be f32 [" + std::to_string(B) + ", " + std::to_string(aw) + "]");
        add = static_cast<const float*>(t.data);
      } else {
        return fail(ND_ERR_INVALID, "predict: unknown conditioning " + name);
      }
    }
    if (!in.context || !add) return fail(ND_ERR_INVALID, "predict: conditioning needs \"context\" and \"add\"");
    in.cos = add;  // carried to stage() (the UNet has no rotary tables)
    return ND_OK;
  }

  int stage(const StepInputs& in, cudaStream_t s) override {
    const cudaMemcpyKind k = in.device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    ND_CUDA(cudaMemcpyAsync(in_latent, in.latent, static_cast<size_t>(latent_elems()) * 4, k, s));
    ND_CUDA(cudaMemcpyAsync(in_ctx, in.context, static_cast<size_t>(B) * ctx * cw * 4, k, s));
    ND_CUDA(cudaMemcpyAsync(in_add, in.cos, static_cast<size_t>(B) * aw * 4, k, s));
    ND_CUDA(cudaEventSynchronize(staged));
    for (int b = 0; b < B; ++b) timestep_embedding(in.timestep, tw, tsin + static_cast<size_t>(b) * tw);
    ND_CUDA(cudaMemcpyAsync(in_tsin, tsin, static_cast<size_t>(B) * tw * 4, cudaMemcpyHostToDevice, s));
    ND_CUDA(cudaEventRecord(staged, s));
    return ND_OK;
  }

#define ND_OP(cls, flops, expr)     \
  do {                              \
    prof_begin(s);                  \
    int rc_ = (expr);               \
    if (rc_) return rc_;            \
    prof_end(s, cls, flops, 0.0);   \
  } while (0)

  int gn(cudaStream_t s, const void* x, void* y, int l, int C, const float* w, const float* b, float eps, int silu) {
    return group_norm(x, y, dt, B, level_h(l) * level_w(l), C, kGroups, w, b, eps, silu, gn_scratch,
                      gn_scratch_bytes, s);
  }

  int conv(cudaStream_t s, const void* x, int l_in, int cin, int stride, const void* w, const float* b,
           int cout, int epi, void* y, const void* addend, const float* batch_bias = nullptr,
           int64_t bias_stride = 0, float* y32 = nullptr) {
    nd_conv_args c{};
    c.dtype = dt;
    c.epilogue = epi;
    c.batch = B;
    c.height = level_h(l_in);
    c.width = level_w(l_in);
    c.in_channels = cin;
    c.out_channels = cout;
    c.stride = stride;
    c.x = x;
    c.weight = w;
    c.bias = batch_bias ? batch_bias : b;
    c.per_batch_bias = batch_bias ? 1 : 0;
    c.bias_stride = bias_stride;
    c.y = y;
    c.y_f32 = y32;
    c.addend = addend;
    return conv2d(c, s);
  }

  int lin(cudaStream_t s, const void* x, int64_t rows, int64_t k, const void* w, const float* b, int64_t n, int epi,
          void* y, float* resid = nullptr, const void* addend = nullptr) {
    nd_linear_args a{};
    a.dtype = dt;
    a.epilogue = epi;
    a.rows = rows;
    a.in_features = k;
    a.out_features = n;
    a.x = x;
    a.ldx = k;
    a.weight = w;
    a.bias = b;
    a.group_split = rows;
    a.y = y;
    a.ldy = n;
    a.residual = resid;
    a.ldr = n;
    a.addend = addend;
    a.ld_add = n;
    return linear(a, s);
  }

  double conv_flops(int l_out, int cin, int cout) const {
    return 2.0 * B * level_h(l_out) * level_w(l_out) * 9.0 * cin * cout;
  }

  // ResBlock at level l: x [B, HW, cin] -> y [B, HW, cout].
  int res(cudaStream_t s, const ResUnit& r, int l, const void* x, void* y) {
    const int64_t px = static_cast<int64_t>(B) * level_h(l) * level_w(l);
    ND_OP("groupnorm", 0.0, gn(s, x, H1, l, r.cin, r.n1w, r.n1b, kResEps, 1));
    ND_OP("conv3x3", conv_flops(l, r.cin, r.cout),
          conv(s, H1, l, r.cin, 1, r.c1w, nullptr, r.cout, ND_EPI_STORE, H2, nullptr, rbias + r.tp_off, tproj_rows));
    ND_OP("groupnorm", 0.0, gn(s, H2, H1, l, r.cout, r.n2w, r.n2b, kResEps, 1));
    const void* sc = x;
    if (r.scw) {
      ND_OP("gemm.shortcut", 2.0 * px * r.cin * r.cout, lin(s, x, px, r.cin, r.scw, r.scb, r.cout, ND_EPI_STORE, SC));
      sc = SC;
    }
    ND_OP("conv3x3", conv_flops(l, r.cout, r.cout),
          conv(s, H1, l, r.cout, 1, r.c2w, r.c2b, r.cout, ND_EPI_ADD_STORE, y, sc));
    return ND_OK;
  }

  // Transformer2D at level l: x [B, HW, C] -> y (x + the blocks' output).
  int t2d(cudaStream_t s, const T2d& t, int l, const void* x, void* y) {
    const int C = t.C;
    const int hw = level_h(l) * level_w(l);
    const int64_t M = static_cast<int64_t>(B) * hw;
    const int heads = C / 64;
    ND_OP("groupnorm", 0.0, gn(s, x, A16, l, C, t.nw, t.nb, kT2dEps, 0));
    ND_OP("gemm.proj", 2.0 * M * C * C, lin(s, A16, M, C, t.pin, t.pib, C, ND_EPI_STORE_F32, nullptr, TOK));
    for (const TBlock& b : t.blocks) {
      // self-attention
      ND_OP("layernorm", 0.0, ln(s, M, C, b.n1w, b.n1b));
      ND_OP("gemm.qkv", 6.0 * M * C * C, lin(s, A16, M, C, b.qkv, nullptr, 3LL * C, ND_EPI_STORE, QKV));
      ND_OP("attention", 4.0 * B * static_cast<double>(hw) * hw * C,
            attend(s, QKV, 3LL * C, static_cast<uint8_t*>(QKV) + C * e, static_cast<uint8_t*>(QKV) + 2 * C * e,
                   3LL * C, heads, hw, hw));
      ND_OP("gemm.out", 2.0 * M * C * C, lin(s, ATT, M, C, b.o1, b.o1b, C, ND_EPI_RESIDUAL_ADD, nullptr, TOK));
      // cross-attention to the text rows
      ND_OP("layernorm", 0.0, ln(s, M, C, b.n2w, b.n2b));
      ND_OP("gemm.cross_q", 2.0 * M * C * C, lin(s, A16, M, C, b.q2, nullptr, C, ND_EPI_STORE, Q2));
      ND_OP("attention", 4.0 * B * static_cast<double>(hw) * ctx * C,
            attend(s, Q2, C, static_cast<uint8_t*>(KV2) + b.kv_col * e, static_cast<uint8_t*>(KV2) + (b.kv_col + C) * e,
                   kv_rows, heads, hw, ctx));
      ND_OP("gemm.out", 2.0 * M * C * C, lin(s, ATT, M, C, b.o2, b.o2b, C, ND_EPI_RESIDUAL_ADD, nullptr, TOK));
      // GEGLU feed-forward
      ND_OP("layernorm", 0.0, ln(s, M, C, b.n3w, b.n3b));
      ND_OP("gemm.up", 16.0 * M * C * C, lin(s, A16, M, C, b.f1, b.f1b, 4LL * C, ND_EPI_GEGLU, FFG));
      ND_OP("gemm.down", 8.0 * M * C * C, lin(s, FFG, M, 4LL * C, b.f2, b.f2b, C, ND_EPI_RESIDUAL_ADD, nullptr, TOK));
    }
    ND_OP("convert", 0.0, convert(TOK, ND_F32, A16, dt, M * C, s));
    ND_OP("gemm.proj", 2.0 * M * C * C, lin(s, A16, M, C, t.pout, t.pob, C, ND_EPI_ADD_STORE, y, nullptr, x));
    return ND_OK;
  }

  int ln(cudaStream_t s, int64_t M, int C, const float* w, const float* b) {
    nd_modulate_args m{};
    m.x = TOK;
    m.ldx = C;
    m.y = A16;
    m.ldy = C;
    m.out_dtype = dt;
    m.rows = M;
    m.width = C;
    m.shift = b;
    m.scale = w;
    m.vec_stride = C;
    m.group_split = M;
    m.eps = kLnEps;
    m.affine = 1;
    return modulate(m, s);
  }

  int attend(cudaStream_t s, const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int heads,
             int q_rows, int kv_rows) {
    nd_attention_args a{};
    a.dtype = dt;
    a.heads = heads;
    a.head_dim = 64;
    a.batch = B;
    a.q_rows = q_rows;
    a.kv_rows = kv_rows;
    a.q = q;
    a.ldq = ldq;
    a.k = k;
    a.ldk = ldkv;
    a.v = v;
    a.ldv = ldkv;
    a.out = ATT;
    a.ldo = static_cast<int64_t>(heads) * 64;
    use_attn_workspace(a);
    return attention(a, s);
  }

  int forward(cudaStream_t s) override {
    PdlScope pdl(true);  // over a thousand short launches: overlap each one's launch with the previous
    const int64_t px0 = static_cast<int64_t>(B) * H0 * W0;
    // embeddings
    ND_OP("layout", 0.0, nchw_to_nhwc(in_latent, xin, dt, B, 4, H0 * W0, cinp, s));
    ND_OP("layout", 0.0, convert(in_ctx, ND_F32, CTX16, dt, static_cast<int64_t>(B) * ctx * cw, s));
    // every block's cross-attention K and V of the (step-constant) context
    ND_OP("gemm.cross_kv", 2.0 * B * ctx * static_cast<double>(kv_rows) * cw,
          lin(s, CTX16, static_cast<int64_t>(B) * ctx, cw, kv_all, nullptr, kv_rows, ND_EPI_STORE, KV2));
    ND_OP("gemv", 0.0, gv(s, t1w, kTembWidth, tw, in_tsin, t1b, false, 1, te1));
    ND_OP("gemv", 0.0, gv(s, t2w, kTembWidth, kTembWidth, te1, t2b, false, 0, te));
    ND_OP("gemv", 0.0, gv(s, a1w, kTembWidth, aw, in_add, a1b, false, 1, ae1));
    ND_OP("gemv", 0.0, gv(s, a2w, kTembWidth, kTembWidth, ae1, a2b, false, 0, ae));
    ND_OP("gemv", 0.0, add_vectors2(temb, te, ae, static_cast<int64_t>(B) * kTembWidth, s));
    ND_OP("gemv", 0.0, gv(s, tproj, tproj_rows, kTembWidth, temb, tproj_bc, true, 0, rbias));
    // down
    int k = 0;
    ND_OP("conv3x3", conv_flops(0, cinp, C0), conv(s, xin, 0, cinp, 1, cin_w, cin_b, C0, ND_EPI_STORE, skips[k++], nullptr));
    const void* x = skips[0];
    for (int l = 0; l < L; ++l) {
      for (int i = 0; i < R; ++i) {
        void* out = skips[k];
        if (depth[l] > 0) {
          ND_TRY_RC(res(s, down_res[l][i], l, x, X0));
          ND_TRY_RC(t2d(s, down_t2d[l][i], l, X0, out));
        } else {
          ND_TRY_RC(res(s, down_res[l][i], l, x, out));
        }
        x = out;
        ++k;
      }
      if (l != L - 1) {
        ND_OP("conv3x3", conv_flops(l + 1, level_c(l), level_c(l)),
              conv(s, x, l, level_c(l), 2, down_w[l], down_b[l], level_c(l), ND_EPI_STORE, skips[k], nullptr));
        x = skips[k++];
      }
    }
    // mid
    const int lm = L - 1, cm = level_c(lm);
    ND_TRY_RC(res(s, mid_res[0], lm, x, X0));
    ND_TRY_RC(t2d(s, mid_t2d, lm, X0, X1));
    ND_TRY_RC(res(s, mid_res[1], lm, X1, X0));
    void* cur = X0;
    void* other = X1;
    int c = cm;
    (void)c;
    // up
    for (int i = 0; i < L; ++i) {
      const int l = L - 1 - i;
      const int64_t px = static_cast<int64_t>(B) * level_h(l) * level_w(l);
      for (int j = 0; j < R + 1; ++j) {
        --k;
        const ResUnit& r = up_res[l][j];
        ND_OP("concat", 0.0, concat_channels(cur, r.cin - skip_c[k], skips[k], skip_c[k], CAT, px, s));
        ND_TRY_RC(res(s, r, l, CAT, other));
        std::swap(cur, other);
        if (depth[l] > 0) {
          ND_TRY_RC(t2d(s, up_t2d[l][j], l, cur, other));
          std::swap(cur, other);
        }
      }
      if (i != L - 1) {
        const int co = level_c(l);
        ND_OP("upsample", 0.0, upsample2x(cur, UPB, B, level_h(l), level_w(l), co, s));
        ND_OP("conv3x3", conv_flops(l - 1, co, co),
              conv(s, UPB, l - 1, co, 1, up_w[i], up_b[i], co, ND_EPI_STORE, other, nullptr));
        std::swap(cur, other);
      }
    }
    // out
    ND_OP("groupnorm", 0.0, gn(s, cur, H1, 0, level_c(0), onw, onb, kResEps, 1));
    ND_OP("conv3x3", conv_flops(0, level_c(0), 4),
          conv(s, H1, 0, level_c(0), 1, cout_w, cout_b, 4, ND_EPI_STORE_F32, nullptr, nullptr, nullptr, 0, out_nhwc));
    ND_OP("layout", 0.0, nhwc_to_nchw(out_nhwc, out_latent, B, 4, H0 * W0, s));
    (void)px0;
    return ND_OK;
  }
#undef ND_OP

  int gv(cudaStream_t s, const void* w, int64_t n, int64_t k, const float* x, const float* b, bool pre_silu, int act,
         float* y) {
    nd_gemv_args g{};
    g.w = w;
    g.w_dtype = dt;
    g.n = n;
    g.k = k;
    g.x = x;
    g.batch = B;
    g.pre_silu = pre_silu ? 1 : 0;
    g.bias = b;
    g.act = act;
    g.y = y;
    return gemv(g, s);
  }
};

}  // namespace

nd_denoiser* make_unet() { return new Unet(); }

}  // namespace nd
