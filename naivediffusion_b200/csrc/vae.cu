// The AutoencoderKL decoder (the SDXL VAE): AutoencoderKl.Decoder
// (Vae/AutoencoderKl.cs:78-116) on the library's kernels, NHWC activations in
// fp16 (or bf16), one latent in, one [3, 8h, 8w] image out.
//
// post_quant_conv (1x1, applied per pixel while the latent is laid out NHWC)
// -> conv_in -> mid block (ResnetBlock, single-head self-attention over every
// pixel, ResnetBlock) -> up blocks (layers_per_block + 1 ResnetBlocks each,
// nearest 2x upsample + conv3x3 between them) -> GroupNorm + SiLU -> conv_out.
// ResnetBlock (:16-36): GroupNorm+SiLU -> conv3x3 -> GroupNorm+SiLU -> conv3x3
// + shortcut (1x1 when the width changes), the add in the conv's epilogue.
// Attention (:40-66): GroupNorm -> q, k, v Linear -> softmax(q k^T / sqrt(C))
// v -> out Linear + the residual; run as the reference runs it, two GEMMs
// around a row softmax (one head of width C, so the flash kernel's 64 / 128
// head widths do not apply): the scores in fp32, the probabilities in the
// compute type.
#include <algorithm>
#include <climits>
#include <cmath>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_common.cuh"
#include "nd_runtime.h"

namespace nd {

namespace {

constexpr int kVaeGroups = 32;
constexpr int kLatentPad = 64;  // conv_in's input channels, zero-padded

// NCHW fp32 latent [B, 4, HW] -> post_quant_conv (1x1: y = P x + p) -> NHWC
// 16-bit [B, HW, 64] with channels 4..63 zero.
__global__ void vae_latent_in_kernel(const float* __restrict__ in, const float* __restrict__ pq_w,
                                     const float* __restrict__ pq_b, void* __restrict__ out, int f16, int B,
                                     int HW) {
  const long long n = static_cast<long long>(B) * HW;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / HW);
    const int p = static_cast<int>(i - static_cast<long long>(b) * HW);
    float x[4], y[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) x[c] = in[(static_cast<long long>(b) * 4 + c) * HW + p];
#pragma unroll
    for (int o = 0; o < 4; ++o) {
      float acc = pq_b[o];
#pragma unroll
      for (int c = 0; c < 4; ++c) acc = fmaf(pq_w[o * 4 + c], x[c], acc);
      y[o] = acc;
    }
    uint32_t w[32];
    w[0] = f16 ? pack_f16(y[0], y[1]) : pack_bf16(y[0], y[1]);
    w[1] = f16 ? pack_f16(y[2], y[3]) : pack_bf16(y[2], y[3]);
#pragma unroll
    for (int k = 2; k < 32; ++k) w[k] = 0u;
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + i * kLatentPad);
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  }
}

// NHWC fp32 [B, HW, 4] (conv_out, its 4th channel a zero pad) -> NCHW [B, 3, HW].
__global__ void vae_image_out_kernel(const float* __restrict__ in, float* __restrict__ out, int B, int HW) {
  const long long n = static_cast<long long>(B) * 3 * HW;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(i % HW);
    const long long bc = i / HW;
    const int c = static_cast<int>(bc % 3);
    const long long b = bc / 3;
    out[i] = in[(b * HW + p) * 4 + c];
  }
}

// Row softmax of fp32 scores times `scale`, written in the compute type:
// p = exp(s * scale - max) / sum (DmlOps.ActivationSoftmax over the last axis
// of the alpha-scaled scores). One block per row.
__global__ void __launch_bounds__(256) vae_softmax_kernel(const float* __restrict__ s, void* __restrict__ p,
                                                          int f16, int cols, float scale) {
  __shared__ float red[8];
  const float* row = s + static_cast<long long>(blockIdx.x) * cols;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  float mx = -INFINITY;
  for (int c = t; c < cols; c += 256) mx = fmaxf(mx, row[c] * scale);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[w] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) mx = fmaxf(mx, red[k]);
  __syncthreads();
  float sum = 0.f;
  for (int c = t; c < cols; c += 256) sum += expf(row[c] * scale - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[w] = sum;
  __syncthreads();
  sum = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) sum += red[k];
  const float inv = 1.0f / sum;
  uint16_t* out = static_cast<uint16_t*>(p) + static_cast<long long>(blockIdx.x) * cols;
  for (int c = t; c < cols; c += 256) {
    const float v = expf(row[c] * scale - mx) * inv;
    if (f16) {
      const __half h = __float2half_rn(v);
      out[c] = *reinterpret_cast<const uint16_t*>(&h);
    } else {
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      out[c] = *reinterpret_cast<const uint16_t*>(&h);
    }
  }
}

// [rows, cols] 16-bit -> [cols, rows], 32 x 32 tiles through shared memory.
__global__ void transpose16_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, int rows, int cols) {
  __shared__ uint16_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[k][threadIdx.x] = in[static_cast<long long>(r) * cols + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[static_cast<long long>(c) * rows + r] = tile[threadIdx.x][k];
  }
}

unsigned grid_of(long long n) {
  return static_cast<unsigned>(std::max<long long>(1, std::min<long long>((n + 255) / 256, sm_count() * 16LL)));
}

struct VaeRes {
  int cin = 0, cout = 0;
  float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr, *c1b = nullptr, *c2b = nullptr,
        *scb = nullptr;
  void *c1w = nullptr, *c2w = nullptr, *scw = nullptr;
};

struct VaeDecoder final : nd_denoiser {
  int B = 1, h0 = 0, w0 = 0, C0 = 128, L = 4, R = 2;
  int mult[4] = {1, 2, 4, 4};
  int dt = ND_F16;
  size_t e = 2;
  float eps = 1e-6f;
  // weights
  float *pq_w = nullptr, *pq_b = nullptr, *cin_b = nullptr, *onw = nullptr, *onb = nullptr, *cout_b = nullptr;
  void *cin_w = nullptr, *cout_w = nullptr;
  VaeRes mid_res[2];
  float *an_w = nullptr, *an_b = nullptr, *aq_b = nullptr, *ak_b = nullptr, *av_b = nullptr, *ao_b = nullptr;
  void *aq = nullptr, *ak = nullptr, *av = nullptr, *ao = nullptr;
  std::vector<std::vector<VaeRes>> up_res;
  std::vector<void*> up_w;
  std::vector<float*> up_b;
  // buffers
  float *in_latent = nullptr, *out_nhwc = nullptr, *out_image = nullptr, *scores = nullptr;
  void *xin = nullptr, *X0 = nullptr, *X1 = nullptr, *H1 = nullptr, *H2 = nullptr, *SC = nullptr, *UPB = nullptr,
       *Q = nullptr, *K = nullptr, *Vb = nullptr, *VT = nullptr, *P = nullptr, *ATT = nullptr, *A16 = nullptr;
  void* gn_scratch = nullptr;
  size_t gn_scratch_bytes = 0;

  // decoder up block i runs at 2^i times the latent's resolution, with width rev(i)
  int rev(int i) const { return C0 * mult[L - 1 - i]; }
  int res_h(int i) const { return h0 << i; }
  int res_w(int i) const { return w0 << i; }

  float* V(int64_t n) { return static_cast<float*>(alloc(static_cast<size_t>(n) * 4, true)); }
  void* Wt(int64_t n) { return alloc(static_cast<size_t>(n) * e, true); }

  void conv_slot(const std::string& name, int cout, int cin, void*& w, float*& b, int cin_pad = 0, int cout_pad = 0) {
    const int cp = cin_pad ? cin_pad : cin;
    w = Wt(static_cast<int64_t>(cout_pad ? cout_pad : cout) * 9 * cp);
    b = V(cout_pad ? cout_pad : cout);
    add_slot(name + ".weight", kConv3x3, cout, 9LL * cp, w);
    slots.back().conv_cin = cin;
    add_slot(name + ".bias", kVector, cout, 1, b, false);
  }

  VaeRes make_res(const std::string& p, int cin, int cout) {
    VaeRes r;
    r.cin = cin;
    r.cout = cout;
    r.n1w = V(cin);
    r.n1b = V(cin);
    add_slot(p + ".norm1.weight", kVector, cin, 1, r.n1w);
    add_slot(p + ".norm1.bias", kVector, cin, 1, r.n1b, false);
    conv_slot(p + ".conv1", cout, cin, r.c1w, r.c1b);
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

  int build() override {
    const nd_model_desc& d = desc;
    if (d.compute != ND_F16 && d.compute != ND_BF16) return fail(ND_ERR_UNSUPPORTED, "vae: compute must be fp16 or bf16");
    if (d.weight_dtype != d.compute) return fail(ND_ERR_UNSUPPORTED, "vae: weights must be stored in the compute dtype");
    if (d.latent_channels != 4) return fail(ND_ERR_INVALID, "vae: the latent has 4 channels");
    if (d.batch < 1 || d.batch > 64) return fail(ND_ERR_INVALID, "vae: batch must be 1..64");
    dt = d.compute;
    B = d.batch;
    C0 = d.width > 0 ? d.width : 128;
    h0 = d.latent_height;
    w0 = d.latent_width;
    eps = d.eps > 0 ? d.eps : 1e-6f;
    if (d.unet_levels > 0) {
      if (d.unet_levels > 4) return fail(ND_ERR_INVALID, "vae: at most 4 levels");
      L = d.unet_levels;
      for (int l = 0; l < L; ++l) mult[l] = d.unet_mult[l];
      R = d.unet_resnets > 0 ? d.unet_resnets : 2;
    }
    if (C0 % 64) return fail(ND_ERR_INVALID, "vae: width must be a multiple of 64");
    for (int i = 0; i < L; ++i) {
      if (mult[i] <= 0) return fail(ND_ERR_INVALID, "vae: level multipliers must be positive");
      const int w = res_w(i), h = res_h(i);
      if ((w <= 128 ? 128 % w != 0 : w % 128 != 0) || (static_cast<int64_t>(h) * w) % 128 != 0)
        return fail(ND_ERR_UNSUPPORTED, "vae: every level's width must divide 128 or be a multiple of 128");
    }
    const int top = rev(0);
    if (static_cast<int64_t>(h0) * w0 % 128) return fail(ND_ERR_UNSUPPORTED, "vae: latent pixels must be a multiple of 128");

    // ---- weights (diffusers' AutoencoderKL names)
    pq_w = V(16);
    pq_b = V(4);
    add_slot("post_quant_conv.weight", kVector, 16, 1, pq_w);
    add_slot("post_quant_conv.bias", kVector, 4, 1, pq_b, false);
    conv_slot("decoder.conv_in", top, 4, cin_w, cin_b, kLatentPad);
    mid_res[0] = make_res("decoder.mid_block.resnets.0", top, top);
    const std::string ap = "decoder.mid_block.attentions.0";
    an_w = V(top);
    an_b = V(top);
    add_slot(ap + ".group_norm.weight", kVector, top, 1, an_w);
    add_slot(ap + ".group_norm.bias", kVector, top, 1, an_b, false);
    const int64_t tt = static_cast<int64_t>(top) * top;
    aq = Wt(tt);
    ak = Wt(tt);
    av = Wt(tt);
    ao = Wt(tt);
    aq_b = V(top);
    ak_b = V(top);
    av_b = V(top);
    ao_b = V(top);
    add_slot(ap + ".to_q.weight", kMatrix, top, top, aq);
    add_slot(ap + ".to_q.bias", kVector, top, 1, aq_b, false);
    add_slot(ap + ".to_k.weight", kMatrix, top, top, ak);
    add_slot(ap + ".to_k.bias", kVector, top, 1, ak_b, false);
    add_slot(ap + ".to_v.weight", kMatrix, top, top, av);
    add_slot(ap + ".to_v.bias", kVector, top, 1, av_b, false);
    add_slot(ap + ".to_out.0.weight", kMatrix, top, top, ao);
    add_slot(ap + ".to_out.0.bias", kVector, top, 1, ao_b, false);
    mid_res[1] = make_res("decoder.mid_block.resnets.1", top, top);
    up_res.resize(L);
    int c = top;
    for (int i = 0; i < L; ++i) {
      const std::string p = "decoder.up_blocks." + std::to_string(i);
      const int co = rev(i);
      for (int j = 0; j < R + 1; ++j) {
        up_res[i].push_back(make_res(p + ".resnets." + std::to_string(j), c, co));
        c = co;
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
    add_slot("decoder.conv_norm_out.weight", kVector, c, 1, onw);
    add_slot("decoder.conv_norm_out.bias", kVector, c, 1, onb, false);
    conv_slot("decoder.conv_out", 3, c, cout_w, cout_b, 0, 4);  // row 4 stays zero

    // ---- buffers
    auto S = [&](size_t bytes) { return alloc(bytes, false); };
    const int64_t lat_px = static_cast<int64_t>(B) * h0 * w0;
    const int64_t img_px = static_cast<int64_t>(B) * res_h(L - 1) * res_w(L - 1);
    int64_t max_act = 0;
    for (int i = 0; i < L; ++i) {
      const int64_t px = static_cast<int64_t>(B) * res_h(i) * res_w(i);
      const int cprev = i == 0 ? top : rev(i - 1);
      max_act = std::max<int64_t>(max_act, px * std::max(cprev, rev(i)));
    }
    in_latent = static_cast<float*>(S(static_cast<size_t>(lat_px) * 4 * 4));
    xin = S(static_cast<size_t>(lat_px) * kLatentPad * e);
    X0 = S(max_act * e);
    X1 = S(max_act * e);
    H1 = S(max_act * e);
    H2 = S(max_act * e);
    SC = S(max_act * e);
    UPB = S(max_act * e);
    const int64_t hw = static_cast<int64_t>(h0) * w0;
    Q = S(hw * top * e);
    K = S(hw * top * e);
    Vb = S(hw * top * e);
    VT = S(hw * top * e);
    ATT = S(hw * top * e);
    A16 = S(lat_px * top * e);
    scores = static_cast<float*>(S(static_cast<size_t>(hw) * hw * 4));
    P = S(static_cast<size_t>(hw) * hw * e);
    out_nhwc = static_cast<float*>(S(static_cast<size_t>(img_px) * 4 * 4));
    out_image = static_cast<float*>(S(static_cast<size_t>(img_px) * 3 * 4));
    size_t gsz = 0;
    for (int i = 0; i < L; ++i)
      gsz = std::max(gsz, group_norm_scratch(B, res_h(i) * res_w(i), std::max(top, rev(i)), kVaeGroups));
    gn_scratch_bytes = gsz;
    gn_scratch = S(gsz);
    if (alloc_failed) return fail(ND_ERR_OOM, "vae: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));
    return ND_OK;
  }

  int64_t latent_elems() const override { return static_cast<int64_t>(B) * 4 * h0 * w0; }
  int64_t output_elems() const override { return static_cast<int64_t>(B) * 3 * res_h(L - 1) * res_w(L - 1); }
  const float* output() const override { return out_image; }

  int check_cond(int n, const nd_named_tensor* cond, StepInputs&) override {
    if (n != 0 || cond) {
      (void)cond;
      if (n != 0) return fail(ND_ERR_INVALID, "vae decode takes no conditioning");
    }
    return ND_OK;
  }

  int stage(const StepInputs& in, cudaStream_t s) override {
    const cudaMemcpyKind k = in.device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    ND_CUDA(cudaMemcpyAsync(in_latent, in.latent, static_cast<size_t>(latent_elems()) * 4, k, s));
    return ND_OK;
  }

#define ND_OP(cls, flops, expr)     \
  do {                              \
    prof_begin(s);                  \
    int rc_ = (expr);               \
    if (rc_) return rc_;            \
    prof_end(s, cls, flops, 0.0);   \
  } while (0)

  int gn(cudaStream_t s, const void* x, void* y, int i, int C, const float* w, const float* b, int silu, int hw = 0) {
    return group_norm(x, y, dt, B, hw ? hw : res_h(i) * res_w(i), C, kVaeGroups, w, b, eps, silu, gn_scratch,
                      gn_scratch_bytes, s);
  }

  int conv(cudaStream_t s, const void* x, int hh, int ww, int cin, const void* w, const float* b, int cout, int epi,
           void* y, const void* addend, float* y32 = nullptr) {
    nd_conv_args c{};
    c.dtype = dt;
    c.epilogue = epi;
    c.batch = B;
    c.height = hh;
    c.width = ww;
    c.in_channels = cin;
    c.out_channels = cout;
    c.stride = 1;
    c.x = x;
    c.weight = w;
    c.bias = b;
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

  double conv_flops(int hh, int ww, int cin, int cout) const { return 2.0 * B * hh * ww * 9.0 * cin * cout; }

  int res(cudaStream_t s, const VaeRes& r, int hh, int ww, const void* x, void* y) {
    const int64_t px = static_cast<int64_t>(B) * hh * ww;
    ND_OP("groupnorm", 0.0, gn(s, x, H1, 0, r.cin, r.n1w, r.n1b, 1, hh * ww));
    ND_OP("conv3x3", conv_flops(hh, ww, r.cin, r.cout), conv(s, H1, hh, ww, r.cin, r.c1w, r.c1b, r.cout, ND_EPI_STORE, H2, nullptr));
    ND_OP("groupnorm", 0.0, gn(s, H2, H1, 0, r.cout, r.n2w, r.n2b, 1, hh * ww));
    const void* sc = x;
    if (r.scw) {
      ND_OP("gemm.shortcut", 2.0 * px * r.cin * r.cout, lin(s, x, px, r.cin, r.scw, r.scb, r.cout, ND_EPI_STORE, SC));
      sc = SC;
    }
    ND_OP("conv3x3", conv_flops(hh, ww, r.cout, r.cout),
          conv(s, H1, hh, ww, r.cout, r.c2w, r.c2b, r.cout, ND_EPI_ADD_STORE, y, sc));
    return ND_OK;
  }

  // Single-head attention over the hw pixels of each image, plus the residual.
  int attn(cudaStream_t s, const void* x, void* y) {
    const int C = rev(0);
    const int64_t hw = static_cast<int64_t>(h0) * w0;
    ND_OP("groupnorm", 0.0, gn(s, x, A16, 0, C, an_w, an_b, 0, static_cast<int>(hw)));
    const float scale = 1.0f / std::sqrt(static_cast<float>(C));
    for (int b = 0; b < B; ++b) {
      const uint8_t* xb = static_cast<const uint8_t*>(A16) + b * hw * C * e;
      ND_OP("gemm.qkv", 2.0 * hw * C * C, lin(s, xb, hw, C, aq, aq_b, C, ND_EPI_STORE, Q));
      ND_OP("gemm.qkv", 2.0 * hw * C * C, lin(s, xb, hw, C, ak, ak_b, C, ND_EPI_STORE, K));
      ND_OP("gemm.qkv", 2.0 * hw * C * C, lin(s, xb, hw, C, av, av_b, C, ND_EPI_STORE, Vb));
      ND_OP("attention", 2.0 * hw * hw * C, lin(s, Q, hw, C, K, nullptr, hw, ND_EPI_STORE_F32, nullptr, scores));
      ND_OP("attention", 0.0, softmax(s, hw, scale));
      ND_OP("attention", 0.0, transpose(s, Vb, VT, hw, C));
      ND_OP("attention", 2.0 * hw * hw * C, lin(s, P, hw, hw, VT, nullptr, C, ND_EPI_STORE, ATT));
      const uint8_t* xres = static_cast<const uint8_t*>(x) + b * hw * C * e;
      uint8_t* yb = static_cast<uint8_t*>(y) + b * hw * C * e;
      ND_OP("gemm.out", 2.0 * hw * C * C, lin(s, ATT, hw, C, ao, ao_b, C, ND_EPI_ADD_STORE, yb, nullptr, xres));
    }
    return ND_OK;
  }

  int softmax(cudaStream_t s, int64_t rows, float scale) {
    if (rows > INT_MAX) return fail(ND_ERR_INVALID, "vae: too many pixels for the attention");
    vae_softmax_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(scores, P, dt == ND_F16, static_cast<int>(rows), scale);
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }

  int transpose(cudaStream_t s, const void* in, void* out, int64_t rows, int cols) {
    dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
    transpose16_kernel<<<grid, dim3(32, 8), 0, s>>>(static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out),
                                                   static_cast<int>(rows), cols);
    ND_CUDA(cudaGetLastError());
    return ND_OK;
  }

  int forward(cudaStream_t s) override {
    const int top = rev(0);
    const int64_t lat_px = static_cast<int64_t>(B) * h0 * w0;
    prof_begin(s);
    vae_latent_in_kernel<<<grid_of(lat_px), 256, 0, s>>>(in_latent, pq_w, pq_b, xin, dt == ND_F16, B, h0 * w0);
    ND_CUDA(cudaGetLastError());
    prof_end(s, "layout", 0.0, 0.0);
    ND_OP("conv3x3", conv_flops(h0, w0, kLatentPad, top),
          conv(s, xin, h0, w0, kLatentPad, cin_w, cin_b, top, ND_EPI_STORE, X0, nullptr));
    ND_TRY_RC(res(s, mid_res[0], h0, w0, X0, X1));
    ND_TRY_RC(attn(s, X1, X0));
    ND_TRY_RC(res(s, mid_res[1], h0, w0, X0, X1));
    void* cur = X1;
    void* other = X0;
    for (int i = 0; i < L; ++i) {
      const int hh = res_h(i), ww = res_w(i);
      for (int j = 0; j < R + 1; ++j) {
        ND_TRY_RC(res(s, up_res[i][j], hh, ww, cur, other));
        std::swap(cur, other);
      }
      if (i != L - 1) {
        const int co = rev(i);
        ND_OP("upsample", 0.0, upsample2x(cur, UPB, B, hh, ww, co, s));
        ND_OP("conv3x3", conv_flops(2 * hh, 2 * ww, co, co),
              conv(s, UPB, 2 * hh, 2 * ww, co, up_w[i], up_b[i], co, ND_EPI_STORE, other, nullptr));
        std::swap(cur, other);
      }
    }
    const int hh = res_h(L - 1), ww = res_w(L - 1), c = rev(L - 1);
    ND_OP("groupnorm", 0.0, gn(s, cur, H1, L - 1, c, onw, onb, 1));
    ND_OP("conv3x3", conv_flops(hh, ww, c, 3),
          conv(s, H1, hh, ww, c, cout_w, cout_b, 4, ND_EPI_STORE_F32, nullptr, nullptr, out_nhwc));
    const int64_t img_px = static_cast<int64_t>(B) * hh * ww;
    prof_begin(s);
    vae_image_out_kernel<<<grid_of(img_px * 3), 256, 0, s>>>(out_nhwc, out_image, B, hh * ww);
    ND_CUDA(cudaGetLastError());
    prof_end(s, "layout", 0.0, 0.0);
    return ND_OK;
  }
#undef ND_OP
};

// ------------------------------------------------------------ Wan decoders
// WanVae.Decoder (Vae/WanVae.cs:170-207, the Wan 2.1 VAE Anima decodes with)
// and Wan22Vae.Decoder (Vae/Wan22Vae.cs:161-206, Qwen-Image 2.1's), on one
// frame: every causal 3-D convolution cut to its last temporal tap (the host
// passes WanVae.SingleFrame's tensors), an RMS norm over each pixel's channels
// instead of GroupNorm, SiLU, a single-head attention in the middle. The
// level channel plan follows the checkpoints: dims = width x [m_last, m
// reversed]; Wan 2.1 halves the width in each upsample convolution (the next
// level's resblocks start from half), Wan 2.2 keeps it and adds a shortcut of
// the level's input beside every upsampling level.

// NCHW fp32 latent [B, C, HW] -> conv2 (1x1: y = W x + b) -> NHWC 16-bit
// [B, HW, Cp] with channels C..Cp-1 zero (the 3x3 conv reads whole 64-channel chunks).
__global__ void wan_latent_in_kernel(const float* __restrict__ in, const float* __restrict__ w,
                                     const float* __restrict__ b, void* __restrict__ out, int f16, int B, int HW,
                                     int C, int Cp) {
  const long long n = static_cast<long long>(B) * HW * Cp;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int o = static_cast<int>(i % Cp);
    const long long pix = i / Cp;
    const int bi = static_cast<int>(pix / HW);
    const int p = static_cast<int>(pix - static_cast<long long>(bi) * HW);
    float acc = 0.f;
    if (o < C) {
      acc = b[o];
      for (int c = 0; c < C; ++c) acc = fmaf(w[o * C + c], in[(static_cast<long long>(bi) * C + c) * HW + p], acc);
    }
    uint16_t* dst = static_cast<uint16_t*>(out) + i;
    if (f16) {
      const __half h = __float2half_rn(acc);
      *dst = *reinterpret_cast<const uint16_t*>(&h);
    } else {
      const __nv_bfloat16 h = __float2bfloat16_rn(acc);
      *dst = *reinterpret_cast<const uint16_t*>(&h);
    }
  }
}

__device__ __forceinline__ void unpack8v(const uint4& u, int f16, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[i]))
                         : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8v(const float (&v)[8], int f16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = f16 ? pack_f16(v[2 * i], v[2 * i + 1]) : pack_bf16(v[2 * i], v[2 * i + 1]);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float ld16(const uint16_t* p, int f16) {
  const uint16_t v = *p;
  return f16 ? __half2float(*reinterpret_cast<const __half*>(&v))
             : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&v));
}

// h [B, 2H, 2W, Co] += Wan22Vae.UpShortcut(x [B, H, W, Ci]) (Vae/Wan22Vae.cs:121-155):
// mode 0 (Ci == Co) nearest upsample; mode 1 (a level that doubled time,
// Ci == 2 Co) the odd input channels, nearest; mode 2 (Ci == 2 Co) output
// channel c takes input channel 2c on even rows and 2c + 1 on odd rows.
__global__ void wan_up_shortcut_kernel(void* __restrict__ h, const void* __restrict__ x, int f16, int B, int H,
                                       int W, int Ci, int Co, int mode) {
  const long long n = static_cast<long long>(B) * 4 * H * W * Co;
  uint16_t* hp = static_cast<uint16_t*>(h);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % Co);
    long long q = i / Co;
    const int X = static_cast<int>(q % (2 * W));
    q /= 2 * W;
    const int Y = static_cast<int>(q % (2 * H));
    const long long b = q / (2 * H);
    const int sc = mode == 0 ? c : (mode == 1 ? 2 * c + 1 : 2 * c + (Y & 1));
    const long long src = ((b * H + (Y >> 1)) * W + (X >> 1)) * Ci + sc;
    const float v = ld16(hp + i, f16) + ld16(xp + src, f16);
    if (f16) {
      const __half r = __float2half_rn(v);
      hp[i] = *reinterpret_cast<const uint16_t*>(&r);
    } else {
      const __nv_bfloat16 r = __float2bfloat16_rn(v);
      hp[i] = *reinterpret_cast<const uint16_t*>(&r);
    }
  }
}

// The same, 8 output channels per thread (Co % 8 == 0): one 16-byte load of
// h, one (mode 0) or two (modes 1, 2: the 16 input channels 2c .. 2c+15) of x.
__global__ void wan_up_shortcut8_kernel(uint4* __restrict__ h, const uint4* __restrict__ x, int f16, int B, int H,
                                        int W, int Ci, int Co, int mode) {
  const int co8 = Co / 8, ci8 = Ci / 8;
  const long long n = static_cast<long long>(B) * 4 * H * W * co8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % co8);
    long long q = i / co8;
    const int X = static_cast<int>(q % (2 * W));
    q /= 2 * W;
    const int Y = static_cast<int>(q % (2 * H));
    const long long b = q / (2 * H);
    const long long src = ((b * H + (Y >> 1)) * W + (X >> 1)) * ci8;
    float hv[8], xv[8];
    unpack8v(h[i], f16, hv);
    if (mode == 0) {
      unpack8v(__ldg(x + src + c), f16, xv);
    } else {
      float lo[8], hi[8];
      unpack8v(__ldg(x + src + 2 * c), f16, lo);
      unpack8v(__ldg(x + src + 2 * c + 1), f16, hi);
      const int odd = mode == 1 ? 1 : (Y & 1);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        xv[k] = lo[2 * k + odd];
        xv[4 + k] = hi[2 * k + odd];
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) hv[k] += xv[k];
    h[i] = pack8v(hv, f16);
  }
}

struct WanRes {
  int cin = 0, cout = 0;
  float *g1 = nullptr, *g2 = nullptr, *c1b = nullptr, *c2b = nullptr, *scb = nullptr;
  void *c1w = nullptr, *c2w = nullptr, *scw = nullptr;
};

struct WanLevel {
  int cin = 0, cout = 0, up_out = 0;  // up_out 0: no upsample
  int sc_mode = -1;                   // Wan 2.2 shortcut mode (-1: none)
  std::vector<WanRes> res;
  void* upw = nullptr;
  float* upb = nullptr;
};

int round64(int c) { return (c + 63) / 64 * 64; }

struct WanDecoder final : nd_denoiser {
  bool v22 = false;
  int B = 1, h0 = 0, w0 = 0, Cl = 16, Clp = 64, W0 = 96, R = 2, L = 4, top = 0, img_c = 3;
  int dt = ND_F16;
  size_t e = 2;
  float *cv2_w = nullptr, *cv2_b = nullptr, *c1_b = nullptr, *head_g = nullptr, *head_b = nullptr;
  void *c1_w = nullptr, *head_w = nullptr;
  WanRes mid0, mid1;
  float *ag = nullptr, *aqkv_b = nullptr, *ap_b = nullptr;
  void *aqkv = nullptr, *ap = nullptr;
  std::vector<WanLevel> lv;
  float *in_latent = nullptr, *out_nhwc = nullptr, *out_image = nullptr, *scores = nullptr;
  void *xin = nullptr, *X[3] = {nullptr, nullptr, nullptr}, *H1 = nullptr, *H2 = nullptr, *SC = nullptr,
       *UPB = nullptr, *Q = nullptr, *K = nullptr, *Vb = nullptr, *VT = nullptr, *P = nullptr, *ATT = nullptr,
       *A16 = nullptr;

  int res_h(int i) const { return h0 << i; }
  int res_w(int i) const { return w0 << i; }
  float* V(int64_t n) { return static_cast<float*>(alloc(static_cast<size_t>(n) * 4, true)); }
  void* Wt(int64_t n) { return alloc(static_cast<size_t>(n) * e, true); }

  void conv_slot(const std::string& name, int cout, int cin, void*& w, float*& b, int cout_pad = 0) {
    const int cp = round64(cin);
    const int co = cout_pad ? cout_pad : cout;
    w = Wt(static_cast<int64_t>(co) * 9 * cp);
    b = V(co);
    add_slot(name + ".weight", kConv3x3, cout, 9LL * cp, w);
    slots.back().conv_cin = cin;
    add_slot(name + ".bias", kVector, cout, 1, b, false);
  }

  WanRes make_res(const std::string& p, int cin, int cout) {
    WanRes r;
    r.cin = cin;
    r.cout = cout;
    r.g1 = V(cin);
    add_slot(p + ".residual.0.gamma", kVector, cin, 1, r.g1);
    conv_slot(p + ".residual.2", cout, cin, r.c1w, r.c1b);
    r.g2 = V(cout);
    add_slot(p + ".residual.3.gamma", kVector, cout, 1, r.g2);
    conv_slot(p + ".residual.6", cout, cout, r.c2w, r.c2b);
    if (cin != cout) {
      r.scw = Wt(static_cast<int64_t>(cout) * cin);
      r.scb = V(cout);
      add_slot(p + ".shortcut.weight", kMatrix, cout, cin, r.scw);
      add_slot(p + ".shortcut.bias", kVector, cout, 1, r.scb, false);
    }
    return r;
  }

  int build() override {
    const nd_model_desc& d = desc;
    v22 = d.family == ND_FAMILY_VAE_WAN22;
    if (d.compute != ND_F16 && d.compute != ND_BF16) return fail(ND_ERR_UNSUPPORTED, "wan vae: compute must be fp16 or bf16");
    if (d.weight_dtype != d.compute) return fail(ND_ERR_UNSUPPORTED, "wan vae: weights must be stored in the compute dtype");
    if (d.batch < 1 || d.batch > 64) return fail(ND_ERR_INVALID, "wan vae: batch must be 1..64");
    dt = d.compute;
    B = d.batch;
    Cl = d.latent_channels > 0 ? d.latent_channels : (v22 ? 64 : 16);
    if (Cl > 64) return fail(ND_ERR_INVALID, "wan vae: at most 64 latent channels");
    Clp = 64;
    W0 = d.width > 0 ? d.width : (v22 ? 144 : 96);
    R = d.unet_resnets > 0 ? d.unet_resnets : 2;
    h0 = d.latent_height;
    w0 = d.latent_width;
    img_c = v22 ? 4 : 3;
    static const int m21[4] = {1, 2, 4, 4};
    static const int m22[5] = {1, 2, 4, 8, 8};
    const int* m = v22 ? m22 : m21;
    L = v22 ? 5 : 4;
    // dims = width x [m_last, m reversed] (the checkpoints' Decoder3d layout)
    std::vector<int> dims(L + 1);
    dims[0] = W0 * m[L - 1];
    for (int i = 0; i < L; ++i) dims[i + 1] = W0 * m[L - 1 - i];
    top = dims[0];
    for (int c : dims)
      if (c % 8 || c < 64) return fail(ND_ERR_INVALID, "wan vae: every level's width must be a multiple of 8, at least 64");
    for (int i = 0; i < L; ++i) {
      const int w = res_w(i), h = res_h(i);
      if ((w <= 128 ? 128 % w != 0 : w % 128 != 0) || (static_cast<int64_t>(h) * w) % 128 != 0)
        return fail(ND_ERR_UNSUPPORTED, "wan vae: every level's width must divide 128 or be a multiple of 128");
    }
    // ---- weights
    cv2_w = V(static_cast<int64_t>(Cl) * Cl);
    cv2_b = V(Cl);
    add_slot("conv2.weight", kVector, static_cast<int64_t>(Cl) * Cl, 1, cv2_w);
    add_slot("conv2.bias", kVector, Cl, 1, cv2_b, false);
    conv_slot("decoder.conv1", top, Cl, c1_w, c1_b);
    mid0 = make_res("decoder.middle.0", top, top);
    ag = V(top);
    add_slot("decoder.middle.1.norm.gamma", kVector, top, 1, ag);
    aqkv = Wt(3LL * top * top);
    aqkv_b = V(3LL * top);
    add_slot("decoder.middle.1.to_qkv.weight", kMatrix, 3LL * top, top, aqkv);
    add_slot("decoder.middle.1.to_qkv.bias", kVector, 3LL * top, 1, aqkv_b, false);
    ap = Wt(static_cast<int64_t>(top) * top);
    ap_b = V(top);
    add_slot("decoder.middle.1.proj.weight", kMatrix, top, top, ap);
    add_slot("decoder.middle.1.proj.bias", kVector, top, 1, ap_b, false);
    mid1 = make_res("decoder.middle.2", top, top);
    lv.resize(L);
    int idx = 0;  // Wan 2.1 numbers its upsamples straight through
    static const bool temporal22[4] = {false, true, true, true};
    for (int i = 0; i < L; ++i) {
      WanLevel& v = lv[i];
      v.cin = (!v22 && i > 0) ? dims[i] / 2 : dims[i];
      v.cout = dims[i + 1];
      const bool up = i != L - 1;
      v.up_out = up ? (v22 ? v.cout : v.cout / 2) : 0;
      const std::string pre = v22 ? "decoder.upsamples." + std::to_string(i) + ".upsamples." : "decoder.upsamples.";
      if (v22) idx = 0;
      int c = v.cin;
      for (int j = 0; j < R + 1; ++j) {
        v.res.push_back(make_res(pre + std::to_string(idx++), c, v.cout));
        c = v.cout;
      }
      if (up) {
        conv_slot(pre + std::to_string(idx++) + ".resample.1", v.up_out, v.cout, v.upw, v.upb);
        if (v22) {
          if (v.cin == v.up_out) v.sc_mode = 0;
          else if (v.cin == 2 * v.up_out) v.sc_mode = temporal22[L - 2 - i] ? 1 : 2;
          else return fail(ND_ERR_INVALID, "wan vae: an up level halves its channels at most");
        }
      }
      if (!v22 && i > 0 && lv[i - 1].up_out != v.cin)
        return fail(ND_ERR_INVALID, "wan vae: level widths do not chain");
    }
    const int last = lv[L - 1].cout;
    head_g = V(last);
    add_slot("decoder.head.0.gamma", kVector, last, 1, head_g);
    conv_slot("decoder.head.2", img_c, last, head_w, head_b, 4);
    // ---- buffers
    auto S = [&](size_t bytes) { return alloc(bytes, false); };
    const int64_t hw0 = static_cast<int64_t>(h0) * w0;
    const int64_t lat_px = B * hw0;
    int64_t max_act = lat_px * top;
    for (int i = 0; i < L; ++i) {
      const int64_t px = static_cast<int64_t>(B) * res_h(i) * res_w(i);
      max_act = std::max<int64_t>(max_act, px * std::max(lv[i].cin, lv[i].cout));
      if (lv[i].up_out) max_act = std::max<int64_t>(max_act, 4 * px * std::max(lv[i].cout, lv[i].up_out));
    }
    const int64_t img_px = static_cast<int64_t>(B) * res_h(L - 1) * res_w(L - 1);
    in_latent = static_cast<float*>(S(static_cast<size_t>(lat_px) * Cl * 4));
    xin = S(static_cast<size_t>(lat_px) * Clp * e);
    for (auto& x : X) x = S(max_act * e);
    H1 = S(max_act * e);
    H2 = S(max_act * e);
    SC = S(max_act * e);
    UPB = S(max_act * e);
    Q = S(hw0 * top * e);
    K = S(hw0 * top * e);
    Vb = S(hw0 * top * e);
    VT = S(hw0 * top * e);
    ATT = S(hw0 * top * e);
    A16 = S(lat_px * top * e);
    scores = static_cast<float*>(S(static_cast<size_t>(hw0) * hw0 * 4));
    P = S(static_cast<size_t>(hw0) * hw0 * e);
    out_nhwc = static_cast<float*>(S(static_cast<size_t>(img_px) * 4 * 4));
    out_image = static_cast<float*>(S(static_cast<size_t>(img_px) * 3 * 4));
    if (alloc_failed) return fail(ND_ERR_OOM, "wan vae: device allocation failed");
    ND_CUDA(cudaEventCreateWithFlags(&staged, cudaEventDisableTiming));
    return ND_OK;
  }

  int64_t latent_elems() const override { return static_cast<int64_t>(B) * Cl * h0 * w0; }
  int64_t output_elems() const override { return static_cast<int64_t>(B) * 3 * res_h(L - 1) * res_w(L - 1); }
  const float* output() const override { return out_image; }

  int check_cond(int n, const nd_named_tensor*, StepInputs&) override {
    if (n != 0) return fail(ND_ERR_INVALID, "wan vae decode takes no conditioning");
    return ND_OK;
  }

  int stage(const StepInputs& in, cudaStream_t s) override {
    const cudaMemcpyKind k = in.device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    ND_CUDA(cudaMemcpyAsync(in_latent, in.latent, static_cast<size_t>(latent_elems()) * 4, k, s));
    return ND_OK;
  }

#define ND_OP(cls, flops, expr)     \
  do {                              \
    prof_begin(s);                  \
    int rc_ = (expr);               \
    if (rc_) return rc_;            \
    prof_end(s, cls, flops, 0.0);   \
  } while (0)

  // WanVae.ChannelRmsNorm (Vae/WanVae.cs:111-121): each pixel's channels over
  // sqrt(mean(x^2) + 1e-24 / C), times gamma; SiLU after where the block has it.
  int rms(cudaStream_t s, const void* x, void* y, int64_t px, int C, const float* g, bool silu_after) {
    nd_rmsnorm_args a{};
    a.x = x;
    a.ldx = C;
    a.in_dtype = dt;
    a.y = y;
    a.ldy = C;
    a.out_dtype = dt;
    a.rows = px;
    a.width = C;
    a.weight = g;
    a.plus_one = 0;
    a.eps = 1e-24f / static_cast<float>(C);
    a.silu = silu_after ? 1 : 0;
    return rmsnorm(a, s);
  }

  int conv(cudaStream_t s, const void* x, int hh, int ww, int cin, const void* w, const float* b, int cout, int epi,
           void* y, const void* addend, float* y32 = nullptr) {
    nd_conv_args c{};
    c.dtype = dt;
    c.epilogue = epi;
    c.batch = B;
    c.height = hh;
    c.width = ww;
    c.in_channels = cin;
    c.out_channels = cout;
    c.stride = 1;
    c.x = x;
    c.weight = w;
    c.bias = b;
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

  double conv_flops(int hh, int ww, int cin, int cout) const { return 2.0 * B * hh * ww * 9.0 * cin * cout; }

  // WanVae.ResidualBlock (Vae/WanVae.cs:132-146).
  int res(cudaStream_t s, const WanRes& r, int hh, int ww, const void* x, void* y) {
    const int64_t px = static_cast<int64_t>(B) * hh * ww;
    ND_OP("rmsnorm", 0.0, rms(s, x, H1, px, r.cin, r.g1, true));
    ND_OP("conv3x3", conv_flops(hh, ww, r.cin, r.cout), conv(s, H1, hh, ww, r.cin, r.c1w, r.c1b, r.cout, ND_EPI_STORE, H2, nullptr));
    ND_OP("rmsnorm", 0.0, rms(s, H2, H1, px, r.cout, r.g2, true));
    const void* sc = x;
    if (r.scw) {
      ND_OP("gemm.shortcut", 2.0 * px * r.cin * r.cout, lin(s, x, px, r.cin, r.scw, r.scb, r.cout, ND_EPI_STORE, SC));
      sc = SC;
    }
    ND_OP("conv3x3", conv_flops(hh, ww, r.cout, r.cout),
          conv(s, H1, hh, ww, r.cout, r.c2w, r.c2b, r.cout, ND_EPI_ADD_STORE, y, sc));
    return ND_OK;
  }

  // WanVae.AttentionBlock (Vae/WanVae.cs:150-168): one head over every pixel.
  int attn(cudaStream_t s, const void* x, void* y) {
    const int C = top;
    const int64_t hw = static_cast<int64_t>(h0) * w0;
    ND_OP("rmsnorm", 0.0, rms(s, x, A16, B * hw, C, ag, false));
    const float scale = 1.0f / std::sqrt(static_cast<float>(C));
    const size_t wrow = static_cast<size_t>(C) * C * e;
    for (int b = 0; b < B; ++b) {
      const uint8_t* xb = static_cast<const uint8_t*>(A16) + b * hw * C * e;
      const uint8_t* w = static_cast<const uint8_t*>(aqkv);
      ND_OP("gemm.qkv", 2.0 * hw * C * C, lin(s, xb, hw, C, w, aqkv_b, C, ND_EPI_STORE, Q));
      ND_OP("gemm.qkv", 2.0 * hw * C * C, lin(s, xb, hw, C, w + wrow, aqkv_b + C, C, ND_EPI_STORE, K));
      ND_OP("gemm.qkv", 2.0 * hw * C * C, lin(s, xb, hw, C, w + 2 * wrow, aqkv_b + 2 * C, C, ND_EPI_STORE, Vb));
      ND_OP("attention", 2.0 * hw * hw * C, lin(s, Q, hw, C, K, nullptr, hw, ND_EPI_STORE_F32, nullptr, scores));
      if (hw > INT_MAX) return fail(ND_ERR_INVALID, "wan vae: too many pixels for the attention");
      prof_begin(s);
      vae_softmax_kernel<<<static_cast<unsigned>(hw), 256, 0, s>>>(scores, P, dt == ND_F16, static_cast<int>(hw), scale);
      ND_CUDA(cudaGetLastError());
      dim3 grid(static_cast<unsigned>((C + 31) / 32), static_cast<unsigned>((hw + 31) / 32));
      transpose16_kernel<<<grid, dim3(32, 8), 0, s>>>(static_cast<const uint16_t*>(Vb), static_cast<uint16_t*>(VT),
                                                     static_cast<int>(hw), C);
      ND_CUDA(cudaGetLastError());
      prof_end(s, "attention", 0.0, 0.0);
      ND_OP("attention", 2.0 * hw * hw * C, lin(s, P, hw, hw, VT, nullptr, C, ND_EPI_STORE, ATT));
      const uint8_t* xres = static_cast<const uint8_t*>(x) + b * hw * C * e;
      uint8_t* yb = static_cast<uint8_t*>(y) + b * hw * C * e;
      ND_OP("gemm.out", 2.0 * hw * C * C, lin(s, ATT, hw, C, ap, ap_b, C, ND_EPI_ADD_STORE, yb, nullptr, xres));
    }
    return ND_OK;
  }

  int forward(cudaStream_t s) override {
    const int64_t lat_px = static_cast<int64_t>(B) * h0 * w0;
    prof_begin(s);
    wan_latent_in_kernel<<<grid_of(lat_px * Clp), 256, 0, s>>>(in_latent, cv2_w, cv2_b, xin, dt == ND_F16, B, h0 * w0,
                                                                Cl, Clp);
    ND_CUDA(cudaGetLastError());
    prof_end(s, "layout", 0.0, 0.0);
    ND_OP("conv3x3", conv_flops(h0, w0, Clp, top), conv(s, xin, h0, w0, Clp, c1_w, c1_b, top, ND_EPI_STORE, X[0], nullptr));
    ND_TRY_RC(res(s, mid0, h0, w0, X[0], X[1]));
    ND_TRY_RC(attn(s, X[1], X[0]));
    ND_TRY_RC(res(s, mid1, h0, w0, X[0], X[1]));
    int cur = 1;  // index into X of the running activation
    for (int i = 0; i < L; ++i) {
      const WanLevel& v = lv[i];
      const int hh = res_h(i), ww = res_w(i);
      const int in = cur;  // the level's input stays put for the Wan 2.2 shortcut
      const int o1 = (in + 1) % 3, o2 = (in + 2) % 3;
      for (int j = 0; j < R + 1; ++j) {
        const int dst = (j % 2 == 0) ? o1 : o2;
        ND_TRY_RC(res(s, v.res[j], hh, ww, X[cur], X[dst]));
        cur = dst;
      }
      if (v.up_out) {
        const int dst = cur == o1 ? o2 : o1;
        ND_OP("upsample", 0.0, upsample2x(X[cur], UPB, B, hh, ww, v.cout, s));
        ND_OP("conv3x3", conv_flops(2 * hh, 2 * ww, v.cout, v.up_out),
              conv(s, UPB, 2 * hh, 2 * ww, v.cout, v.upw, v.upb, v.up_out, ND_EPI_STORE, X[dst], nullptr));
        cur = dst;
        if (v.sc_mode >= 0) {
          const int64_t n = static_cast<int64_t>(B) * 4 * hh * ww * v.up_out;
          prof_begin(s);
          if (v.up_out % 8 == 0)
            wan_up_shortcut8_kernel<<<grid_of(n / 8), 256, 0, s>>>(static_cast<uint4*>(X[cur]),
                                                                   static_cast<const uint4*>(X[in]), dt == ND_F16, B,
                                                                   hh, ww, v.cin, v.up_out, v.sc_mode);
          else
            wan_up_shortcut_kernel<<<grid_of(n), 256, 0, s>>>(X[cur], X[in], dt == ND_F16, B, hh, ww, v.cin, v.up_out,
                                                              v.sc_mode);
          ND_CUDA(cudaGetLastError());
          prof_end(s, "upsample", 0.0, 0.0);
        }
      }
    }
    const int hh = res_h(L - 1), ww = res_w(L - 1), c = lv[L - 1].cout;
    const int64_t img_px = static_cast<int64_t>(B) * hh * ww;
    ND_OP("rmsnorm", 0.0, rms(s, X[cur], H1, img_px, c, head_g, true));
    ND_OP("conv3x3", conv_flops(hh, ww, c, img_c),
          conv(s, H1, hh, ww, c, head_w, head_b, 4, ND_EPI_STORE_F32, nullptr, nullptr, out_nhwc));
    prof_begin(s);
    vae_image_out_kernel<<<grid_of(img_px * 3), 256, 0, s>>>(out_nhwc, out_image, B, hh * ww);
    ND_CUDA(cudaGetLastError());
    prof_end(s, "layout", 0.0, 0.0);
    return ND_OK;
  }
#undef ND_OP
};

}  // namespace

nd_denoiser* make_vae_decoder() { return new VaeDecoder(); }
nd_denoiser* make_wan_decoder() { return new WanDecoder(); }

}  // namespace nd
