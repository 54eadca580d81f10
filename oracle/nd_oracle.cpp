// nd_oracle — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
//
// A CPU restatement (C++17, OpenMP) of NaiveDiffusion's layer arithmetic for
// the denoiser forward step. Only the tests, __graft_entry__.smoke() and the
// cpu_baseline / reference leg of bench.py may load it, and only as the
// checker or the timed CPU baseline; libnd_denoise never links or calls it.
//
// Each function names the reference code it follows (paths relative to the
// NaiveDiffusion project root). The reference is C# on .NET; there is no
// dotnet toolchain here, so it cannot be compiled or run: this restatement
// is pinned against the known-answer checks its own tests and smoke command
// hold (tests/test_oracle.py restates them), not against its binary.
//
// Conventions: row-major float32 arrays; nn.Linear weights are [out, in].

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#if defined(_OPENMP)
#include <omp.h>
#endif

#define EXPORT extern "C" __attribute__((visibility("default")))

namespace {

// CpuMath.Dot (Tensors/CpuMath.cs:311-335): four vector accumulators of
// Vector<float>.Count lanes (8 with AVX2), summed, then a scalar tail.
inline float dot(const float* a, const float* b, int n) {
  constexpr int W = 8;
  float s[4][W] = {};
  int i = 0;
  for (; i + 4 * W <= n; i += 4 * W) {
    for (int u = 0; u < 4; ++u)
      for (int l = 0; l < W; ++l) s[u][l] += a[i + u * W + l] * b[i + u * W + l];
  }
  float v[W];
  for (int l = 0; l < W; ++l) v[l] = s[0][l] + s[1][l] + s[2][l] + s[3][l];
  float total = 0.f;
  for (int l = 0; l < W; ++l) total += v[l];
  for (; i < n; ++i) total += a[i] * b[i];
  return total;
}

// IEEE binary16 conversions, round to nearest even (System.Half semantics).
inline uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) {  // inf / nan
    return static_cast<uint16_t>(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // overflow -> inf
  if (absx < 0x38800000u) {  // subnormal half (or zero)
    if (absx < 0x33000000u) return static_cast<uint16_t>(sign);  // < 2^-25 rounds to 0
    const uint32_t e = absx >> 23;
    const uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e;  // 14 + (113 - e)
    uint32_t half = m >> (shift);
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t mid = 1u << (shift - 1u);
    if (rem > mid || (rem == mid && (half & 1u))) ++half;
    return static_cast<uint16_t>(sign | half);
  }
  uint32_t r = absx - 0x38000000u;  // rebias exponent 127 -> 15
  const uint32_t rem = r & 0x1FFFu;
  uint32_t half = r >> 13;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) ++half;
  return static_cast<uint16_t>(sign | half);
}

inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
      e = 113;
      while (!(m & 0x400u)) {
        m <<= 1;
        --e;
      }
      x = sign | (e << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    x = sign | 0x7F800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

inline uint16_t f32_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((x >> 16) | 0x40u);
  x += 0x7FFFu + ((x >> 16) & 1u);
  return static_cast<uint16_t>(x >> 16);
}

inline float bf16_to_f32(uint16_t b) {
  uint32_t x = static_cast<uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// CpuMath.Erf (Tensors/CpuMath.cs:297-307), Abramowitz & Stegun 7.1.26.
inline float erf_as(float x) {
  const float sign = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
  x = std::fabs(x);
  const float t = 1.0f / (1.0f + 0.3275911f * x);
  const float series =
      ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
       0.254829592f) *
      t;
  return sign * (1.0f - series * std::exp(-x * x));
}

}  // namespace

// ------------------------------------------------------------------ dtypes

EXPORT void nd_oracle_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f32_to_f16(x[i]);
}
EXPORT void nd_oracle_f16_to_f32(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f16_to_f32(x[i]);
}
EXPORT void nd_oracle_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f32_to_bf16(x[i]);
}
EXPORT void nd_oracle_bf16_to_f32(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = bf16_to_f32(x[i]);
}

EXPORT int nd_oracle_threads(void) {
#if defined(_OPENMP)
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// ------------------------------------------------------------------ layers

// CpuMath.Linear (Tensors/CpuMath.cs:34-64): y[m, o] = dot(x[m], w[o]) + b[o].
// The reference runs one task per output column (Parallel.For over `outer`);
// here the (row, column) pairs are visited in cache tiles of 64 rows x 16
// columns. Every element is still one dot() over the whole inner length plus
// the bias, so the result is the same bit for bit; only the visiting order
// (which the arithmetic does not depend on) changes.
EXPORT void nd_oracle_linear(const float* x, int rows, int inner, const float* w,
                             const float* bias, float* y, int outer) {
  constexpr int kRows = 64, kCols = 16;
  const int rblocks = (rows + kRows - 1) / kRows, cblocks = (outer + kCols - 1) / kCols;
#pragma omp parallel for collapse(2) schedule(static)
  for (int cb = 0; cb < cblocks; ++cb)
    for (int rb = 0; rb < rblocks; ++rb) {
      const int m1 = std::min(rows, (rb + 1) * kRows), o1 = std::min(outer, (cb + 1) * kCols);
      for (int m = rb * kRows; m < m1; ++m) {
        const float* xm = x + static_cast<int64_t>(m) * inner;
        for (int o = cb * kCols; o < o1; ++o)
          y[static_cast<int64_t>(m) * outer + o] =
              dot(xm, w + static_cast<int64_t>(o) * inner, inner) + (bias ? bias[o] : 0.f);
      }
    }
}

// CpuMath.LayerNorm (Tensors/CpuMath.cs:92-122): two passes in double.
// weight/bias may be NULL: the affine-free LayerNorm a DiT modulates
// (Graph/Layers.cs:225-226).
EXPORT void nd_oracle_layernorm(const float* x, int rows, int width, const float* weight,
                                const float* bias, float* y, float eps) {
#pragma omp parallel for schedule(static)
  for (int m = 0; m < rows; ++m) {
    const float* s = x + static_cast<int64_t>(m) * width;
    float* t = y + static_cast<int64_t>(m) * width;
    double sum = 0;
    for (int i = 0; i < width; ++i) sum += s[i];
    const double mean = sum / width;
    double square = 0;
    for (int i = 0; i < width; ++i) {
      const double c = s[i] - mean;
      square += c * c;
    }
    const double scale = 1.0 / std::sqrt(square / width + eps);
    for (int i = 0; i < width; ++i) {
      const float n = static_cast<float>((s[i] - mean) * scale);
      t[i] = n * (weight ? weight[i] : 1.f) + (bias ? bias[i] : 0.f);
    }
  }
}

// Transformer.Modulate (Graph/Transformer.cs:72-80): LayerNorm without an
// affine, times (1 + scale), plus shift (NULL: none). scale/shift are one
// [width] vector for every row.
EXPORT void nd_oracle_modulate(const float* x, int rows, int width, const float* shift,
                               const float* scale, float* y, float eps) {
  nd_oracle_layernorm(x, rows, width, nullptr, nullptr, y, eps);
#pragma omp parallel for schedule(static)
  for (int m = 0; m < rows; ++m) {
    float* t = y + static_cast<int64_t>(m) * width;
    for (int i = 0; i < width; ++i) t[i] = t[i] * (scale[i] + 1.0f) + (shift ? shift[i] : 0.f);
  }
}

// CpuMath.RmsNorm (Tensors/CpuMath.cs:128-146): sum of squares in double.
// Rows may be heads ([tokens * heads] rows of head_dim).
EXPORT void nd_oracle_rmsnorm(const float* x, int rows, int width, const float* weight, float* y,
                              float eps) {
#pragma omp parallel for schedule(static)
  for (int m = 0; m < rows; ++m) {
    const float* s = x + static_cast<int64_t>(m) * width;
    float* t = y + static_cast<int64_t>(m) * width;
    double square = 0;
    for (int i = 0; i < width; ++i) square += static_cast<double>(s[i]) * s[i];
    const float scale = static_cast<float>(1.0 / std::sqrt(square / width + eps));
    for (int i = 0; i < width; ++i) t[i] = s[i] * scale * (weight ? weight[i] : 1.f);
  }
}

// CpuMath.Rope (Tensors/CpuMath.cs:154-173) / Transformer.Rotate
// (Graph/Transformer.cs:50-64): rotate-half, in place over [rows, heads, dim]
// with [rows, dim/2] tables.
EXPORT void nd_oracle_rope(float* x, int rows, int heads, int dim, const float* cos,
                           const float* sin) {
  const int half = dim / 2;
#pragma omp parallel for schedule(static)
  for (int m = 0; m < rows; ++m) {
    const float* c = cos + static_cast<int64_t>(m) * half;
    const float* s = sin + static_cast<int64_t>(m) * half;
    for (int h = 0; h < heads; ++h) {
      float* v = x + (static_cast<int64_t>(m) * heads + h) * dim;
      for (int i = 0; i < half; ++i) {
        const float lo = v[i], hi = v[i + half];
        v[i] = lo * c[i] - hi * s[i];
        v[i + half] = hi * c[i] + lo * s[i];
      }
    }
  }
}

// CpuMath.Attention (Tensors/CpuMath.cs:203-248), plus the key-count mask of
// DmlOps.MultiheadAttention's KeySequenceLength form (Dml/DmlOps.cs:460-479):
// keys at or beyond key_len are left out, as SmokeTest.MaskedAttention's CPU
// check does (NaiveDiffusion.Cli/SmokeTest.cs:393-485). key_len <= 0 or
// > key_rows means every key. q: [rows, qheads*dim]; k, v: [key_rows,
// kheads*dim]; y like q. Strides ldq/ldk/ldv/ldy in elements (0 = packed).
EXPORT void nd_oracle_attention(const float* q, const float* k, const float* v, int rows,
                                int key_rows, int qheads, int kheads, int dim, int causal,
                                int key_len, float* y, int64_t ldq, int64_t ldk, int64_t ldv,
                                int64_t ldy) {
  const int64_t qw = ldq ? ldq : static_cast<int64_t>(qheads) * dim;
  const int64_t kw = ldk ? ldk : static_cast<int64_t>(kheads) * dim;
  const int64_t vw = ldv ? ldv : static_cast<int64_t>(kheads) * dim;
  const int64_t yw = ldy ? ldy : static_cast<int64_t>(qheads) * dim;
  const int group = qheads / kheads;
  const float scale = 1.0f / std::sqrt(static_cast<float>(dim));
  const int keys = (key_len > 0 && key_len < key_rows) ? key_len : key_rows;
#pragma omp parallel
  {
    std::vector<float> scores(key_rows);
#pragma omp for schedule(static)
    for (int work = 0; work < qheads * rows; ++work) {
      const int head = work / rows;
      const int i = work % rows;
      const int64_t qo = static_cast<int64_t>(head) * dim;
      const int64_t ko = static_cast<int64_t>(head / group) * dim;
      const int visible = causal ? std::min(i + 1, keys) : keys;
      const float* qi = q + i * qw + qo;
      float largest = -INFINITY;
      for (int j = 0; j < visible; ++j) {
        const float sc = dot(qi, k + j * kw + ko, dim) * scale;
        scores[j] = sc;
        largest = std::fmax(largest, sc);
      }
      float total = 0.f;
      for (int j = 0; j < visible; ++j) {
        scores[j] = std::exp(scores[j] - largest);
        total += scores[j];
      }
      const float normalize = 1.0f / total;
      float* t = y + i * yw + qo;
      for (int d = 0; d < dim; ++d) t[d] = 0.f;
      for (int j = 0; j < visible; ++j) {
        const float wgt = scores[j] * normalize;
        const float* vj = v + j * vw + ko;
        for (int d = 0; d < dim; ++d) t[d] += wgt * vj[d];
      }
    }
  }
}

// CpuMath.Gelu (Tensors/CpuMath.cs:289-295): exact GELU through A&S erf.
EXPORT void nd_oracle_gelu(float* x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) x[i] = 0.5f * x[i] * (1.0f + erf_as(x[i] * 0.70710678f));
}

// QwenImageDit.GeluTanh (Models/QwenImage/QwenImageDit.cs:510-515):
// x * sigmoid(2 * sqrt(2/pi) * (x + 0.044715 x^3)).
EXPORT void nd_oracle_gelu_tanh(float* x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    const float cubic = v * v * v * 0.044715f + v;
    x[i] = v * (1.0f / (1.0f + std::exp(-(cubic * (2.0f * 0.7978845608f)))));
  }
}

// CpuMath.Silu (Tensors/CpuMath.cs:260-266).
EXPORT void nd_oracle_silu(float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] *= 1.0f / (1.0f + std::exp(-x[i]));
}

// Transformer.Sinusoid (Graph/Transformer.cs:20-32): half cosines then half
// sines of time * 10000^(-i/half), in float.
EXPORT void nd_oracle_sinusoid(float time, int width, float* out) {
  const int half = width / 2;
  for (int i = 0; i < half; ++i) {
    const float frequency = std::exp(-std::log(10000.0f) * i / half);
    const float angle = time * frequency;
    out[i] = std::cos(angle);
    out[half + i] = std::sin(angle);
  }
}

// QwenImageDit.RopeTables (Models/QwenImage/QwenImageDit.cs:189-240): one
// row per token -- image cells in row-major order, then context_rows text
// rows -- and 64 pair columns over the three axes 16/56/56. A text token p
// sits at (p, p, p); image cell (i, j) at (text_len, i - ceil(h/2), j - ceil(w/2)).
EXPORT void nd_oracle_qwen_rope_tables(int rows, int columns, int text_len, int context_rows,
                                       float* cos, float* sin) {
  const int axes[3] = {16, 56, 56};
  const int pairs = 64;
  double freq[64];
  int p = 0;
  for (int a = 0; a < 3; ++a)
    for (int k = 0; k < axes[a] / 2; ++k) freq[p++] = 1.0 / std::pow(10000.0, 2.0 * k / axes[a]);
  auto fill = [&](int token, double first, double second, double third) {
    const int64_t off = static_cast<int64_t>(token) * pairs;
    const double pos[3] = {first, second, third};
    int pr = 0;
    for (int a = 0; a < 3; ++a)
      for (int k = 0; k < axes[a] / 2; ++k, ++pr) {
        const double angle = pos[a] * freq[pr];
        cos[off + pr] = static_cast<float>(std::cos(angle));
        sin[off + pr] = static_cast<float>(std::sin(angle));
      }
  };
  const int row_start = rows - rows / 2, col_start = columns - columns / 2;
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < columns; ++j) fill(i * columns + j, text_len, i - row_start, j - col_start);
  for (int t = 0; t < context_rows; ++t) fill(rows * columns + t, t, t, t);
}

// AnimaDit.RopeTables (Models/Anima/AnimaDit.cs:149-188): 22 still temporal
// pairs, then 21 row and 21 column pairs at the NTK-scaled base.
EXPORT void nd_oracle_anima_rope_tables(int rows, int columns, int head_dim, float* cos,
                                        float* sin) {
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

// ------------------------------------------------------------------ int8

// BlockQuantizer.Quantize (Tensors/BlockQuantizer.cs:34-105), generalised to
// a group of `group` columns (32 in the reference; group == columns gives
// one scale per output channel). Scale = |max| / 127, stored as fp16 (RNE)
// when scale_f16 != 0 or fp32 otherwise; values quantized against the scale
// as stored: q = clamp(rint(w * (1 / stored)), -127, 127); a zero stored
// scale leaves the group zero. scales: [rows, columns / group].
EXPORT int nd_oracle_quantize(const float* w, int rows, int columns, int group, int scale_f16,
                              int8_t* q, void* scales) {
  if (rows <= 0 || group <= 0 || columns % group != 0) return 1;
  const int blocks = columns / group;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    for (int b = 0; b < blocks; ++b) {
      const float* src = w + static_cast<int64_t>(r) * columns + static_cast<int64_t>(b) * group;
      int8_t* dst = q + static_cast<int64_t>(r) * columns + static_cast<int64_t>(b) * group;
      float peak = 0.f;
      for (int i = 0; i < group; ++i) peak = std::fmax(peak, std::fabs(src[i]));
      float stored;
      const int64_t si = static_cast<int64_t>(r) * blocks + b;
      if (scale_f16) {
        const uint16_t h = f32_to_f16(peak / 127.f);
        static_cast<uint16_t*>(scales)[si] = h;
        stored = f16_to_f32(h);
      } else {
        stored = peak / 127.f;
        static_cast<float*>(scales)[si] = stored;
      }
      if (stored == 0.f) {
        std::memset(dst, 0, group);
        continue;
      }
      const float inverse = 1.0f / stored;
      for (int i = 0; i < group; ++i) {
        float v = std::nearbyint(src[i] * inverse);
        v = std::fmax(-127.f, std::fmin(127.f, v));
        dst[i] = static_cast<int8_t>(v);
      }
    }
  }
  return 0;
}

// DmlOps.Dequantize (Dml/DmlOps.cs:208-228): w = q * scale, in fp32.
EXPORT void nd_oracle_dequantize(const int8_t* q, const void* scales, int scale_f16, int rows,
                                 int columns, int group, float* w) {
  const int blocks = columns / group;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < columns; ++c) {
      const int64_t si = static_cast<int64_t>(r) * blocks + c / group;
      const float s = scale_f16 ? f16_to_f32(static_cast<const uint16_t*>(scales)[si])
                                : static_cast<const float*>(scales)[si];
      w[static_cast<int64_t>(r) * columns + c] = static_cast<float>(q[static_cast<int64_t>(r) * columns + c]) * s;
    }
}

// ------------------------------------------------------------------ blocks

// One stream's weights of a Qwen-Image-style dual-stream (MMDiT) block.
// Layout follows nn.Linear ([out, in]); q/k/v of one stream are separate.
struct nd_oracle_mmdit_stream {
  const float *mod_w, *mod_b;              // [6D, D], [6D]: shift1 scale1 gate1 shift2 scale2 gate2
  const float *q_w, *q_b, *k_w, *k_b, *v_w, *v_b;  // [D, D], [D]
  const float *norm_q, *norm_k;            // [head_dim]
  const float *out_w, *out_b;              // [D, D], [D]
  const float *up_w, *up_b;                // [F, D], [F]
  const float *down_w, *down_b;            // [D, F], [D]
};

// The benchmark configuration-3 block. The reference has no dual-stream
// Qwen-Image model (QwenImageCheckpoint refuses it); this block is composed
// from the reference's own primitives in the order its single-stream
// QwenImageDit.Block uses them (Models/QwenImage/QwenImageDit.cs:309-425):
//   per stream: mod = Linear(silu(temb));  n = Modulate(x, shift1, scale1)
//               q, k, v = Linear(n); q, k = HeadNorm (RMSNorm * w)
//   joint: RoPE(q, k) over [image rows; text rows]; attention over all rows
//          with the key-count mask
//   per stream: x += gate1 * Linear(attn)
//               x += gate2 * Linear(gelu_tanh(Linear(Modulate(x, shift2, scale2))))
// x: [n_img + n_txt, D] fp32, image rows first, updated in place.
EXPORT void nd_oracle_mmdit_block(const nd_oracle_mmdit_stream* img,
                                  const nd_oracle_mmdit_stream* txt, int width, int heads,
                                  int head_dim, int mlp, float* x, int n_img, int n_txt,
                                  const float* temb, const float* cos, const float* sin,
                                  int key_len, float eps) {
  const int D = width, M = n_img + n_txt;
  const nd_oracle_mmdit_stream* st[2] = {img, txt};
  const int start[2] = {0, n_img}, count[2] = {n_img, n_txt};
  std::vector<float> t(temb, temb + D);
  nd_oracle_silu(t.data(), D);
  std::vector<float> mod[2];
  std::vector<float> q(static_cast<size_t>(M) * D), k(q.size()), v(q.size()), a(q.size());
  std::vector<float> n(q.size());
  for (int s = 0; s < 2; ++s) {
    mod[s].resize(6 * D);
    nd_oracle_linear(t.data(), 1, D, st[s]->mod_w, st[s]->mod_b, mod[s].data(), 6 * D);
    if (!count[s]) continue;
    float* xs = x + static_cast<int64_t>(start[s]) * D;
    float* ns = n.data() + static_cast<int64_t>(start[s]) * D;
    nd_oracle_modulate(xs, count[s], D, mod[s].data(), mod[s].data() + D, ns, eps);
    float* qs = q.data() + static_cast<int64_t>(start[s]) * D;
    float* ks = k.data() + static_cast<int64_t>(start[s]) * D;
    float* vs = v.data() + static_cast<int64_t>(start[s]) * D;
    nd_oracle_linear(ns, count[s], D, st[s]->q_w, st[s]->q_b, qs, D);
    nd_oracle_linear(ns, count[s], D, st[s]->k_w, st[s]->k_b, ks, D);
    nd_oracle_linear(ns, count[s], D, st[s]->v_w, st[s]->v_b, vs, D);
    nd_oracle_rmsnorm(qs, count[s] * heads, head_dim, st[s]->norm_q, qs, eps);
    nd_oracle_rmsnorm(ks, count[s] * heads, head_dim, st[s]->norm_k, ks, eps);
  }
  nd_oracle_rope(q.data(), M, heads, head_dim, cos, sin);
  nd_oracle_rope(k.data(), M, heads, head_dim, cos, sin);
  nd_oracle_attention(q.data(), k.data(), v.data(), M, M, heads, heads, head_dim, 0, key_len,
                      a.data(), 0, 0, 0, 0);
  std::vector<float> o(static_cast<size_t>(M) * D);
  std::vector<float> h(static_cast<size_t>(M) * mlp);
  for (int s = 0; s < 2; ++s) {
    if (!count[s]) continue;
    const float* gate1 = mod[s].data() + 2 * D;
    const float* gate2 = mod[s].data() + 5 * D;
    float* xs = x + static_cast<int64_t>(start[s]) * D;
    const int64_t cnt = count[s];
    nd_oracle_linear(a.data() + start[s] * static_cast<int64_t>(D), count[s], D, st[s]->out_w,
                     st[s]->out_b, o.data(), D);
    for (int64_t r = 0; r < cnt; ++r)
      for (int c = 0; c < D; ++c) xs[r * D + c] += gate1[c] * o[r * D + c];
    nd_oracle_modulate(xs, count[s], D, mod[s].data() + 3 * D, mod[s].data() + 4 * D, n.data(), eps);
    nd_oracle_linear(n.data(), count[s], D, st[s]->up_w, st[s]->up_b, h.data(), mlp);
    nd_oracle_gelu_tanh(h.data(), cnt * mlp);
    nd_oracle_linear(h.data(), count[s], mlp, st[s]->down_w, st[s]->down_b, o.data(), D);
    for (int64_t r = 0; r < cnt; ++r)
      for (int c = 0; c < D; ++c) xs[r * D + c] += gate2[c] * o[r * D + c];
  }
}

// Weights of one Anima (Cosmos-Predict2) block; no biases anywhere.
struct nd_oracle_anima_block_w {
  // low-rank adaLN per sub-block: [r, D] then [3D, r]
  const float *self_mod1, *self_mod2, *cross_mod1, *cross_mod2, *mlp_mod1, *mlp_mod2;
  const float *sq, *sk, *sv, *so, *sq_norm, *sk_norm;  // self-attn [D, D], norms [hd]
  const float *cq, *ck, *cv, *co, *cq_norm, *ck_norm;  // cross: ck, cv [D, ctx_width]
  const float *fc1, *fc2;                              // [F, D], [D, F]
};

// AnimaDit.Block (Models/Anima/AnimaDit.cs:270-358): three adaLN-modulated
// sub-blocks (self-attention with head norms and 3-D RoPE, cross-attention to
// the context with head norms, exact-GELU MLP), each residual gated in fp32.
// Modulation(prefix) = Linear(Linear(silu(temb), mod1), mod2) + lora, cut into
// shift, scale, gate (:270-291). x: [tokens, D]; context: [ctx_rows, ctx_width];
// temb: [D] (already RMS-normed); lora: [3D].
EXPORT void nd_oracle_anima_block(const nd_oracle_anima_block_w* w, int width, int heads,
                                  int head_dim, int mlp, int rank, float* x, int tokens,
                                  const float* context, int ctx_rows, int ctx_width,
                                  const float* temb, const float* lora, const float* cos,
                                  const float* sin, float eps) {
  const int D = width;
  const int64_t MD = static_cast<int64_t>(tokens) * D;
  std::vector<float> t(temb, temb + D);
  nd_oracle_silu(t.data(), D);
  auto modulation = [&](const float* m1, const float* m2, std::vector<float>& out) {
    std::vector<float> low(rank);
    nd_oracle_linear(t.data(), 1, D, m1, nullptr, low.data(), rank);
    out.resize(3 * D);
    nd_oracle_linear(low.data(), 1, rank, m2, nullptr, out.data(), 3 * D);
    for (int i = 0; i < 3 * D; ++i) out[i] += lora[i];
  };
  std::vector<float> ms, mc, mm;
  modulation(w->self_mod1, w->self_mod2, ms);
  modulation(w->cross_mod1, w->cross_mod2, mc);
  modulation(w->mlp_mod1, w->mlp_mod2, mm);

  std::vector<float> n(MD), q(MD), a(MD), o(MD);
  // self-attention
  {
    std::vector<float> k(MD), v(MD);
    nd_oracle_modulate(x, tokens, D, ms.data(), ms.data() + D, n.data(), eps);
    nd_oracle_linear(n.data(), tokens, D, w->sq, nullptr, q.data(), D);
    nd_oracle_linear(n.data(), tokens, D, w->sk, nullptr, k.data(), D);
    nd_oracle_linear(n.data(), tokens, D, w->sv, nullptr, v.data(), D);
    nd_oracle_rmsnorm(q.data(), tokens * heads, head_dim, w->sq_norm, q.data(), eps);
    nd_oracle_rmsnorm(k.data(), tokens * heads, head_dim, w->sk_norm, k.data(), eps);
    nd_oracle_rope(q.data(), tokens, heads, head_dim, cos, sin);
    nd_oracle_rope(k.data(), tokens, heads, head_dim, cos, sin);
    nd_oracle_attention(q.data(), k.data(), v.data(), tokens, tokens, heads, heads, head_dim, 0, 0,
                        a.data(), 0, 0, 0, 0);
    nd_oracle_linear(a.data(), tokens, D, w->so, nullptr, o.data(), D);
    for (int64_t i = 0; i < MD; ++i) x[i] += ms[2 * D + i % D] * o[i];
  }
  // cross-attention
  {
    const int64_t CD = static_cast<int64_t>(ctx_rows) * D;
    std::vector<float> k(CD), v(CD);
    nd_oracle_modulate(x, tokens, D, mc.data(), mc.data() + D, n.data(), eps);
    nd_oracle_linear(n.data(), tokens, D, w->cq, nullptr, q.data(), D);
    nd_oracle_linear(context, ctx_rows, ctx_width, w->ck, nullptr, k.data(), D);
    nd_oracle_linear(context, ctx_rows, ctx_width, w->cv, nullptr, v.data(), D);
    nd_oracle_rmsnorm(q.data(), tokens * heads, head_dim, w->cq_norm, q.data(), eps);
    nd_oracle_rmsnorm(k.data(), ctx_rows * heads, head_dim, w->ck_norm, k.data(), eps);
    nd_oracle_attention(q.data(), k.data(), v.data(), tokens, ctx_rows, heads, heads, head_dim, 0,
                        0, a.data(), 0, 0, 0, 0);
    nd_oracle_linear(a.data(), tokens, D, w->co, nullptr, o.data(), D);
    for (int64_t i = 0; i < MD; ++i) x[i] += mc[2 * D + i % D] * o[i];
  }
  // MLP
  {
    std::vector<float> h(static_cast<size_t>(tokens) * mlp);
    nd_oracle_modulate(x, tokens, D, mm.data(), mm.data() + D, n.data(), eps);
    nd_oracle_linear(n.data(), tokens, D, w->fc1, nullptr, h.data(), mlp);
    nd_oracle_gelu(h.data(), static_cast<int64_t>(tokens) * mlp);
    nd_oracle_linear(h.data(), tokens, mlp, w->fc2, nullptr, o.data(), D);
    for (int64_t i = 0; i < MD; ++i) x[i] += mm[2 * D + i % D] * o[i];
  }
}

// ------------------------------------------------------------------ UNet

// GroupNorm over one image [C, HW] (Layers.GroupNorm, Graph/Layers.cs:166-185;
// the smoke check's recipe, NaiveDiffusion.Cli/SmokeTest.cs:208-239): each
// group of C/G channels normalized over its C/G x HW values with double mean
// and variance, then y = n * w[c] + b[c] (NULL: 1 / 0), then SiLU if asked
// (UNetModel.ResnetBlock, Models/Sdxl/UNetModel.cs:230-254).
EXPORT void nd_oracle_group_norm(const float* x, int C, int HW, int groups, const float* w,
                                 const float* b, float eps, int silu, float* y) {
  const int cg = C / groups;
#pragma omp parallel for schedule(static)
  for (int g = 0; g < groups; ++g) {
    const int64_t n = static_cast<int64_t>(cg) * HW;
    const float* s = x + static_cast<int64_t>(g) * n;
    double mean = 0;
    for (int64_t i = 0; i < n; ++i) mean += s[i];
    mean /= n;
    double var = 0;
    for (int64_t i = 0; i < n; ++i) var += (s[i] - mean) * (s[i] - mean);
    var /= n;
    const double inv = 1.0 / std::sqrt(var + eps);
    for (int c = 0; c < cg; ++c) {
      const int ch = g * cg + c;
      for (int p = 0; p < HW; ++p) {
        const int64_t i = static_cast<int64_t>(c) * HW + p;
        float v = static_cast<float>((s[i] - mean) * inv) * (w ? w[ch] : 1.f) + (b ? b[ch] : 0.f);
        if (silu) v *= 1.0f / (1.0f + std::exp(-v));
        y[static_cast<int64_t>(g) * n + i] = v;
      }
    }
  }
}

// 2-D convolution, NCHW one image (Layers.Conv2d, Graph/Layers.cs:115-128, as
// the smoke check computes it, SmokeTest.cs:241-281): y[o, r, c] = b[o] +
// sum over (i, dy, dx) of w[o, i, dy, dx] * x[i, r*s + dy - pad, c*s + dx - pad],
// zero outside the image; float sums.
EXPORT void nd_oracle_conv2d(const float* x, int Cin, int H, int W, const float* w, const float* b,
                             int Cout, int k, int stride, int pad, float* y) {
  const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  // Output rows in bands of ~2048 values so a band's sums stay in L1 while
  // every (i, dy, dx) term is added in; each element still receives its terms
  // in the order (i, dy, dx), so the band split does not change any sum.
  const int band = std::max(1, 2048 / std::max(1, Wo));
  const int bands = (Ho + band - 1) / band;
#pragma omp parallel for collapse(2) schedule(static)
  for (int o = 0; o < Cout; ++o)
    for (int rb = 0; rb < bands; ++rb) {
      float* yo = y + static_cast<int64_t>(o) * Ho * Wo;
      const int r0 = rb * band, r1 = std::min(Ho, r0 + band);
      for (int p = r0 * Wo; p < r1 * Wo; ++p) yo[p] = b ? b[o] : 0.f;
      for (int i = 0; i < Cin; ++i)
        for (int dy = 0; dy < k; ++dy)
          for (int dx = 0; dx < k; ++dx) {
            const float wv = w[((static_cast<int64_t>(o) * Cin + i) * k + dy) * k + dx];
            const float* xi = x + static_cast<int64_t>(i) * H * W;
            // columns c with 0 <= c*stride + dx - pad < W
            const int c0 = std::max(0, (pad - dx + stride - 1) / stride);
            const int last = W - 1 + pad - dx;  // c*stride <= last
            const int c1 = last < 0 ? 0 : std::min(Wo, last / stride + 1);
            for (int r = r0; r < r1; ++r) {
              const int yy = r * stride + dy - pad;
              if (yy < 0 || yy >= H) continue;
              float* yr = yo + static_cast<int64_t>(r) * Wo;
              const float* xr = xi + static_cast<int64_t>(yy) * W + dx - pad;
              if (stride == 1) {
                for (int c = c0; c < c1; ++c) yr[c] += wv * xr[c];
              } else {
                for (int c = c0; c < c1; ++c) yr[c] += wv * xr[c * stride];
              }
            }
          }
    }
}

// ---------------------------------------------------------------- sampling
// The guidance combine and one solver step, element by element with the
// reference's types: float arithmetic where its arrays are float[], double
// where it widens (Pipeline/GuidanceStrategy.cs:32-41; Sampling/Schedulers.cs
// EulerScheduler.Step :270-280, EulerAncestralScheduler.Step :298-333,
// DpmPlusPlus2MScheduler.Step :348-385, DpmPlusPlus2MSdeScheduler.Step
// :404-445; Sampling/Prediction.cs Denoise / Derivative). The scalars the
// reference derives from the sigmas in double come in as arguments.
// sampler: 0 Euler, 1 Euler a, 2 DPM++ 2M, 3 DPM++ 2M SDE;
// prediction: 0 epsilon, 1 velocity, 2 flow.
namespace {

float oracle_denoise(int prediction, float out, float sample, double sigma) {
  if (prediction == 1) {  // VelocityPrediction.Denoise
    const double variance = sigma * sigma + 1.0;
    const double skip = 1.0 / variance;
    const double output = sigma / std::sqrt(variance);
    return static_cast<float>(sample * skip - out * output);
  }
  return static_cast<float>(sample - sigma * out);  // Epsilon / Flow
}

float oracle_derivative(int prediction, float out, float sample, double sigma) {
  if (prediction == 1) {  // (sample - denoised) / sigma
    const float denoised = oracle_denoise(prediction, out, sample, sigma);
    return static_cast<float>((sample - denoised) / sigma);
  }
  return out;
}

}  // namespace

EXPORT void nd_oracle_sampler_step(int sampler, int prediction, int64_t n, int branches, const float* out,
                                   float guidance, float* sample, float* last_denoised, const float* noise,
                                   float* denoised_out, float sigma_f, float sigma_next_f, double up, double down,
                                   double rescale, double noise_scale, double shrink, double weight,
                                   int second_order) {
  for (int64_t i = 0; i < n; ++i) {
    float pred = out[i];
    if (branches == 2) {
      const float uncond = out[i], cond = out[n + i];
      pred = uncond + guidance * (cond - uncond);
    }
    const double sigma = sigma_f;
    if (denoised_out) denoised_out[i] = oracle_denoise(prediction, pred, sample[i], sigma);
    if (sampler == 0) {
      const float derivative = oracle_derivative(prediction, pred, sample[i], sigma);
      const float delta = sigma_next_f - sigma_f;
      sample[i] += derivative * delta;
    } else if (sampler == 1) {
      const float derivative = oracle_derivative(prediction, pred, sample[i], sigma);
      const float delta = static_cast<float>(down - sigma);
      if (rescale == 1.0) {
        const float up_scale = static_cast<float>(up);
        sample[i] += derivative * delta + noise[i] * up_scale;
      } else {
        sample[i] = static_cast<float>(rescale * (sample[i] + derivative * delta) + noise[i] * noise_scale);
      }
    } else {
      const float denoised = oracle_denoise(prediction, pred, sample[i], sigma);
      if (sigma_next_f <= 0.0f) {
        sample[i] = denoised;
        continue;
      }
      if (sampler == 2) {
        const double p = second_order ? (1.0 + weight) * denoised - weight * last_denoised[i]
                                      : static_cast<double>(denoised);
        sample[i] = static_cast<float>(shrink * sample[i] + (1.0 - shrink) * p);
      } else {
        const double keep = shrink * shrink;
        const double take = 1.0 - keep;
        const float noise_scale_f = static_cast<float>(noise_scale);
        double next = keep * sample[i] + take * denoised;
        if (second_order) next += weight * (denoised - last_denoised[i]);
        sample[i] = static_cast<float>(rescale * next + noise[i] * noise_scale_f);
      }
      last_denoised[i] = denoised;
    }
  }
}
