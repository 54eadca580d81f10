// fp32 flash attention on the CUDA cores: the attention of the fp32 compute
// mode (model_desc.compute == ND_F32), where the reference runs
// DmlOps.MultiheadAttention (Dml/DmlOps.cs:480-524) in fp32 and its CPU check
// is CpuMath.Attention (Tensors/CpuMath.cs: max-subtracted softmax in float).
// Scores, exponentials, sums and the P.V products are all fp32 (no 16-bit
// rounding anywhere), with the online (flash) softmax so the [Nq, Nk] score
// matrix never leaves the SM.
//
// One CTA = 64 query rows of one head of one batch item, 128 threads as a
// 16 x 8 grid: thread (ty, tx) owns query rows 4ty..4ty+3 and, of each 64-key
// tile, keys 4tx + 32j + {0..3}; of the output, columns 4tx + 32j + {0..3}.
// Shared memory: Q^T [d][64] for the CTA's life; per key tile K^T [d][64]
// (reused for P^T [64][68] once the scores are in registers) and V [64][d].
#include <cfloat>
#include <climits>
#include <cmath>

#include "nd_common.cuh"
#include "nd_internal.h"

namespace nd {

namespace {

struct AttnF32Args {
  const float* q;
  const float* k;
  const float* v;
  long long ldq, ldk, ldv;
  void* out;
  long long ldo;
  int out_split;     // 0: fp32 out; 1: bf16 hi|lo pair, lo lo_off elements along
  long long lo_off;
  int q_rows, kv_rows, key_limit, causal;
  int kv_group;      // query heads per key / value head
  float scale;
};

constexpr int kBQ = 64;
constexpr int kBK = 64;
constexpr int kPLd = 68;  // P^T row stride: four-way (minimum) bank spread for the float4 stores

template <int HD>
struct AttnF32Smem {
  static constexpr int kQ = HD * kBQ;
  static constexpr int kKP = HD * kBK > kBK * kPLd ? HD * kBK : kBK * kPLd;
  static constexpr int kV = kBK * HD;
  static constexpr int kBytes = (kQ + kKP + kV) * 4;
};

template <int HD>
__global__ void __launch_bounds__(128) attention_f32_kernel(const AttnF32Args g) {
  constexpr int NJ = HD / 32;  // output column groups per thread
  extern __shared__ float sm[];
  float* qt = sm;                                 // [HD][64]
  float* kt = sm + AttnF32Smem<HD>::kQ;           // [HD][64], then P^T [64][kPLd]
  float* vs = kt + AttnF32Smem<HD>::kKP;          // [64][HD]
  const int tid = threadIdx.x;
  const int ty = tid >> 3, tx = tid & 7;
  const int q0 = blockIdx.x * kBQ;
  const int head = blockIdx.y;
  const int b = blockIdx.z;
  const long long qbase = static_cast<long long>(b) * g.q_rows;
  const long long kbase = static_cast<long long>(b) * g.kv_rows;
  const int col0 = head * HD;
  const int kv_col0 = (head / g.kv_group) * HD;

  // Q^T, pre-multiplied by nothing: the scale is applied to the scores.
  for (int idx = tid; idx < kBQ * HD / 4; idx += 128) {
    const int r = idx % kBQ, d4 = idx / kBQ;
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < g.q_rows)
      t = __ldg(reinterpret_cast<const float4*>(g.q + (qbase + q0 + r) * g.ldq + col0) + d4);
    qt[(4 * d4 + 0) * kBQ + r] = t.x;
    qt[(4 * d4 + 1) * kBQ + r] = t.y;
    qt[(4 * d4 + 2) * kBQ + r] = t.z;
    qt[(4 * d4 + 3) * kBQ + r] = t.w;
  }

  float o[4][NJ][4];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int u = 0; u < 4; ++u) o[i][j][u] = 0.f;
  }

  int kv_end = g.key_limit;
  if (g.causal) kv_end = min(kv_end, q0 + kBQ);
  for (int k0 = 0; k0 < kv_end; k0 += kBK) {
    __syncthreads();  // the previous tile's P^T / V reads are done
    for (int idx = tid; idx < kBK * HD / 4; idx += 128) {
      const int c = idx % kBK, d4 = idx / kBK;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + c < g.kv_rows)
        t = __ldg(reinterpret_cast<const float4*>(g.k + (kbase + k0 + c) * g.ldk + kv_col0) + d4);
      kt[(4 * d4 + 0) * kBK + c] = t.x;
      kt[(4 * d4 + 1) * kBK + c] = t.y;
      kt[(4 * d4 + 2) * kBK + c] = t.z;
      kt[(4 * d4 + 3) * kBK + c] = t.w;
    }
    for (int idx = tid; idx < kBK * HD / 4; idx += 128) {
      const int j = idx / (HD / 4), d4 = idx % (HD / 4);
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + j < g.kv_rows)
        t = __ldg(reinterpret_cast<const float4*>(g.v + (kbase + k0 + j) * g.ldv + kv_col0) + d4);
      reinterpret_cast<float4*>(vs)[idx] = t;
    }
    __syncthreads();

    // S = Q K^T for this thread's 4 rows x 8 keys
    float s[4][2][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int u = 0; u < 4; ++u) s[i][j][u] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; ++d) {
      const float4 a = *reinterpret_cast<const float4*>(qt + d * kBQ + 4 * ty);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float4 kk = *reinterpret_cast<const float4*>(kt + d * kBK + 4 * tx + 32 * j);
        const float kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int u = 0; u < 4; ++u) s[i][j][u] = fmaf(av[i], kv[u], s[i][j][u]);
      }
    }
    __syncthreads();  // K^T is read out: its space becomes P^T

    // online softmax over this tile's keys
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = q0 + 4 * ty + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int key = k0 + 4 * tx + 32 * j + u;
          const bool ok = key < g.key_limit && (!g.causal || key <= qi);
          s[i][j][u] = ok ? s[i][j][u] * g.scale : -INFINITY;
          mx = fmaxf(mx, s[i][j][u]);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float mn = fmaxf(m[i], mx);
      const float corr = (m[i] == -INFINITY) ? (mn == -INFINITY ? 1.f : 0.f) : expf(m[i] - mn);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float p = s[i][j][u] == -INFINITY ? 0.f : expf(s[i][j][u] - mn);
          s[i][j][u] = p;
          sum += p;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      l[i] = l[i] * corr + sum;
      m[i] = mn;
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int u = 0; u < 4; ++u) o[i][j][u] *= corr;
    }
    float* pt = kt;  // [64 keys][kPLd]: P^T
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = 4 * tx + 32 * j + u;
        *reinterpret_cast<float4*>(pt + c * kPLd + 4 * ty) =
            make_float4(s[0][j][u], s[1][j][u], s[2][j][u], s[3][j][u]);
      }
    __syncthreads();

    // O += P V
#pragma unroll 4
    for (int c = 0; c < kBK; ++c) {
      const float4 p = *reinterpret_cast<const float4*>(pt + c * kPLd + 4 * ty);
      const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const float4 vv = *reinterpret_cast<const float4*>(vs + c * HD + 4 * tx + 32 * j);
        const float vf[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int u = 0; u < 4; ++u) o[i][j][u] = fmaf(pv[i], vf[u], o[i][j][u]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + 4 * ty + i;
    if (qi >= g.q_rows) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    const long long row = (qbase + qi) * g.ldo + col0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int c = 4 * tx + 32 * j;
      const float4 r = make_float4(o[i][j][0] * inv, o[i][j][1] * inv, o[i][j][2] * inv, o[i][j][3] * inv);
      if (g.out_split) {
        uint2 h, lo;
        pack_split(r.x, r.y, h.x, lo.x);
        pack_split(r.z, r.w, h.y, lo.y);
        uint16_t* out = static_cast<uint16_t*>(g.out);
        *reinterpret_cast<uint2*>(out + row + c) = h;
        *reinterpret_cast<uint2*>(out + row + c + g.lo_off) = lo;
      } else {
        *reinterpret_cast<float4*>(static_cast<float*>(g.out) + row + c) = r;
      }
    }
  }
}

template <int HD>
int launch_f32(const AttnF32Args& g, int heads, int batch, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    ND_CUDA(cudaFuncSetAttribute(attention_f32_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 AttnF32Smem<HD>::kBytes));
    configured[dev & 63] = true;
  }
  dim3 grid(static_cast<unsigned>((g.q_rows + kBQ - 1) / kBQ), static_cast<unsigned>(heads),
            static_cast<unsigned>(batch));
  attention_f32_kernel<HD><<<grid, 128, AttnF32Smem<HD>::kBytes, stream>>>(g);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace

int attention_f32(const nd_attention_args& a, cudaStream_t stream) {
  const int hd = a.head_dim;
  if (hd != 128 && hd != 64) return fail(ND_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  if (a.heads <= 0 || a.batch <= 0 || a.q_rows <= 0 || a.kv_rows <= 0)
    return fail(ND_ERR_INVALID, "attention: empty shape");
  if (a.heads > 65535 || a.batch > 65535 || a.q_rows > INT_MAX / 4 || a.kv_rows > INT_MAX / 4)
    return fail(ND_ERR_INVALID, "attention: shape too large");
  if (!a.q || !a.k || !a.v || !a.out) return fail(ND_ERR_INVALID, "attention: null operand");
  const int out_dtype = a.out_dtype ? a.out_dtype : ND_F32;
  if (out_dtype != ND_F32 && out_dtype != ND_BF16X2)
    return fail(ND_ERR_INVALID, "attention: fp32 attention writes f32 or bf16x2");
  const int kvh = a.kv_heads > 0 ? a.kv_heads : a.heads;
  if (a.heads % kvh) return fail(ND_ERR_INVALID, "attention: kv_heads must divide heads");
  const int64_t width = static_cast<int64_t>(a.heads) * hd;
  const int64_t kv_width = static_cast<int64_t>(kvh) * hd;
  if (a.ldq < width || a.ldk < kv_width || a.ldv < kv_width || a.ldq % 4 || a.ldk % 4 || a.ldv % 4)
    return fail(ND_ERR_INVALID, "attention: fp32 q/k/v need ld >= heads (kv_heads) * head_dim, ld % 4 == 0");
  const auto mis16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (mis16(a.q) || mis16(a.k) || mis16(a.v) || mis16(a.out))
    return fail(ND_ERR_INVALID, "attention: operands must be 16-byte aligned");
  if (out_dtype == ND_F32 && (a.ldo < width || a.ldo % 4))
    return fail(ND_ERR_INVALID, "attention: fp32 out needs ldo >= heads * head_dim, ldo % 4 == 0");
  if (out_dtype == ND_BF16X2 && (a.ldo < 2 * width || a.ldo % 4))
    return fail(ND_ERR_INVALID, "attention: bf16x2 out needs ldo >= 2 * heads * head_dim, ldo % 4 == 0");
  if (a.causal && a.q_rows != a.kv_rows) return fail(ND_ERR_INVALID, "attention: causal needs q_rows == kv_rows");

  AttnF32Args g{};
  g.q = static_cast<const float*>(a.q);
  g.k = static_cast<const float*>(a.k);
  g.v = static_cast<const float*>(a.v);
  g.ldq = a.ldq;
  g.ldk = a.ldk;
  g.ldv = a.ldv;
  g.out = a.out;
  g.ldo = a.ldo;
  g.out_split = out_dtype == ND_BF16X2;
  g.lo_off = width;
  g.q_rows = static_cast<int>(a.q_rows);
  g.kv_rows = static_cast<int>(a.kv_rows);
  g.key_limit = static_cast<int>(a.key_limit <= 0 || a.key_limit > a.kv_rows ? a.kv_rows : a.key_limit);
  g.causal = a.causal ? 1 : 0;
  g.kv_group = a.heads / kvh;
  g.scale = a.scale > 0.f ? a.scale : 1.0f / std::sqrt(static_cast<float>(hd));
  return hd == 128 ? launch_f32<128>(g, a.heads, a.batch, stream) : launch_f32<64>(g, a.heads, a.batch, stream);
}

}  // namespace nd
