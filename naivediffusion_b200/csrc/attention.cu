// Host side of the tcgen05 flash-attention kernel (attention_sm100.cuh).
#include <climits>
#include <cmath>

#include "attention_sm100.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

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

  dim3 grid(static_cast<unsigned>((a.q_rows + 255) / 256), static_cast<unsigned>(a.heads),
            static_cast<unsigned>(a.batch));
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  if (hd == 128) {
    static bool configured[64] = {};
    if (!configured[dev & 63]) {
      int rc = check_register_split(reinterpret_cast<const void*>(attention_sm100_kernel<128>), kAttnThreads,
                                    kAttnRegsNeeded, "attention");
      if (rc) return rc;
      ND_CUDA(cudaFuncSetAttribute(attention_sm100_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   AttnSmem<128>::kLaunchBytes));
      configured[dev & 63] = true;
    }
    ND_CUDA(launch_pdl(attention_sm100_kernel<128>, grid, dim3(kAttnThreads), AttnSmem<128>::kLaunchBytes, stream, tq, tk, tv, g));
  } else {
    static bool configured[64] = {};
    if (!configured[dev & 63]) {
      int rc = check_register_split(reinterpret_cast<const void*>(attention_sm100_kernel<64>), kAttnThreads,
                                    kAttnRegsNeeded, "attention");
      if (rc) return rc;
      ND_CUDA(cudaFuncSetAttribute(attention_sm100_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   AttnSmem<64>::kLaunchBytes));
      configured[dev & 63] = true;
    }
    ND_CUDA(launch_pdl(attention_sm100_kernel<64>, grid, dim3(kAttnThreads), AttnSmem<64>::kLaunchBytes, stream, tq, tk, tv, g));
  }
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd
