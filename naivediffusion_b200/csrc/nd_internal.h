// Host-side internals shared by the translation units of libnd_denoise.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/nd_denoise.h"

namespace nd {

// ----------------------------------------------------------------- errors

// Record a message for nd_last_error() and return `code`.
int fail(int code, const std::string& msg);
// Map a CUDA runtime error to a status (ND_ERR_OOM / ND_ERR_CUDA), recording it.
int cuda_fail(cudaError_t e, const char* what);
// Current device's SM count (cached per device).
int sm_count();

#define ND_CUDA(call)                                   \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return ::nd::cuda_fail(e_, #call); \
  } while (0)

// ----------------------------------------------------------------- TMA

// A 2-D tensor map over a row-major [rows, cols] matrix of `elem_bytes`
// elements with leading dimension `ld` (elements), box [box_rows, box_cols],
// 128-byte swizzle (box_cols * elem_bytes must be 128) or none.
int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, int64_t rows, int64_t cols,
                 int64_t ld, int box_rows, int box_cols, bool swizzle128);
// Same with an explicit element type (ND_F32 for a float reduce-add) and
// swizzle span in bytes (0, 32, 64 or 128).
int make_tmap_2d_typed(CUtensorMap* map, const void* base, int nd_dtype, int64_t rows, int64_t cols,
                       int64_t ld, int box_rows, int box_cols, int swizzle_bytes);

// A 4-D tensor map (innermost first) with a [box] and traversal strides.
int make_tmap_4d(CUtensorMap* map, const void* base, int nd_dtype, const int64_t dims[4],
                 const int64_t strides_bytes[3], const int box[4], const int elem_strides[4],
                 int swizzle_bytes);

// ----------------------------------------------------------------- kernels

int linear(const nd_linear_args& a, cudaStream_t stream);
int conv2d(const nd_conv_args& c, cudaStream_t stream);
int dequantize(const int8_t* q, const void* scales, int scale_dtype, int64_t quant_group, int64_t rows,
               int64_t cols, void* out, int out_dtype, cudaStream_t stream);
// A kernel that moves registers between its warpgroups (setmaxnreg) may only
// hand out what it was launched with: fail unless the compiled per-thread
// count x threads covers `needed`.
int check_register_split(const void* kernel, int threads, int needed, const char* what);
int attention(const nd_attention_args& a, cudaStream_t stream);
// Bytes of nd_attention_args::workspace for head_dim 64 / 128 (0 otherwise).
int64_t attention_workspace_bytes(int head_dim);
int attention_f32(const nd_attention_args& a, cudaStream_t stream);
int sampler_step(const nd_sampler_args& a, cudaStream_t stream);
int modulate(const nd_modulate_args& a, cudaStream_t stream);
int rmsnorm(const nd_rmsnorm_args& a, cudaStream_t stream);
int gemv(const nd_gemv_args& a, cudaStream_t stream);
int gemv_w8(const nd_gemv_args& a, cudaStream_t stream);
int quantize_weights(const void* src, int src_dtype, int64_t rows, int64_t cols, int64_t group,
                     int scale_f16, int8_t* q, void* scales, cudaStream_t stream);
int patchify(const float* lat, void* tok, int out_dtype, int B, int C, int H, int W, int p,
             int64_t ldt, cudaStream_t stream);
int unpatchify(const float* tok, int64_t ldt, float* lat, int B, int C, int H, int W, int p,
               cudaStream_t stream);
// UNet (NHWC) kernels
size_t group_norm_scratch(int B, int HW, int C, int G);
int group_norm(const void* x, void* y, int dtype, int B, int HW, int C, int G, const float* w,
               const float* bias, float eps, int silu_after, void* scratch, size_t scratch_bytes,
               cudaStream_t s);
int geglu(const void* in, void* out, int dtype, int64_t rows, int64_t F, cudaStream_t s);
int upsample2x(const void* in, void* out, int B, int H, int W, int C, cudaStream_t s);
int concat_channels(const void* a, int ca, const void* b, int cb, void* out, int64_t pixels, cudaStream_t s);
int nchw_to_nhwc(const float* in, void* out, int dtype, int B, int C, int HW, int cpad, cudaStream_t s);
int nhwc_to_nchw(const float* in, float* out, int B, int C, int HW, cudaStream_t s);
int add_vectors(float* dst, const float* src, int64_t n, cudaStream_t s);          // dst += src
int add_vectors2(float* out, const float* a, const float* b, int64_t n, cudaStream_t s);  // out = a + b

}  // namespace nd
