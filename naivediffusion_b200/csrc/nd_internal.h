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

// ----------------------------------------------------------------- kernels

int linear(const nd_linear_args& a, cudaStream_t stream);
int dequantize(const int8_t* q, const void* scales, int scale_dtype, int64_t quant_group, int64_t rows,
               int64_t cols, void* out, int out_dtype, cudaStream_t stream);
int attention(const nd_attention_args& a, cudaStream_t stream);
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

}  // namespace nd
