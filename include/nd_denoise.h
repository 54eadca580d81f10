/* libnd_denoise — the denoiser forward step of NaiveDiffusion on B200 (sm_100a).
 *
 * C ABI (no C++ or torch types): plain pointers, sizes and an int status
 * (0 = ND_OK). The message of the last failure on the calling thread is in
 * nd_last_error().
 *
 * Two layers:
 *  - the denoiser plug-in (nd_device_*, nd_denoiser_*), the native side of
 *    the reference's IDenoiser (src/NaiveDiffusion/Pipeline/IDenoiser.cs:10-32)
 *    and IModelFamily.BuildDenoiser (Pipeline/IModelFamily.cs:142-143);
 *  - op-level entry points (nd_op_*) over device pointers, the native side of
 *    the operator checks in src/NaiveDiffusion.Cli/SmokeTest.cs, used by the
 *    parity tests and by callers that compose their own blocks.
 */
#ifndef ND_DENOISE_H
#define ND_DENOISE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ND_API __attribute__((visibility("default")))
#else
#define ND_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes
 * Replace the reference's exceptions: ArgumentException /
 * InvalidDataException (shape mismatch, QwenImageDit.cs:110-131),
 * OutOfVideoMemoryException and DeviceRemovedException
 * (Dml/DeviceExceptions.cs:5-21). */
#define ND_OK 0
#define ND_ERR_INVALID 1        /* bad argument or shape */
#define ND_ERR_OOM 2            /* device allocation failed */
#define ND_ERR_CUDA 3           /* CUDA runtime error (device removed, fault) */
#define ND_ERR_TIMEOUT 4        /* a kernel's bounded wait ran out; context still usable */
#define ND_ERR_STATE 5          /* call out of order (e.g. predict before finalize) */
#define ND_ERR_UNSUPPORTED 6    /* configuration this build does not run */
#define ND_ERR_MISSING_WEIGHT 7 /* finalize found a required tensor unset */

/* ------------------------------------------------------------ element types */
#define ND_F32 0
#define ND_F16 1
#define ND_BF16 2
#define ND_I8 3
#define ND_I32 4

/* Message of the last failure on this thread ("" if none). */
ND_API const char* nd_last_error(void);

/* Library version string. */
ND_API const char* nd_version(void);

/* ------------------------------------------------------------ GEMM op
 * y[rows, out] = x[rows, in] . W[out, in]^T (+ bias), with a fused epilogue.
 * Replaces Layers.Linear (src/NaiveDiffusion/Graph/Layers.cs:131-160) ->
 * DmlOps.Gemm (src/NaiveDiffusion/Dml/DmlOps.cs:231-262).
 *
 * Row groups: rows >= group_split use weight rows [out, 2*out) and the
 * second half of bias / gate / qk_norm (a dual-stream block's text rows).
 * group_split must be a multiple of 128 or >= rows (one group). */
#define ND_EPI_STORE 0           /* y = acc + bias                          */
#define ND_EPI_GELU_TANH 1       /* y = gelu_tanh(acc + bias)               */
#define ND_EPI_GELU_ERF 2        /* y = gelu(acc + bias), exact             */
#define ND_EPI_SILU 3            /* y = silu(acc + bias)                    */
#define ND_EPI_RESIDUAL_GATE 4   /* residual(f32) += gate * (acc + bias)    */
#define ND_EPI_STORE_F32 5       /* residual(f32) = acc + bias              */
#define ND_EPI_QK_NORM_ROPE 6    /* cols < qk_cols: head RMSNorm * w, RoPE  */
#define ND_EPI_RESIDUAL_ADD 7    /* residual(f32) += acc + bias             */

typedef struct nd_linear_args {
  int dtype;            /* ND_BF16 or ND_F16: x, W and y */
  int epilogue;         /* ND_EPI_* */
  int64_t rows, in_features, out_features;
  const void* x;        /* [rows, ldx] */
  int64_t ldx;
  const void* weight;   /* [groups * out_features, in_features], row-major */
  const float* bias;    /* [groups * out_features] or NULL */
  int64_t group_split;  /* first row of group 1; >= rows for one group */
  void* y;              /* [rows, ldy] (ND_EPI_STORE, GELU*, SILU, QK_NORM_ROPE) */
  int64_t ldy;
  float* residual;      /* [rows, ldr] fp32 (RESIDUAL_*, STORE_F32) */
  int64_t ldr;
  const float* gate;    /* [groups * out_features] (RESIDUAL_GATE) */
  const float* qk_norm; /* [groups][2][128]: q then k norm weight (QK_NORM_ROPE) */
  const float* rope_cos; /* [rows, 64] */
  const float* rope_sin; /* [rows, 64] */
  int64_t qk_cols;      /* leading columns that are q then k (2 * width) */
  float eps;            /* RMSNorm epsilon */
} nd_linear_args;

/* Device pointers; stream is a cudaStream_t (NULL = legacy default stream).
 * Asynchronous: errors of the launch are returned, kernel faults surface at
 * the next synchronizing call. */
ND_API int nd_op_linear(const nd_linear_args* args, void* stream);

/* ------------------------------------------------------------ attention op
 * O = softmax(Q K^T * scale [+ mask]) V over packed heads, head_dim 128.
 * Replaces Layers.Attend (src/NaiveDiffusion/Graph/Layers.cs:260-279) ->
 * DmlOps.MultiheadAttention (src/NaiveDiffusion/Dml/DmlOps.cs:480-524).
 * Masks: key_limit (keys >= key_limit left out: the KeySequenceLength mask)
 * and causal (row i sees keys 0..i). Batch items are stacked row blocks:
 * item b's queries are rows [b*q_rows, (b+1)*q_rows) of q. */
typedef struct nd_attention_args {
  int dtype;            /* ND_BF16 or ND_F16 */
  int heads, head_dim, batch;
  int64_t q_rows, kv_rows;
  int64_t key_limit;    /* <= 0: all kv_rows keys */
  int causal;
  const void* q; int64_t ldq;  /* head h at columns [h*head_dim, (h+1)*head_dim) */
  const void* k; int64_t ldk;
  const void* v; int64_t ldv;
  void* out; int64_t ldo;
  float scale;          /* <= 0: 1/sqrt(head_dim) */
} nd_attention_args;

ND_API int nd_op_attention(const nd_attention_args* args, void* stream);

/* ------------------------------------------------------------ norms
 * adaLN modulation: y = LayerNorm(x, no affine) * (1 + scale) + shift
 * (Transformer.Modulate, src/NaiveDiffusion/Graph/Transformer.cs:72-80).
 * x fp32; scale/shift fp32 vectors [groups][vec_stride]; rows >= group_split
 * use the second vectors. shift may be NULL. */
typedef struct nd_modulate_args {
  const float* x; int64_t ldx;
  void* y; int64_t ldy; int out_dtype;   /* ND_BF16, ND_F16 or ND_F32 */
  int64_t rows, width;
  const float* shift; const float* scale;
  int64_t vec_stride;   /* 0: width */
  int64_t group_split;  /* >= rows: one group */
  float eps;
} nd_modulate_args;

ND_API int nd_op_modulate(const nd_modulate_args* args, void* stream);

/* RMSNorm over rows: y = x * rsqrt(mean(x^2) + eps) * (weight + plus_one)
 * (Layers.RmsNorm, src/NaiveDiffusion/Graph/Layers.cs:209-221; CpuMath.RmsNorm).
 * weight may be NULL (then the factor is 1). */
typedef struct nd_rmsnorm_args {
  const void* x; int64_t ldx; int in_dtype;
  void* y; int64_t ldy; int out_dtype;
  int64_t rows, width;
  const float* weight;
  int plus_one;         /* zero-centred stored weight (QwenImageDit txt_in norm) */
  float eps;
} nd_rmsnorm_args;

ND_API int nd_op_rmsnorm(const nd_rmsnorm_args* args, void* stream);

/* ------------------------------------------------------------ GEMV
 * y[b, n] = act(sum_k W[n, k] * pre(x[b, k]) + bias[n]), W bf16/f16 [n, k],
 * x and y fp32, batch 1..4. pre_silu applies SiLU to x first; act 0 none,
 * 1 SiLU, 2 tanh. The modulation vectors (Layers.Linear over 1-2 rows). */
typedef struct nd_gemv_args {
  const void* w; int w_dtype;
  int64_t n, k;
  const float* x; int batch; int pre_silu;
  const float* bias; int act;
  float* y;
} nd_gemv_args;

ND_API int nd_op_gemv(const nd_gemv_args* args, void* stream);

/* ------------------------------------------------------------ layout
 * latent [B, C, H, W] fp32 <-> tokens [B * (H/p) * (W/p), C*p*p] (row stride
 * ldt); feature c*p*p + m*p + n of patch (i, j) is channel c at (p*i+m, p*j+n)
 * (AnimaDit.Patchify, src/NaiveDiffusion/Models/Anima/AnimaDit.cs:193-247). */
ND_API int nd_op_patchify(const float* latent, void* tokens, int out_dtype, int batch,
                          int channels, int height, int width, int patch, int64_t ldt,
                          void* stream);
ND_API int nd_op_unpatchify(const float* tokens, int64_t ldt, float* latent, int batch,
                            int channels, int height, int width, int patch, void* stream);

/* Synchronize `stream` and report any kernel's timed-out wait (ND_ERR_TIMEOUT)
 * or CUDA fault (ND_ERR_CUDA) since the last check on this device. */
ND_API int nd_op_sync(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ND_DENOISE_H */
