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

/* Synchronize `stream` and report any kernel's timed-out wait (ND_ERR_TIMEOUT)
 * or CUDA fault (ND_ERR_CUDA) since the last check on this device. */
ND_API int nd_op_sync(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ND_DENOISE_H */
