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
/* An fp32 tensor carried as a pair of bf16 tensors so that the bf16 tensor
 * cores can multiply it at fp32 accuracy. A [rows, cols] value v is stored
 * [rows, 2 * cols]: hi = bf16(v) in columns [0, cols), lo = bf16(v - hi) in
 * [cols, 2 * cols) (round to nearest even both times; |v - hi - lo| <=
 * 2^-16 |v|). The GEMM sums hi.hi + hi.lo + lo.hi in fp32 (three passes over
 * K on the same tcgen05 pipeline); the dropped lo.lo term is below 2^-16 of
 * each product. This is how model_desc.compute == ND_F32 runs. */
#define ND_BF16X2 5

/* Message of the last failure on this thread ("" if none). */
ND_API const char* nd_last_error(void);

/* Library version string. */
ND_API const char* nd_version(void);

/* ------------------------------------------------------------ denoiser plug-in
 * The native side of IDenoiser (src/NaiveDiffusion/Pipeline/IDenoiser.cs:10-32):
 * a model is created from a description, its weights are copied into HBM
 * once (set_weight), then predict() runs one forward step per call. Weights
 * stay resident (no streaming); the caller's host buffers are only read
 * during the call that receives them. One caller at a time per handle, as
 * the reference's DmlDevice (Dml/DmlDevice.cs:9-14). */
#define ND_FAMILY_MMDIT 0   /* Qwen-Image-style dual-stream DiT (60 x 3072 at full size) */
#define ND_FAMILY_ANIMA 1   /* Anima / Cosmos-Predict2 DiT (Models/Anima/AnimaDit.cs) */
#define ND_FAMILY_SDXL 2    /* SDXL UNet (Models/Sdxl/UNetModel.cs) */
#define ND_FAMILY_VAE_KL 3  /* AutoencoderKL decoder (Vae/AutoencoderKl.cs), the SDXL VAE:
                               predict() takes the VAE latent (already divided by the
                               scaling factor) and returns the [batch, 3, 8h, 8w] image;
                               width = base channels, unet_mult = block_out_channels /
                               width, unet_resnets = layers_per_block; no conditioning */
#define ND_FAMILY_QWEN_IMAGE 4 /* Qwen-Image 2.1 single-stream DiT (Models/QwenImage/
                               QwenImageDit.cs): image rows then text rows through
                               shared weights, one modulation for every block (the
                               noise level's row for image rows, time zero's for text
                               rows), SwiGLU feed-forward, image queries over every
                               visible key, text queries causal over the text; patch 1 */
#define ND_FAMILY_VAE_WAN21 5  /* Wan 2.1 VAE decoder on one frame (Vae/WanVae.cs), Anima's:
                               width = base dim (96), latent_channels 16, 8x upsampling;
                               unet_resnets = resblocks per level - 1 (2); weights as
                               WanVae.SingleFrame leaves them (3-D kernels cut to their
                               last temporal tap); output [batch, 3, 8h, 8w] */
#define ND_FAMILY_VAE_WAN22 6  /* Wan 2.2-layout VAE decoder of Qwen-Image 2.1
                               (Vae/Wan22Vae.cs): width 144, latent_channels 64, five
                               levels, 16x upsampling, the up shortcuts; the RGB of
                               its RGBA output, [batch, 3, 16h, 16w] */
#define ND_FAMILY_QWEN3_TEXT 7 /* Qwen3 decoder as a text encoder (Text/Qwen/Qwen3TextModel.cs):
                               width, heads x head_dim 128, kv_heads, blocks = layers,
                               mlp_width, vocab, rope_theta; context_rows = most tokens
                               per call; run with nd_text_encode */
#define ND_FAMILY_LLM_ADAPTER 8 /* Anima's LLM adapter (Models/Anima/LlmAdapter.cs): width
                               1024, heads 16 x 64, blocks 6, mlp_width 4096, vocab (T5),
                               rope_theta 1e4; context_rows = most T5 ids per call,
                               source_rows = most Qwen3 rows; run with nd_text_encode */

typedef struct nd_device nd_device;
typedef struct nd_denoiser nd_denoiser;

typedef struct nd_model_desc {
  int family;                 /* ND_FAMILY_* */
  int width, heads, head_dim; /* transformer width, heads x head_dim == width */
  int blocks, mlp_width;
  int context_rows, context_width; /* text rows per predict and their width */
  int latent_channels, latent_height, latent_width, patch;
  int time_width;             /* sinusoid width of the timestep embedder */
  int batch;                  /* latents per predict (stacked CFG branches): 1..4; the VAE
                                 decoders 1..64 (a tiled decode's tiles) */
  int compute;                /* ND_BF16 (DiTs), ND_F16 (SDXL), or ND_F32 (the DiTs' fp32
                                 mode: bf16 hi|lo operand pairs on the tensor cores) */
  int weight_dtype;           /* storage: the compute dtype, or ND_I8 (weight-only, 16-bit compute) */
  int quant_group;            /* int8: columns per scale (32 = BlockQuantizer); 0 = per output channel */
  int quant_scale_dtype;      /* int8: ND_F16 (BlockQuantizer) or ND_F32 */
  int adaln_rank;             /* Anima: rank of the low-rank adaLN (256) */
  float eps;                  /* norm epsilon (1e-6 for the DiTs) */
  /* SDXL UNet levels (UNetModel.cs:20-40): channel multiplier of `width` and
   * transformer depth per level, resnets per level; 0 levels: SDXL's
   * {1, 2, 4} x 320, depths {0, 2, 10}, 2 resnets. */
  int unet_levels;
  int unet_mult[4];
  int unet_depth[4];
  int unet_resnets;
  int add_width;              /* SDXL: width of the "add" conditioning (2816) */
  /* text towers (ND_FAMILY_QWEN3_TEXT, ND_FAMILY_LLM_ADAPTER) */
  int kv_heads;               /* key / value heads (grouped-query attention; 0 = heads) */
  int vocab;                  /* rows of the token embedding table */
  int source_rows;            /* LLM adapter: most Qwen3 rows one call cross-attends to */
  double rope_theta;          /* rotary base (Qwen3-0.6B 1e6, Qwen3-VL-8B 5e6, adapter 1e4) */
} nd_model_desc;

typedef struct nd_named_tensor {
  const char* name;
  int dtype;                  /* ND_F32 / ND_I32 ... */
  int rank;
  const int64_t* shape;
  const void* data;
} nd_named_tensor;

typedef struct nd_memory {
  uint64_t persistent_bytes;  /* folded weights, wherever they are */
  uint64_t streamed_bytes;    /* of those, read from system memory per step (always 0) */
  uint64_t resident_bytes;    /* of those, in HBM */
  uint64_t temporary_bytes;   /* scratch one step needs on top */
  int graph_count;            /* captured CUDA graphs */
} nd_memory;

/* Open device `ordinal` (its own CUDA stream). */
ND_API int nd_device_open(int ordinal, nd_device** out);
ND_API int nd_device_close(nd_device* dev);

/* IModelFamily.BuildDenoiser (Pipeline/IModelFamily.cs:142-143): allocate the
 * model's resident weights and scratch for `desc`. */
ND_API int nd_denoiser_create(nd_device* dev, const nd_model_desc* desc, nd_denoiser** out);

/* Name and 2-D shape ([rows, cols]; vectors [n, 1]) of expected tensor
 * `index` (0-based); ND_ERR_INVALID past the last. `required` is 0 for
 * tensors that default to zero (biases). */
ND_API int nd_denoiser_weight_info(const nd_denoiser* d, int index, const char** name,
                                   int64_t* rows, int64_t* cols, int* required);

/* Copy one tensor into HBM, converting to the storage type. `data` is host
 * memory (set_weight) or device memory of the same device (set_weight_device);
 * dtype ND_F32 / ND_F16 / ND_BF16. The shape must match weight_info. */
ND_API int nd_denoiser_set_weight(nd_denoiser* d, const char* name, int dtype,
                                  const int64_t* shape, int rank, const void* data);
ND_API int nd_denoiser_set_weight_device(nd_denoiser* d, const char* name, int dtype,
                                         const int64_t* shape, int rank, const void* data);

/* A matrix already quantized on the host by BlockQuantizer
 * (Tensors/BlockQuantizer.cs:34-105): q int8 [rows, cols] and scales
 * [rows, cols / quant_group] (quant_group 32, scale_dtype ND_F16: the
 * reference's blocks) or [rows] (quant_group 0, ND_F32: per output channel),
 * host memory. Only for a model created with weight_dtype ND_I8, whose group
 * and scale type must match. Matrices given through set_weight instead are
 * quantized on the device by the same rules, bit for bit. */
ND_API int nd_denoiser_set_weight_q8(nd_denoiser* d, const char* name, const int64_t* shape, int rank,
                                     const int8_t* q, int scale_dtype, const void* scales,
                                     int64_t quant_group);

/* Quantize a matrix on the device (the same rules): src [rows, cols] f32 /
 * f16 / bf16 device memory -> q int8 [rows, cols] and scales. */
ND_API int nd_op_quantize(const void* src, int src_dtype, int64_t rows, int64_t cols,
                          int64_t quant_group, int scale_dtype, int8_t* q, void* scales,
                          void* stream);

/* Check every required tensor was set and prepare the step (ND_ERR_MISSING_WEIGHT). */
ND_API int nd_denoiser_finalize(nd_denoiser* d);

/* IDenoiser.Predict: latent [batch, C, H, W] fp32 host memory in, the model's
 * prediction (same shape, fp32) out. timestep is the training-table index
 * (UNet), sigma the noise level (flow models' time). Conditioning by name:
 *   MMDiT: "context" [batch, rows, context_width] f32 (required);
 *          "cos", "sin" [image tokens + rows, 64] f32 (default: the
 *          reference's Qwen-Image rotary tables with text length = rows);
 *          "key_length" i32 [1] (visible keys; default all).
 *   QWEN_IMAGE (QwenImageConditioning, Models/QwenImage/QwenImageConditioner.cs):
 *          "context" [1, rows, context_width] f32 (required, zero-padded rows);
 *          "key_length" i32 [1] = image tokens + real text rows (default all);
 *          "text_mask" i32 [rows, rows] (optional; must be the causal table
 *          closed over the padding for that real length: row i reads key j
 *          iff j <= i and j < real; checked when given in host memory);
 *          "cos", "sin" [image tokens + rows, 64] f32 (default: the
 *          reference's tables with text length = the real rows).
 *   SDXL: "context" [batch, 77, 2048], "add" [batch, 2816] f32.
 * Synchronous. */
ND_API int nd_denoiser_predict(nd_denoiser* d, const float* latent, double timestep, double sigma,
                               int n_cond, const nd_named_tensor* cond, float* out);

/* The same with latent, conditioning data and out in device memory, enqueued
 * on `stream` (NULL: the device's own stream); returns after enqueueing. */
ND_API int nd_denoiser_predict_device(nd_denoiser* d, const float* latent, double timestep,
                                      double sigma, int n_cond, const nd_named_tensor* cond,
                                      float* out, void* stream);

/* The text towers, the step before the path: Qwen3TextModel.Forward
 * (Text/Qwen/Qwen3TextModel.cs:47-104) for ND_FAMILY_QWEN3_TEXT and
 * LlmAdapter.Forward (Models/Anima/LlmAdapter.cs:29-78) for
 * ND_FAMILY_LLM_ADAPTER, on a denoiser handle of that family (weights set
 * and finalized as for the denoisers). ids: `rows` token ids in host memory
 * (rows <= desc.context_rows, every id < desc.vocab); source: the adapter's
 * Qwen3 hidden states [source_rows, width] fp32 host (NULL, 0 for Qwen3);
 * final_norm: Qwen3 only, 1 = through model.norm (what Anima's adapter reads),
 * 0 = the last block's output (what Qwen-Image 2.1 reads). out: [rows, width]
 * fp32 host. Synchronous. */
ND_API int nd_text_encode(nd_denoiser* d, const int32_t* ids, int rows, const float* source, int source_rows,
                          int final_norm, float* out);

/* Per-head RMSNorm then rotate-half RoPE, in place (Transformer.HeadNorm +
 * Transformer.Rotate, Graph/Transformer.cs:37-64; CpuMath.RmsNorm + Rope):
 * x [rows, ld] bf16 / f16 / f32, heads of head_dim (64 or 128) from column 0;
 * each head's features times rsqrt(mean(x^2) + eps) * weight[head_dim], then
 * rotated by row r's angles cos / sin [rows, head_dim / 2] (NULL: no rotation). */
ND_API int nd_op_head_norm_rope(void* x, int dtype, int64_t ld, int64_t rows, int heads, int head_dim,
                                const float* weight, const float* cos, const float* sin, float eps,
                                void* stream);

/* Per-kernel-class timing: run the step `steps` times eagerly on the last
 * staged inputs with a CUDA event pair around every launch, and return per
 * class (e.g. "gemm.qkv", "attention") the launches, device milliseconds,
 * algorithmic FLOPs and bytes of ONE step (times averaged over the runs).
 * Launches shorter than the host's enqueue time read long. The
 * reference's counterpart is MemoryLog's per-stage report
 * (src/NaiveDiffusion/Dml/MemoryLog.cs:110-224) and DenoiseCommand's
 * Stopwatch (NaiveDiffusion.Cli/DenoiseCommand.cs:139-144). */
typedef struct nd_kernel_time {
  const char* name;     /* static string owned by the library */
  int launches;
  double total_ms;
  double flops;
  double bytes;
} nd_kernel_time;

ND_API int nd_denoiser_profile(nd_denoiser* d, int steps, nd_kernel_time* out, int max_entries,
                               int* n_entries);

/* IDenoiser's memory figures. */
ND_API int nd_denoiser_memory(const nd_denoiser* d, nd_memory* out);
ND_API int nd_denoiser_destroy(nd_denoiser* d);

/* ------------------------------------------------------------ GEMM op
 * y[rows, out] = x[rows, in] . W[out, in]^T (+ bias), with a fused epilogue.
 * Replaces Layers.Linear (src/NaiveDiffusion/Graph/Layers.cs:131-160) ->
 * DmlOps.Gemm (src/NaiveDiffusion/Dml/DmlOps.cs:231-262).
 *
 * Row groups: rows >= group_split use weight rows [out, 2*out) and the
 * second half of bias / gate / qk_norm (a dual-stream block's text rows).
 * group_split must be a multiple of 128 or >= rows (one group). With
 * shared_weights = 1 every row reads weight rows [0, out) and only bias and
 * gate differ per group, chosen per row (a single-stream block's image and
 * text rows under their own modulation), so group_split may be any row;
 * QK_NORM_ROPE then uses the first group's bias and norm weights. */
#define ND_EPI_STORE 0           /* y = acc + bias                          */
#define ND_EPI_GELU_TANH 1       /* y = gelu_tanh(acc + bias)               */
#define ND_EPI_GELU_ERF 2        /* y = gelu(acc + bias), exact             */
#define ND_EPI_SILU 3            /* y = silu(acc + bias)                    */
#define ND_EPI_RESIDUAL_GATE 4   /* residual(f32) += gate * (acc + bias)    */
#define ND_EPI_STORE_F32 5       /* residual(f32) = acc + bias              */
#define ND_EPI_QK_NORM_ROPE 6    /* cols < qk_cols: head RMSNorm * w, RoPE  */
#define ND_EPI_RESIDUAL_ADD 7    /* residual(f32) += acc + bias             */
#define ND_EPI_ADD_STORE 8       /* y = acc + bias + addend (like y)        */
#define ND_EPI_SWIGLU 9          /* y[:, j] = silu(g_j + bias_j) * (u_j + bias_F+j),
                                    g = x W[0:F]^T, u = x W[F:2F]^T: W is the
                                    fused [gate; up] matrix [2F, in], out_features
                                    = F (a multiple of 128), bias [2F] or NULL
                                    (QwenImageDit.FeedForward) */
#define ND_EPI_GEGLU 10          /* y[:, j] = (h_j + bias_j) * gelu(g_j + bias_F+j), exact
                                    GELU, W = [h; g] [2F, in] (UNetLayers.Geglu) */

typedef struct nd_linear_args {
  int dtype;            /* ND_BF16 or ND_F16: x, W and y. ND_BF16X2 (fp32
                           compute): x [rows, 2 * in] and W [groups * out,
                           2 * in] are hi|lo pairs, in % 64 == 0; STORE, GELU*
                           and SILU write y as a pair [rows, 2 * out];
                           QK_NORM_ROPE writes y as fp32 [rows, out] (the
                           attention input); ADD_STORE is not offered */
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
  const float* gate;    /* [groups][gate_stride] (RESIDUAL_GATE) */
  int64_t gate_stride;  /* 0: out_features */
  const float* qk_norm; /* [groups][2][128]: q then k norm weight (QK_NORM_ROPE) */
  const float* rope_cos; /* [rows, 64] */
  const float* rope_sin; /* [rows, 64] */
  int64_t qk_cols;      /* leading columns that are q then k (2 * width) */
  float eps;            /* RMSNorm epsilon */
  /* int8 weight-only (BlockQuantizer scheme, Tensors/BlockQuantizer.cs:34-105):
   * weight_dtype ND_I8 makes `weight` int8 [groups * out, in] and widens
   * w = q * scale inside the GEMM; scales [groups * out, in / quant_group]
   * (quant_group 32: the reference's blocks) or [groups * out] (quant_group 0:
   * per output channel), dtype scale_dtype (ND_F16 or ND_F32).
   * weight_dtype 0 (or == dtype): weights are already bf16 / fp16. */
  int weight_dtype;
  const void* scales;
  int scale_dtype;
  int64_t quant_group;
  /* QK_NORM_ROPE details: columns [0, qk_cols) are normed, each run of
   * norm_span columns with its own 128-wide weight (qk_norm[group][col /
   * norm_span]; 0 = qk_cols / 2: q then k). rope_cos == NULL: norm only, no
   * rotation (cross-attention). rope_period: table row = row % rope_period
   * (0 = row), for batch items stacked by rows. */
  int64_t norm_span;
  int64_t rope_period;
  const void* addend;   /* ADD_STORE: [rows, ld_add], dtype like y */
  int64_t ld_add;
  int shared_weights;   /* 1: one weight matrix for both row groups (see above) */
} nd_linear_args;

/* ------------------------------------------------------------ conv op
 * 3x3 convolution, padding 1, stride 1 or 2, NHWC activations, as an
 * implicit GEMM on the same tcgen05 mainloop: rows = output pixels, K = the
 * nine taps x input channels, each tap's patch loaded by TMA straight from the
 * input (borders zero-filled). Replaces Layers.Conv2d
 * (src/NaiveDiffusion/Graph/Layers.cs:115-128) -> DmlOps.Convolution
 * (src/NaiveDiffusion/Dml/DmlOps.cs:265). Limits: in_channels a multiple of
 * 8, at least 64; output width divides 128 or is a multiple of 128; output
 * pixels per image a multiple of 128. */
typedef struct nd_conv_args {
  int dtype;            /* ND_F16 or ND_BF16 */
  int epilogue;         /* ND_EPI_STORE, ND_EPI_ADD_STORE, ND_EPI_STORE_F32, ND_EPI_SILU */
  int batch, height, width, in_channels, out_channels, stride;
  const void* x;        /* [batch, height, width, in_channels] */
  const void* weight;   /* [out_channels, 3, 3, in_channels rounded up to 64], the pad zero */
  const float* bias;    /* [out_channels], or [batch][out_channels] with per_batch_bias */
  int per_batch_bias;   /* the ResBlock's time-embedding projection folded into the bias */
  int64_t bias_stride;  /* per_batch_bias: floats between batch items' bias vectors (0: out_channels) */
  void* y;              /* [batch, H_out, W_out, out_channels] */
  float* y_f32;         /* STORE_F32 output */
  const void* addend;   /* ADD_STORE: like y */
} nd_conv_args;

ND_API int nd_op_conv2d(const nd_conv_args* args, void* stream);

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
  int dtype;            /* ND_BF16 or ND_F16 (tensor cores, head_dim 64 / 128), or
                           ND_F32 (fp32 on the CUDA cores, head_dim 64 / 128) */
  int heads, head_dim, batch;
  int64_t q_rows, kv_rows;
  int64_t key_limit;    /* <= 0: all kv_rows keys */
  int causal;
  const void* q; int64_t ldq;  /* head h at columns [h*head_dim, (h+1)*head_dim) */
  const void* k; int64_t ldk;
  const void* v; int64_t ldv;
  void* out; int64_t ldo;
  float scale;          /* <= 0: 1/sqrt(head_dim) */
  int out_dtype;        /* 0: dtype. With dtype ND_F32 also ND_BF16X2: out is a
                           hi|lo pair [rows, 2 * heads * head_dim] (ldo counts
                           bf16 elements) */
  int kv_heads;         /* 0: heads. Fewer (dividing heads) is grouped-query
                           attention: query head h reads key / value head
                           h / (heads / kv_heads) (CpuMath.Attention,
                           Tensors/CpuMath.cs:196-248); k and v are then
                           [rows, kv_heads * head_dim] */
  void* workspace;      /* NULL, or nd_attention_workspace_bytes(head_dim) bytes,
                           zero-filled once before first use (the kernel leaves
                           it zeroed). With it, when the (query-tile pair x head
                           x batch) units do not fill the last wave of SMs, the
                           16-bit non-causal kernel splits the last wave's units
                           along the keys and merges the pieces in a fixed order
                           (bit-identical from run to run). One workspace per
                           stream: launches that share one must be ordered. */
  int64_t workspace_bytes;
} nd_attention_args;

ND_API int nd_op_attention(const nd_attention_args* args, void* stream);

/* Bytes of the workspace above for head_dim 64 or 128 on the current device
 * (0 for other head dims). */
ND_API int64_t nd_attention_workspace_bytes(int head_dim);

/* ------------------------------------------------------------ norms
 * adaLN modulation: y = LayerNorm(x, no affine) * (1 + scale) + shift
 * (Transformer.Modulate, src/NaiveDiffusion/Graph/Transformer.cs:72-80).
 * x fp32; scale/shift fp32 vectors [groups][vec_stride]; rows >= group_split
 * use the second vectors. shift may be NULL. */
typedef struct nd_modulate_args {
  const float* x; int64_t ldx;
  void* y; int64_t ldy; int out_dtype;   /* ND_BF16, ND_F16, ND_F32, or ND_BF16X2
                                            (y [rows, 2 * width] hi|lo pair) */
  int64_t rows, width;
  const float* shift; const float* scale;
  int64_t vec_stride;   /* 0: width */
  int64_t group_split;  /* >= rows: one group */
  float eps;
  int affine;           /* 1: y = LayerNorm(x) * scale + shift (a plain nn.LayerNorm,
                           Layers.LayerNorm, Graph/Layers.cs:189-207) */
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
  int silu;             /* 1: y = silu(y) after the norm (WanVae's norm + SiLU pairs) */
} nd_rmsnorm_args;

ND_API int nd_op_rmsnorm(const nd_rmsnorm_args* args, void* stream);

/* ------------------------------------------------------------ GEMV
 * y[b, n] = act(sum_k W[n, k] * pre(x[b, k]) + bias[n]), W bf16/f16 [n, k],
 * x and y fp32, batch 1..4. pre_silu applies SiLU to x first; act 0 none,
 * 1 SiLU, 2 tanh. The modulation vectors (Layers.Linear over 1-2 rows). */
typedef struct nd_gemv_args {
  const void* w; int w_dtype;   /* ND_BF16 / ND_F16, ND_BF16X2 ([n, 2k] hi|lo
                                   pair), or ND_I8 with scales */
  int64_t n, k;
  const float* x; int batch; int pre_silu;
  const float* bias; int act;
  float* y;
  const void* scales; int scale_dtype; int64_t quant_group;  /* int8 weights only */
  int64_t x_rows_per_vec;  /* > 0: output row n reads input vector n / x_rows_per_vec (batch 1) */
  int64_t bias_period;     /* > 0: bias index n % bias_period */
} nd_gemv_args;

ND_API int nd_op_gemv(const nd_gemv_args* args, void* stream);

/* ------------------------------------------------------------ UNet ops
 * GroupNorm over NHWC fp16/bf16: groups of channels normalized over
 * (pixels, C/groups), then y = n * weight[c] + bias[c], optionally SiLU
 * (Layers.GroupNorm, src/NaiveDiffusion/Graph/Layers.cs:166-185, and the
 * ResBlocks' SiLU, Models/Sdxl/UNetModel.cs:230-254). x, y: [batch, pixels,
 * channels], batch <= 1024; weight / bias may be NULL (1 / 0). Uses
 * library-owned device scratch for its partial sums (allocated zeroed on
 * first use per device and grown when a larger shape needs it). Two
 * launches: the partial sums (whose last block per image forms the group
 * statistics) and the normalization. */
ND_API int nd_op_group_norm(const void* x, void* y, int dtype, int batch, int pixels, int channels,
                            int groups, const float* weight, const float* bias, float eps,
                            int silu_after, void* stream);

/* nd_op_group_norm that allocates no memory (no counterpart in the reference:
 * its DirectML graphs own their temporaries). Same arguments, same kernels,
 * same results. Its scratch is one fixed 4 MiB device array inside the
 * library, so it suits hosts that cannot let the library allocate: device
 * memory already fully committed (a serving pool, full weight residency), or
 * a pipeline that must not meet cudaFree's device-wide wait.
 *  - Limit: 4096 + batch * ceil(pixels / 32) * groups * 8 (rounded up to
 *    256) + batch * groups * 8 + 256 bytes must fit in 4 MiB (SDXL at 1024
 *    x 1024, batch 2: 0.27 MB; at 32 groups up to about 512 K pixels over
 *    the batch); larger shapes fail with ND_ERR_INVALID and launch nothing.
 *  - The array's first 4 KB are one arrival counter per image (batch <=
 *    1024): zero when the library loads, and every call leaves them zero
 *    (the last block of each image resets its counter). Partial sums and
 *    group statistics are written before they are read within a call.
 *  - The first call on each device looks up the array's address (with that
 *    device current); make that first call before any stream capture. The
 *    address stays valid for the life of the device's CUDA context: a process
 *    that calls cudaDeviceReset must not call this entry point afterwards
 *    (the cached address would point into the destroyed context).
 *  - One array per device: calls in flight at the same time on one device
 *    (different streams or host threads) race on it. Calls on one stream,
 *    or otherwise ordered, are fine. */
ND_API int nd_op_group_norm_noalloc(const void* x, void* y, int dtype, int batch, int pixels, int channels,
                                    int groups, const float* weight, const float* bias, float eps,
                                    int silu_after, void* stream);

/* GEGLU: in [rows, 2F] -> out [rows, F] = in[:, :F] * gelu(in[:, F:])
 * (UNetLayers.Geglu, src/NaiveDiffusion/Models/Sdxl/UNetLayers.cs:30-46). */
ND_API int nd_op_geglu(const void* in, void* out, int dtype, int64_t rows, int64_t F, void* stream);

/* ------------------------------------------------------------ layout
 * latent [B, C, H, W] fp32 <-> tokens [B * (H/p) * (W/p), C*p*p] (row stride
 * ldt); feature c*p*p + m*p + n of patch (i, j) is channel c at (p*i+m, p*j+n)
 * (AnimaDit.Patchify, src/NaiveDiffusion/Models/Anima/AnimaDit.cs:193-247).
 * out_dtype ND_BF16X2: the lo half of feature f sits at column C*p*p + f. */
ND_API int nd_op_patchify(const float* latent, void* tokens, int out_dtype, int batch,
                          int channels, int height, int width, int patch, int64_t ldt,
                          void* stream);
ND_API int nd_op_unpatchify(const float* tokens, int64_t ldt, float* latent, int batch,
                            int channels, int height, int width, int patch, void* stream);

/* ------------------------------------------------------------ tiled VAE
 * The reference decodes in overlapping square tiles by default
 * (GenerationOptions.TileVae, src/NaiveDiffusion/Pipeline/GenerationOptions.cs:79;
 * TiledVaeDecoder.Run, src/NaiveDiffusion/Vae/TiledVae.cs:136-159). Here every
 * tile goes through the decoder in ONE batch: a VAE decoder created for the
 * tile's size with batch = the tile count (each batch item is normalised on
 * its own, as a tile run alone is).
 *   nd_op_tile_gather: latent [channels, height, width] fp32 -> tiles
 *     [n_rows * n_cols, channels, tile, tile], tile (i, j) starting at
 *     (rows[i], cols[j]) (CopyTile, TiledVae.cs:67-82).
 *   nd_op_tile_blend: decoded tiles [n_rows * n_cols, channels, side, side]
 *     -> out [channels, height, width]: each tile weighted by
 *     vertical[y] * horizontal[x] (VaeTiling.Window), summed over the tiles in
 *     row-then-column order together with the weights, then multiplied by the
 *     reciprocal of the weight sum (BlendTile / DivideByWeights,
 *     TiledVae.cs:84-121), one rounding per float operation as there: for the
 *     same tiles the result is bit-identical to the reference's.
 * rows / cols: HOST arrays of 1..256 tile origins (latent cells for the
 * gather, pixels for the blend), each tile inside the image (ND_ERR_INVALID
 * otherwise); vertical / horizontal: DEVICE arrays of `side` floats
 * (VaeTiling.Crossfade); channels <= 16 for the blend. */
ND_API int nd_op_tile_gather(const float* latent, int channels, int height, int width, const int32_t* rows,
                             int n_rows, const int32_t* cols, int n_cols, int tile, float* tiles, void* stream);
ND_API int nd_op_tile_blend(const float* tiles, int channels, int side, const int32_t* rows, int n_rows,
                            const int32_t* cols, int n_cols, const float* vertical, const float* horizontal,
                            float* out, int height, int width, void* stream);

/* Widen int8 weights: out[r, c] = round(q[r, c] * scale(r, c)) in out_dtype
 * (ND_BF16 or ND_F16), scale as in nd_linear_args (quant_group 32 or 0). The
 * same arithmetic the int8 GEMM applies to its tiles (DmlOps.Dequantize,
 * src/NaiveDiffusion/Dml/DmlOps.cs:208-228). */
ND_API int nd_op_dequantize(const int8_t* q, const void* scales, int scale_dtype,
                            int64_t quant_group, int64_t rows, int64_t cols, void* out,
                            int out_dtype, void* stream);

/* ------------------------------------------------------------ sampler step
 * One solver step on the device, fused with the guidance combine, so the
 * latent never leaves HBM between denoiser calls: per element
 *   prediction = branches == 2 ? uncond + guidance * (cond - uncond) : out
 *   sample     = the sampler's update of `sample` with that prediction
 * in the reference's arithmetic, operation by operation (float where it
 * computes in float, double where it does), so a step is bit-identical to
 * the reference's CPU one:
 *   ClassifierFreeGuidance.Combine (Pipeline/GuidanceStrategy.cs:32-41),
 *   EulerScheduler / EulerAncestralScheduler / DpmPlusPlus2MScheduler /
 *   DpmPlusPlus2MSdeScheduler.Step (Sampling/Schedulers.cs:263-445), with the
 *   prediction types' Denoise / Derivative / Renoise (Sampling/Prediction.cs).
 * The per-step scalars the reference computes in double (log, sqrt of the
 * sigmas) are passed in, computed on the host as it does: see the comments. */
#define ND_SAMPLER_EULER 0
#define ND_SAMPLER_EULER_A 1
#define ND_SAMPLER_DPMPP_2M 2
#define ND_SAMPLER_DPMPP_2M_SDE 3
#define ND_PRED_EPSILON 0
#define ND_PRED_VELOCITY 1
#define ND_PRED_FLOW 2

typedef struct nd_sampler_args {
  int sampler;               /* ND_SAMPLER_* */
  int prediction;            /* ND_PRED_* */
  int64_t n;                 /* elements of one latent */
  int branches;              /* 1, or 2: out holds [uncond][cond] */
  const float* out;          /* the denoiser's prediction(s) [branches][n] */
  float guidance;
  float* sample;             /* [n], updated in place */
  float* last_denoised;      /* DPM++: [n] previous step's denoised, read if
                                second_order, always overwritten */
  const float* noise;        /* EULER_A / DPMPP_2M_SDE: [n] unit noise in the
                                generator's order */
  float* denoised_out;       /* optional [n]: PredictedSample (the preview) */
  float* next_input;         /* optional [n]: sample * next_input_scale, the
                                next denoiser call's input (ScaleModelInput) */
  float next_input_scale;
  float sigma, sigma_next;   /* Sigmas[step], Sigmas[step + 1] */
  /* EULER_A: up = sn * sqrt(max(s^2 - sn^2, 0)) / s, down = sqrt(max(sn^2 -
   * up^2, 0)) and Renoise(down, sn) -> (rescale, noise_scale), in double.
   * DPMPP: step_size = log(s / sn), shrink = sn / s, weight = step_size /
   * (2 * last_step_size) (2M) or 0.5 * (1 - shrink^2) * step_size /
   * last_step_size (SDE), rescale / noise_scale = Renoise(sn * shrink, sn). */
  double up, down, rescale, noise_scale, shrink, weight;
  int second_order;          /* DPMPP: use last_denoised this step */
} nd_sampler_args;

ND_API int nd_op_sampler_step(const nd_sampler_args* args, void* stream);

/* Synchronize `stream` and report any kernel's timed-out wait (ND_ERR_TIMEOUT)
 * or CUDA fault (ND_ERR_CUDA) since the last check on this device. */
ND_API int nd_op_sync(void* stream);

/* The device-timeout path on demand (DeviceRemovedException,
 * src/NaiveDiffusion/Dml/DeviceExceptions.cs:13-21, which the reference
 * raises after a dispatch's fence wait, Dml/DmlDevice.cs:920-948). Launches
 * `ctas` CTAs that wait on an mbarrier through the library's bounded wait,
 * giving up after `limit_ns` (1 ns .. 10 s). armed = 0: nothing arrives on
 * the barrier, the wait runs out, the kernel records a timeout in the
 * device's status word and returns; the next nd_op_sync on the device
 * reports ND_ERR_TIMEOUT and clears the word. armed = 1: the barrier is
 * arrived on first and the wait completes at once. Either way the CUDA
 * context stays usable. */
ND_API int nd_op_wait_probe(uint64_t limit_ns, int ctas, int armed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ND_DENOISE_H */
