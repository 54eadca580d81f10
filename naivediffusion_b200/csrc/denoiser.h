// The denoiser plug-in's C++ side: device handles, the weight registry and
// the per-family forward step. The C ABI in include/nd_denoise.h wraps it.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "nd_internal.h"

struct nd_device {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
};

#define ND_TRY_RC(expr)     \
  do {                      \
    int rc_ = (expr);       \
    if (rc_) return rc_;    \
  } while (0)

namespace nd {

enum SlotKind { kMatrix = 0, kVector = 1, kConv3x3 = 2 };

struct WeightSlot {
  std::string name;
  int kind = kMatrix;
  int64_t rows = 0, cols = 1;
  void* dst = nullptr;     // device destination (compute dtype / int8 for matrices, fp32 vectors)
  void* scales = nullptr;  // int8 matrices: their scales (quant_group / scale type of the model)
  int64_t src_cols = 0;    // > cols: the checkpoint tensor is wider; keep its first `cols` columns
  int conv_cin = 0;        // kConv3x3: torch [rows, conv_cin, 3, 3] stored as [rows, 3, 3, cols / 9]
  // > 0: rows are features of heads this wide, reordered on upload from
  // adjacent pairs (2i, 2i+1) to halves (i, half + i), so the rotate-half
  // RoPE turns the pairs the checkpoint's model turns.
  int head_perm = 0;
  bool required = true;
  bool set = false;
};

// A matrix kind stored for the GEMM / GEMV: compute dtype, or int8 + scales.
struct Mat {
  void* w = nullptr;
  void* scales = nullptr;
  bool q8 = false;
  bool split = false;  // fp32 compute: rows are bf16 hi|lo pairs, 4 bytes per weight
  int64_t cols = 0;
  // element offset of sub-matrix row `row` in w, and of its scales
  void* at(int64_t row, int elem_bytes) const {
    return static_cast<uint8_t*>(w) + row * cols * (q8 ? 1 : split ? 4 : elem_bytes);
  }
  void* scales_at(int64_t row, int64_t scale_cols, bool f16) const {
    return scales ? static_cast<uint8_t*>(scales) + row * scale_cols * (f16 ? 2 : 4) : nullptr;
  }
};

// Host-side values of one predict call, already validated.
struct StepInputs {
  const float* latent = nullptr;   // [batch, C, H, W]
  const float* context = nullptr;  // [batch, rows, width]
  const float* cos = nullptr;      // optional
  const float* sin = nullptr;
  int key_limit = 0;               // 0: all keys
  bool device = false;             // pointers are device memory
  double timestep = 0, sigma = 0;
};

// Converts `n` elements of `src` (dtype) into `dst` (dst_dtype) on the device.
int convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, cudaStream_t s);
// torch conv weights [cout, cin, 3, 3] -> [cout, 3, 3, cin_pad] (zero padded).
int permute_conv3x3(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t cout, int cin,
                    int cin_pad, cudaStream_t s);
// Rows of a row-major [rows, cols] src (elem_bytes each) reordered within
// every `head` rows from pairs to halves (QwenImageDit.PairsToHalves).
int permute_head_rows(const void* src, void* dst, int64_t rows, int64_t cols, int elem_bytes, int head,
                      cudaStream_t s);
// Rows x cols of a row-major src (leading dimension src_ld) into a packed dst.
int convert_cols(const void* src, int src_dtype, int64_t src_ld, void* dst, int dst_dtype, int64_t rows,
                 int64_t cols, cudaStream_t s);

}  // namespace nd

struct nd_denoiser {
  nd_device* dev = nullptr;
  nd_model_desc desc{};
  std::vector<nd::WeightSlot> slots;
  std::unordered_map<std::string, size_t> index;
  std::vector<void*> allocations;
  std::vector<void*> host_allocations;
  cudaEvent_t staged = nullptr;  // recorded after the last host->device copy of pinned inputs
  bool alloc_failed = false;
  uint64_t weight_bytes = 0, work_bytes = 0;
  bool finalized = false;
  void* staging = nullptr;
  size_t staging_bytes = 0;
  void* staging2 = nullptr;  // the permuted copy of a head_perm slot's tensor
  size_t staging2_bytes = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int graph_key = -1;  // key_limit the captured graph was built for

  // Per-kernel-class CUDA-event timing of eager forward runs (nd_denoiser_profile).
  struct ProfRecord {
    const char* cls;
    double flops, bytes;
    cudaEvent_t start, stop;
  };
  bool profiling = false;
  std::vector<ProfRecord> prof;
  std::vector<cudaEvent_t> prof_pool;
  size_t prof_used = 0;
  cudaEvent_t prof_start_ev = nullptr;
  void prof_begin(cudaStream_t s);
  void prof_end(cudaStream_t s, const char* cls, double flops, double bytes);

  virtual ~nd_denoiser();
  // Allocate (zeroed) device memory tracked for destroy(); weights count
  // toward weight_bytes, everything else toward work_bytes.
  void* alloc(size_t bytes, bool weight);
  // Pinned host memory, freed with the denoiser (nullptr + alloc_failed on failure).
  void* pinned(size_t bytes);
  // The attention workspace (zeroed by alloc; the kernel keeps it zeroed),
  // shared by this denoiser's attention launches, which its one stream orders.
  void* attn_ws = nullptr;
  int64_t attn_ws_bytes = 0;
  void alloc_attn_workspace(int head_dim) {
    attn_ws_bytes = nd::attention_workspace_bytes(head_dim);
    attn_ws = attn_ws_bytes > 0 ? alloc(static_cast<size_t>(attn_ws_bytes), false) : nullptr;
  }
  void use_attn_workspace(nd_attention_args& a) const {
    a.workspace = attn_ws;
    a.workspace_bytes = attn_ws ? attn_ws_bytes : 0;
  }
  void add_slot(const std::string& name, int kind, int64_t rows, int64_t cols, void* dst,
                bool required = true, void* scales = nullptr);
  // int8 storage of matrices (desc.weight_dtype == ND_I8): columns per scale
  // (0 = per output channel) and whether scales are fp16.
  bool q8() const { return desc.weight_dtype == ND_I8; }
  // Storage of the matrices the GEMMs read: the compute dtype, or bf16 hi|lo
  // pairs when the model computes in fp32.
  int mat_dtype() const { return desc.compute == ND_F32 ? ND_BF16X2 : desc.compute; }
  int64_t qgroup(int64_t cols) const { return desc.quant_group > 0 ? desc.quant_group : cols; }
  bool qf16() const { return desc.quant_scale_dtype == ND_F16; }
  // Whether a [rows, cols] matrix is stored as int8: the reference's rule
  // (ModelBuilder.Weight: at least 65,536 elements, whole blocks per row).
  bool quantizes(int64_t rows, int64_t cols) const {
    return q8() && rows * cols >= 65536 && cols % qgroup(cols) == 0 && cols % 16 == 0;
  }
  // Allocate a matrix kind of `rows` x `cols` (sub-matrices of `per_rows`
  // rows each stacked; the int8 rule applies per sub-matrix).
  nd::Mat alloc_mat(int64_t rows, int64_t cols, int64_t per_rows);

  virtual int build() = 0;          // allocate weights + scratch, register slots
  virtual int prepare() { return ND_OK; }  // after every weight is set
  // Copy this call's inputs into the model's fixed input buffers.
  virtual int stage(const nd::StepInputs& in, cudaStream_t s) = 0;
  // Enqueue the whole forward step on `s` (capturable: no sync, no alloc).
  virtual int forward(cudaStream_t s) = 0;
  virtual const float* output() const = 0;
  virtual int64_t latent_elems() const = 0;
  // Floats predict() returns (the latent's shape for denoisers; an image for
  // the VAE decoder).
  virtual int64_t output_elems() const { return latent_elems(); }
  virtual int check_cond(int n, const nd_named_tensor* cond, nd::StepInputs& in) = 0;
  // Text towers (nd_text_encode): one call over `rows` token ids.
  virtual int encode(const int32_t* ids, int rows, const float* source, int source_rows, int final_norm,
                     float* out);
};

namespace nd {
nd_denoiser* make_mmdit();
nd_denoiser* make_anima();
nd_denoiser* make_unet();
nd_denoiser* make_vae_decoder();
nd_denoiser* make_qwen_image();
nd_denoiser* make_wan_decoder();
nd_denoiser* make_qwen3_text();
nd_denoiser* make_llm_adapter();
int head_norm_rope(void* x, int dtype, int64_t ld, int64_t rows, int heads, int head_dim, const float* weight,
                   const float* cos, const float* sin, float eps, cudaStream_t s);
}  // namespace nd
