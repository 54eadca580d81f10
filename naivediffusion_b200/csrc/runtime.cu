// Errors, per-device state, tensor-map encoding and the op-level C ABI.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {
thread_local std::string g_last_error;
std::mutex g_dev_mutex;
unsigned* g_status[64] = {};
int g_sms[64] = {};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}
}  // namespace

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  std::string msg = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return fail(e == cudaErrorMemoryAllocation ? ND_ERR_OOM : ND_ERR_CUDA, msg);
}

int check_register_split(const void* kernel, int threads, int needed, const char* what) {
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
  if (static_cast<long long>(fa.numRegs) * threads < needed)
    return fail(ND_ERR_UNSUPPORTED, std::string(what) + ": kernel compiled with " + std::to_string(fa.numRegs) +
                                        " registers per thread, fewer than its warpgroups' register split needs");
  return ND_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (!g_sms[dev & 63]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev & 63] = n > 0 ? n : 148;
  }
  return g_sms[dev & 63];
}

unsigned* device_status() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (!g_status[dev & 63]) {
    unsigned* p = nullptr;
    if (cudaMalloc(&p, 64) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, 64) != cudaSuccess) return nullptr;
    g_status[dev & 63] = p;
  }
  return g_status[dev & 63];
}

namespace {
void* g_op_scratch[64] = {};
size_t g_op_scratch_bytes[64] = {};
}  // namespace

int op_scratch(size_t need, void** ptr, size_t* bytes) {
  int dev = 0;
  ND_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (g_op_scratch_bytes[dev & 63] < need) {
    // Growing: wait for work that may still read the old buffer.
    ND_CUDA(cudaDeviceSynchronize());
    if (g_op_scratch[dev & 63]) cudaFree(g_op_scratch[dev & 63]);
    g_op_scratch[dev & 63] = nullptr;
    g_op_scratch_bytes[dev & 63] = 0;
    void* p = nullptr;
    ND_CUDA(cudaMalloc(&p, need));
    // zeroed: group_norm's arrival counters must start at zero
    if (cudaMemset(p, 0, need) != cudaSuccess) {
      cudaFree(p);
      return fail(ND_ERR_CUDA, "op scratch: memset failed");
    }
    g_op_scratch[dev & 63] = p;
    g_op_scratch_bytes[dev & 63] = need;
  }
  *ptr = g_op_scratch[dev & 63];
  *bytes = g_op_scratch_bytes[dev & 63];
  return ND_OK;
}

namespace {
thread_local bool t_pdl = false;
}  // namespace

bool pdl_enabled() { return t_pdl; }
PdlScope::PdlScope(bool on) : prev(t_pdl) { t_pdl = on; }
PdlScope::~PdlScope() { t_pdl = prev; }

int check_device_status(cudaStream_t stream) {
  ND_CUDA(cudaStreamSynchronize(stream));
  unsigned* st = device_status();
  if (!st) return fail(ND_ERR_CUDA, "no device status word");
  unsigned host = 0;
  ND_CUDA(cudaMemcpy(&host, st, sizeof(host), cudaMemcpyDeviceToHost));
  if (host != 0) {
    ND_CUDA(cudaMemset(st, 0, sizeof(unsigned)));
    char buf[128];
    snprintf(buf, sizeof(buf), "a kernel's bounded wait ran out (status 0x%x)", host);
    return fail(ND_ERR_TIMEOUT, buf);
  }
  return ND_OK;
}

int make_tmap_2d_typed(CUtensorMap* map, const void* base, int nd_dtype, int64_t rows, int64_t cols,
                       int64_t ld, int box_rows, int box_cols, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ND_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int elem_bytes = nd_dtype == ND_F32 || nd_dtype == ND_I32 ? 4 : nd_dtype == ND_I8 ? 1 : 2;
  if (reinterpret_cast<uintptr_t>(base) & 15u) return fail(ND_ERR_INVALID, "TMA base must be 16-byte aligned");
  if ((ld * elem_bytes) % 16 != 0) return fail(ND_ERR_INVALID, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMapDataType dt;
  switch (nd_dtype) {
    case ND_F32: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case ND_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case ND_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case ND_I32: dt = CU_TENSOR_MAP_DATA_TYPE_INT32; break;
    default: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
  }
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[192];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld ld=%lld box=%dx%d",
             static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(cols),
             static_cast<long long>(ld), box_rows, box_cols);
    return fail(ND_ERR_INVALID, buf);
  }
  return ND_OK;
}

int make_tmap_4d(CUtensorMap* map, const void* base, int nd_dtype, const int64_t dims[4],
                 const int64_t strides_bytes[3], const int box[4], const int elem_strides[4],
                 int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ND_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) & 15u) return fail(ND_ERR_INVALID, "TMA base must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (strides_bytes[i] % 16) return fail(ND_ERR_INVALID, "TMA strides must be multiples of 16 bytes");
  CUtensorMapDataType dt = nd_dtype == ND_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : nd_dtype == ND_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t d[4], st[3];
  cuuint32_t b[4], es[4];
  for (int i = 0; i < 4; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    b[i] = static_cast<cuuint32_t>(box[i]);
    es[i] = static_cast<cuuint32_t>(elem_strides[i]);
  }
  for (int i = 0; i < 3; ++i) st[i] = static_cast<cuuint64_t>(strides_bytes[i]);
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled (4-D) failed (%d)", static_cast<int>(r));
    return fail(ND_ERR_INVALID, buf);
  }
  return ND_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, int64_t rows, int64_t cols,
                 int64_t ld, int box_rows, int box_cols, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ND_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) & 15u) return fail(ND_ERR_INVALID, "TMA base must be 16-byte aligned");
  if ((ld * elem_bytes) % 16 != 0) return fail(ND_ERR_INVALID, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                           : elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32
                                             : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[192];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld ld=%lld box=%dx%d",
             static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(cols),
             static_cast<long long>(ld), box_rows, box_cols);
    return fail(ND_ERR_INVALID, buf);
  }
  return ND_OK;
}

}  // namespace nd

extern "C" {

const char* nd_last_error(void) { return nd::g_last_error.c_str(); }

const char* nd_version(void) { return "nd_denoise 0.1 (sm_100a)"; }

int nd_op_linear(const nd_linear_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_linear: null args");
  return nd::linear(*args, static_cast<cudaStream_t>(stream));
}

int nd_op_attention(const nd_attention_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_attention: null args");
  return nd::attention(*args, static_cast<cudaStream_t>(stream));
}

int64_t nd_attention_workspace_bytes(int head_dim) { return nd::attention_workspace_bytes(head_dim); }

int nd_op_modulate(const nd_modulate_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_modulate: null args");
  return nd::modulate(*args, static_cast<cudaStream_t>(stream));
}

int nd_op_rmsnorm(const nd_rmsnorm_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_rmsnorm: null args");
  return nd::rmsnorm(*args, static_cast<cudaStream_t>(stream));
}

int nd_op_gemv(const nd_gemv_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_gemv: null args");
  return nd::gemv(*args, static_cast<cudaStream_t>(stream));
}

int nd_op_patchify(const float* latent, void* tokens, int out_dtype, int batch, int channels,
                   int height, int width, int patch, int64_t ldt, void* stream) {
  return nd::patchify(latent, tokens, out_dtype, batch, channels, height, width, patch, ldt,
                      static_cast<cudaStream_t>(stream));
}

int nd_op_unpatchify(const float* tokens, int64_t ldt, float* latent, int batch, int channels,
                     int height, int width, int patch, void* stream) {
  return nd::unpatchify(tokens, ldt, latent, batch, channels, height, width, patch,
                        static_cast<cudaStream_t>(stream));
}

int nd_op_dequantize(const int8_t* q, const void* scales, int scale_dtype, int64_t quant_group,
                     int64_t rows, int64_t cols, void* out, int out_dtype, void* stream) {
  return nd::dequantize(q, scales, scale_dtype, quant_group, rows, cols, out, out_dtype,
                        static_cast<cudaStream_t>(stream));
}

int nd_op_quantize(const void* src, int src_dtype, int64_t rows, int64_t cols, int64_t quant_group,
                   int scale_dtype, int8_t* q, void* scales, void* stream) {
  if (src_dtype != ND_F32 && src_dtype != ND_F16 && src_dtype != ND_BF16)
    return nd::fail(ND_ERR_INVALID, "nd_op_quantize: src must be f32, f16 or bf16");
  if (scale_dtype != ND_F16 && scale_dtype != ND_F32)
    return nd::fail(ND_ERR_INVALID, "nd_op_quantize: scale_dtype must be ND_F16 or ND_F32");
  return nd::quantize_weights(src, src_dtype, rows, cols, quant_group, scale_dtype == ND_F16, q, scales,
                              static_cast<cudaStream_t>(stream));
}

int nd_op_conv2d(const nd_conv_args* args, void* stream) {
  if (!args) return nd::fail(ND_ERR_INVALID, "nd_op_conv2d: null args");
  return nd::conv2d(*args, static_cast<cudaStream_t>(stream));
}

int nd_op_group_norm(const void* x, void* y, int dtype, int batch, int pixels, int channels, int groups,
                     const float* weight, const float* bias, float eps, int silu_after, void* stream) {
  if (batch <= 0 || pixels <= 0 || channels <= 0 || groups <= 0)
    return nd::fail(ND_ERR_INVALID, "nd_op_group_norm: bad shape");
  void* scratch = nullptr;
  size_t bytes = 0;
  int rc = nd::op_scratch(nd::group_norm_scratch(batch, pixels, channels, groups), &scratch, &bytes);
  if (rc) return rc;
  return nd::group_norm(x, y, dtype, batch, pixels, channels, groups, weight, bias, eps, silu_after,
                        scratch, bytes, static_cast<cudaStream_t>(stream));
}

int nd_op_geglu(const void* in, void* out, int dtype, int64_t rows, int64_t F, void* stream) {
  if (!in || !out) return nd::fail(ND_ERR_INVALID, "nd_op_geglu: null operand");
  return nd::geglu(in, out, dtype, rows, F, static_cast<cudaStream_t>(stream));
}

int nd_op_sync(void* stream) { return nd::check_device_status(static_cast<cudaStream_t>(stream)); }

}  // extern "C"
