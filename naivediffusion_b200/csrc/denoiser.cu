// The denoiser plug-in C ABI: device handles, weight upload, finalize (warm-up
// run + CUDA-graph capture of the step), predict, memory figures.
//
// Replaces, from IDenoiser.Predict (Pipeline/IDenoiser.cs:10-32) down, the
// reference's ChainDenoiser / GraphChain.Run (Graph/ChainDenoiser.cs,
// Graph/GraphChain.cs:218-282): instead of ~200 synchronous DirectML
// submissions per step, one captured graph of kernel launches on one stream.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "denoiser.h"
#include "nd_common.cuh"
#include "nd_runtime.h"

namespace nd {

namespace {

__global__ void convert_kernel(const void* __restrict__ src, int st, void* __restrict__ dst, int dt,
                               long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v;
    if (st == ND_F32) v = static_cast<const float*>(src)[i];
    else if (st == ND_F16) v = __half2float(static_cast<const __half*>(src)[i]);
    else v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
    if (dt == ND_F32) static_cast<float*>(dst)[i] = v;
    else if (dt == ND_F16) static_cast<__half*>(dst)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
  }
}

__global__ void convert_cols_kernel(const void* __restrict__ src, int st, long long src_ld,
                                    void* __restrict__ dst, int dt, long long rows, long long cols) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols, c = i % cols, j = r * src_ld + c;
    float v;
    if (st == ND_F32) v = static_cast<const float*>(src)[j];
    else if (st == ND_F16) v = __half2float(static_cast<const __half*>(src)[j]);
    else v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[j]);
    if (dt == ND_BF16X2) {
      // row r of the hi|lo pair: hi at column c, lo at column cols + c
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(dst) + r * 2 * cols + c;
      o[0] = hi;
      o[cols] = __float2bfloat16_rn(v - __bfloat162float(hi));
    } else if (dt == ND_F32) static_cast<float*>(dst)[i] = v;
    else if (dt == ND_F16) static_cast<__half*>(dst)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
  }
}

__global__ void permute_conv_kernel(const void* __restrict__ src, int st, void* __restrict__ dst, int dt,
                                    long long cout, int cin, int cin_pad) {
  const long long n = cout * 9 * cin_pad;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cin_pad);
    const int tap = static_cast<int>((i / cin_pad) % 9);
    const long long o = i / (9LL * cin_pad);
    float v = 0.f;
    if (c < cin) {
      const long long j = (o * cin + c) * 9 + tap;
      if (st == ND_F32) v = static_cast<const float*>(src)[j];
      else if (st == ND_F16) v = __half2float(static_cast<const __half*>(src)[j]);
      else v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[j]);
    }
    if (dt == ND_F16) static_cast<__half*>(dst)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
  }
}

int elem_bytes(int dt) { return dt == ND_F32 || dt == ND_I32 ? 4 : dt == ND_I8 ? 1 : 2; }

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int ordinal) {
    cudaGetDevice(&prev);
    cudaSetDevice(ordinal);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

int convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, cudaStream_t s) {
  if (n <= 0) return ND_OK;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, sm_count() * 8LL));
  convert_kernel<<<grid, 256, 0, s>>>(src, src_dtype, dst, dst_dtype, n);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

// dst row r = src row of the same head at feature 2f (f < half) or
// 2(f - half) + 1 (QwenImageDit.PairsToHalves, Models/QwenImage/QwenImageDit.cs:261-279).
__global__ void permute_head_rows_kernel(const void* __restrict__ src, void* __restrict__ dst, int64_t rows,
                                         int64_t cols, int elem_bytes, int head) {
  const int64_t n = rows * cols;
  const int half = head / 2;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int64_t base = r - r % head;
    const int f = static_cast<int>(r - base);
    const int64_t from = base + (f < half ? 2 * f : 2 * (f - half) + 1);
    if (elem_bytes == 2)
      static_cast<uint16_t*>(dst)[i] = static_cast<const uint16_t*>(src)[from * cols + c];
    else
      static_cast<uint32_t*>(dst)[i] = static_cast<const uint32_t*>(src)[from * cols + c];
  }
}

int permute_conv3x3(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t cout, int cin,
                    int cin_pad, cudaStream_t s) {
  const int64_t n = cout * 9 * cin_pad;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, sm_count() * 8LL));
  permute_conv_kernel<<<grid, 256, 0, s>>>(src, src_dtype, dst, dst_dtype, cout, cin, cin_pad);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int permute_head_rows(const void* src, void* dst, int64_t rows, int64_t cols, int elem_bytes, int head,
                      cudaStream_t s) {
  const int64_t n = rows * cols;
  if (n <= 0) return ND_OK;
  if (elem_bytes != 2 && elem_bytes != 4) return fail(ND_ERR_INVALID, "permute_head_rows: element size");
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, sm_count() * 8LL));
  permute_head_rows_kernel<<<grid, 256, 0, s>>>(src, dst, rows, cols, elem_bytes, head);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int convert_cols(const void* src, int src_dtype, int64_t src_ld, void* dst, int dst_dtype, int64_t rows,
                 int64_t cols, cudaStream_t s) {
  const int64_t n = rows * cols;
  if (n <= 0) return ND_OK;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, sm_count() * 8LL));
  convert_cols_kernel<<<grid, 256, 0, s>>>(src, src_dtype, src_ld, dst, dst_dtype, rows, cols);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

}  // namespace nd

void nd_denoiser::prof_begin(cudaStream_t s) {
  if (!profiling || prof_used + 2 > prof_pool.size()) return;
  prof_start_ev = prof_pool[prof_used++];
  cudaEventRecord(prof_start_ev, s);
}

void nd_denoiser::prof_end(cudaStream_t s, const char* cls, double flops, double bytes) {
  if (!profiling || !prof_start_ev) return;
  cudaEvent_t stop = prof_pool[prof_used++];
  cudaEventRecord(stop, s);
  prof.push_back(ProfRecord{cls, flops, bytes, prof_start_ev, stop});
  prof_start_ev = nullptr;
}

nd_denoiser::~nd_denoiser() {
  for (cudaEvent_t e : prof_pool) cudaEventDestroy(e);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  for (void* p : allocations) cudaFree(p);
  for (void* p : host_allocations) cudaFreeHost(p);
  if (staged) cudaEventDestroy(staged);
  if (staging) cudaFree(staging);
  if (staging2) cudaFree(staging2);
}

void* nd_denoiser::pinned(size_t bytes) {
  void* p = nullptr;
  if (cudaMallocHost(&p, bytes) != cudaSuccess) {
    alloc_failed = true;
    return nullptr;
  }
  host_allocations.push_back(p);
  return p;
}

void* nd_denoiser::alloc(size_t bytes, bool weight) {
  void* p = nullptr;
  bytes = (bytes + 255) & ~static_cast<size_t>(255);
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    alloc_failed = true;
    return nullptr;
  }
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    alloc_failed = true;
    return nullptr;
  }
  allocations.push_back(p);
  (weight ? weight_bytes : work_bytes) += bytes;
  return p;
}

nd::Mat nd_denoiser::alloc_mat(int64_t rows, int64_t cols, int64_t per_rows) {
  nd::Mat m;
  m.cols = cols;
  m.q8 = quantizes(per_rows, cols);
  if (m.q8) {
    m.w = alloc(static_cast<size_t>(rows * cols), true);
    const int64_t sc = cols / qgroup(cols);
    m.scales = alloc(static_cast<size_t>(rows * sc) * (qf16() ? 2 : 4), true);
  } else {
    m.split = mat_dtype() == ND_BF16X2;
    m.w = alloc(static_cast<size_t>(rows * cols) * (m.split ? 4 : 2), true);
  }
  return m;
}

void nd_denoiser::add_slot(const std::string& name, int kind, int64_t rows, int64_t cols, void* dst,
                           bool required, void* scales) {
  nd::WeightSlot s;
  s.name = name;
  s.kind = kind;
  s.rows = rows;
  s.cols = cols;
  s.dst = dst;
  s.scales = scales;
  s.required = required;
  index[name] = slots.size();
  slots.push_back(s);
}

namespace {

// Grow a device buffer (kept between calls) to at least `bytes`.
int grow(void** buf, size_t* have, size_t bytes) {
  if (*have >= bytes) return ND_OK;
  if (*buf) cudaFree(*buf);
  *buf = nullptr;
  *have = 0;
  ND_CUDA(cudaMalloc(buf, bytes));
  *have = bytes;
  return ND_OK;
}

// Copy a host tensor into the denoiser's device staging buffer.
int upload_staging(nd_denoiser* d, const void* data, size_t bytes, cudaStream_t st, const void** src) {
  ND_TRY_RC(grow(&d->staging, &d->staging_bytes, bytes));
  ND_CUDA(cudaMemcpyAsync(d->staging, data, bytes, cudaMemcpyHostToDevice, st));
  *src = d->staging;
  return ND_OK;
}

int set_weight_impl(nd_denoiser* d, const char* name, int dtype, const int64_t* shape, int rank,
                    const void* data, bool device) {
  using namespace nd;
  if (!d || !name || !data) return fail(ND_ERR_INVALID, "set_weight: null argument");
  if (d->finalized) return fail(ND_ERR_STATE, "set_weight: denoiser already finalized");
  auto it = d->index.find(name);
  if (it == d->index.end()) return fail(ND_ERR_INVALID, std::string("set_weight: unknown tensor ") + name);
  WeightSlot& s = d->slots[it->second];
  if (dtype != ND_F32 && dtype != ND_F16 && dtype != ND_BF16)
    return fail(ND_ERR_INVALID, std::string("set_weight: ") + name + " must be f32, f16 or bf16");
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) n *= shape[i];
  const bool sliced = s.src_cols > s.cols && rank == 2 && shape[0] == s.rows && shape[1] == s.src_cols;
  const bool pointwise = s.kind == kMatrix && rank == 4 && shape[0] == s.rows && shape[1] == s.cols &&
                         shape[2] == 1 && shape[3] == 1;  // a 1x1 convolution's [out, in, 1, 1]
  const bool shape_ok = s.kind == kConv3x3 || sliced || pointwise ||
                        (rank == 2 && shape[0] == s.rows && shape[1] == s.cols) ||
                        (rank == 1 && s.cols == 1 && shape[0] == s.rows) ||
                        (n == s.rows * s.cols && s.kind == kVector);
  if (!shape_ok) {
    return fail(ND_ERR_INVALID, std::string("set_weight: ") + name + " has the wrong shape (expected [" +
                                    std::to_string(s.rows) + ", " + std::to_string(s.src_cols > s.cols ? s.src_cols : s.cols) + "])");
  }
  if (s.head_perm > 0) {
    // Reorder the rows within each head (pairs -> halves) into a second
    // device buffer, then store that copy the usual way.
    const int64_t rows = rank >= 1 ? shape[0] : 1;
    const int64_t cols = rows > 0 ? n / rows : 0;
    if (rows % s.head_perm != 0 || s.head_perm % 2 != 0)
      return fail(ND_ERR_INVALID, std::string("set_weight: ") + name + " rows do not divide into heads");
    DeviceGuard g(d->dev->ordinal);
    cudaStream_t st = d->dev->stream;
    const size_t src_bytes = static_cast<size_t>(n) * elem_bytes(dtype);
    const void* src = data;
    if (!device) ND_TRY_RC(upload_staging(d, data, src_bytes, st, &src));
    ND_TRY_RC(grow(&d->staging2, &d->staging2_bytes, src_bytes));
    ND_TRY_RC(permute_head_rows(src, d->staging2, rows, cols, static_cast<int>(elem_bytes(dtype)), s.head_perm, st));
    const int head = s.head_perm;
    s.head_perm = 0;
    const int rc = set_weight_impl(d, name, dtype, shape, rank, d->staging2, true);
    s.head_perm = head;
    return rc;
  }
  if (s.kind == kConv3x3) {
    if (!(rank == 4 && shape[0] == s.rows && shape[1] == s.conv_cin && shape[2] == 3 && shape[3] == 3))
      return fail(ND_ERR_INVALID, std::string("set_weight: ") + name + " must be [" + std::to_string(s.rows) +
                                      ", " + std::to_string(s.conv_cin) + ", 3, 3]");
    DeviceGuard g(d->dev->ordinal);
    cudaStream_t st = d->dev->stream;
    const size_t src_bytes = static_cast<size_t>(n) * elem_bytes(dtype);
    const void* src = data;
    if (!device) ND_TRY_RC(upload_staging(d, data, src_bytes, st, &src));
    int rc = permute_conv3x3(src, dtype, s.dst, d->desc.compute, s.rows, s.conv_cin,
                             static_cast<int>(s.cols / 9), st);
    if (rc) return rc;
    ND_CUDA(cudaStreamSynchronize(st));
    s.set = true;
    return ND_OK;
  }
  if (sliced) {
    // Keep the first `cols` columns of the checkpoint's wider matrix.
    DeviceGuard g(d->dev->ordinal);
    cudaStream_t st = d->dev->stream;
    const size_t src_bytes = static_cast<size_t>(n) * elem_bytes(dtype);
    const void* src = data;
    if (!device) ND_TRY_RC(upload_staging(d, data, src_bytes, st, &src));
    int rc = convert_cols(src, dtype, s.src_cols, s.dst, d->mat_dtype(), s.rows, s.cols, st);
    if (rc) return rc;
    ND_CUDA(cudaStreamSynchronize(st));
    s.set = true;
    return ND_OK;
  }
  DeviceGuard g(d->dev->ordinal);
  cudaStream_t st = d->dev->stream;
  const int dst_type = s.kind == kMatrix ? d->mat_dtype() : ND_F32;
  const size_t src_bytes = static_cast<size_t>(n) * elem_bytes(dtype);
  if (s.scales) {
    // int8 storage: quantize on the device (BlockQuantizer's rules).
    const void* src = data;
    if (!device) ND_TRY_RC(upload_staging(d, data, src_bytes, st, &src));
    int rc = quantize_weights(src, dtype, s.rows, s.cols, d->qgroup(s.cols), d->qf16() ? 1 : 0,
                              static_cast<int8_t*>(s.dst), s.scales, st);
    if (rc) return rc;
    ND_CUDA(cudaStreamSynchronize(st));
    s.set = true;
    return ND_OK;
  }
  if (dtype == dst_type) {
    ND_CUDA(cudaMemcpyAsync(s.dst, data, src_bytes, device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
  } else {
    const void* src = data;
    if (!device) ND_TRY_RC(upload_staging(d, data, src_bytes, st, &src));
    int rc = dst_type == ND_BF16X2 ? convert_cols(src, dtype, s.cols, s.dst, dst_type, s.rows, s.cols, st)
                                   : convert(src, dtype, s.dst, dst_type, n, st);
    if (rc) return rc;
  }
  ND_CUDA(cudaStreamSynchronize(st));
  s.set = true;
  return ND_OK;
}

int run_predict(nd_denoiser* d, const float* latent, double timestep, double sigma, int n_cond,
                const nd_named_tensor* cond, float* out, bool device, cudaStream_t stream) {
  using namespace nd;
  if (!d || !latent || !out) return fail(ND_ERR_INVALID, "predict: null argument");
  if (!d->finalized) return fail(ND_ERR_STATE, "predict: call nd_denoiser_finalize first");
  if (n_cond < 0 || (n_cond > 0 && !cond)) return fail(ND_ERR_INVALID, "predict: bad conditioning list");
  DeviceGuard g(d->dev->ordinal);
  StepInputs in;
  in.latent = latent;
  in.device = device;
  in.timestep = timestep;
  in.sigma = sigma;
  int rc = d->check_cond(n_cond, cond, in);
  if (rc) return rc;
  cudaStream_t st = stream ? stream : d->dev->stream;
  rc = d->stage(in, st);
  if (rc) return rc;
  // The captured step is specialised on the visible-key count (a kernel
  // argument): recapture when it changes.
  if (!d->exec || d->graph_key != in.key_limit) {
    if (d->exec) {
      cudaGraphExecDestroy(d->exec);
      d->exec = nullptr;
    }
    if (d->graph) {
      cudaGraphDestroy(d->graph);
      d->graph = nullptr;
    }
    ND_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    rc = d->forward(st);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "predict: graph capture");
    d->graph = graph;
    ND_CUDA(cudaGraphInstantiate(&d->exec, d->graph, 0));
    d->graph_key = in.key_limit;
  }
  ND_CUDA(cudaGraphLaunch(d->exec, st));
  const size_t out_bytes = static_cast<size_t>(d->output_elems()) * sizeof(float);
  ND_CUDA(cudaMemcpyAsync(out, d->output(), out_bytes, device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
  if (!device) return check_device_status(st);
  return ND_OK;
}

}  // namespace

extern "C" {

int nd_device_open(int ordinal, nd_device** out) {
  if (!out) return nd::fail(ND_ERR_INVALID, "nd_device_open: null out");
  *out = nullptr;
  int count = 0;
  ND_CUDA(cudaGetDeviceCount(&count));
  if (ordinal < 0 || ordinal >= count) return nd::fail(ND_ERR_INVALID, "nd_device_open: no such device");
  nd::DeviceGuard g(ordinal);
  cudaDeviceProp prop;
  ND_CUDA(cudaGetDeviceProperties(&prop, ordinal));
  if (prop.major != 10) return nd::fail(ND_ERR_UNSUPPORTED, "nd_device_open: this library runs on sm_100 (B200) only");
  auto* d = new nd_device();
  d->ordinal = ordinal;
  cudaError_t e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete d;
    return nd::cuda_fail(e, "nd_device_open: stream");
  }
  if (!nd::device_status()) {
    cudaStreamDestroy(d->stream);
    delete d;
    return nd::fail(ND_ERR_OOM, "nd_device_open: status word");
  }
  *out = d;
  return ND_OK;
}

int nd_device_close(nd_device* dev) {
  if (!dev) return ND_OK;
  nd::DeviceGuard g(dev->ordinal);
  cudaStreamSynchronize(dev->stream);
  cudaStreamDestroy(dev->stream);
  delete dev;
  return ND_OK;
}

int nd_denoiser_create(nd_device* dev, const nd_model_desc* desc, nd_denoiser** out) {
  if (!dev || !desc || !out) return nd::fail(ND_ERR_INVALID, "nd_denoiser_create: null argument");
  *out = nullptr;
  nd::DeviceGuard g(dev->ordinal);
  nd_denoiser* d = nullptr;
  switch (desc->family) {
    case ND_FAMILY_MMDIT: d = nd::make_mmdit(); break;
    case ND_FAMILY_ANIMA: d = nd::make_anima(); break;
    case ND_FAMILY_SDXL: d = nd::make_unet(); break;
    case ND_FAMILY_VAE_KL: d = nd::make_vae_decoder(); break;
    case ND_FAMILY_QWEN_IMAGE: d = nd::make_qwen_image(); break;
    case ND_FAMILY_VAE_WAN21:
    case ND_FAMILY_VAE_WAN22: d = nd::make_wan_decoder(); break;
    case ND_FAMILY_QWEN3_TEXT: d = nd::make_qwen3_text(); break;
    case ND_FAMILY_LLM_ADAPTER: d = nd::make_llm_adapter(); break;
    default: return nd::fail(ND_ERR_UNSUPPORTED, "nd_denoiser_create: unknown model family");
  }
  d->dev = dev;
  d->desc = *desc;
  int rc = d->build();
  if (rc) {
    delete d;  // a failed build releases everything (ChainDenoiser.Build)
    return rc;
  }
  *out = d;
  return ND_OK;
}

int nd_denoiser_weight_info(const nd_denoiser* d, int index, const char** name, int64_t* rows,
                            int64_t* cols, int* required) {
  if (!d) return nd::fail(ND_ERR_INVALID, "weight_info: null denoiser");
  if (index < 0 || index >= static_cast<int>(d->slots.size())) return ND_ERR_INVALID;
  const nd::WeightSlot& s = d->slots[index];
  if (name) *name = s.name.c_str();
  if (rows) *rows = s.rows;
  if (cols) *cols = s.cols;
  if (required) *required = s.required ? 1 : 0;
  return ND_OK;
}

int nd_denoiser_set_weight(nd_denoiser* d, const char* name, int dtype, const int64_t* shape, int rank,
                           const void* data) {
  return set_weight_impl(d, name, dtype, shape, rank, data, false);
}

int nd_denoiser_set_weight_device(nd_denoiser* d, const char* name, int dtype, const int64_t* shape,
                                  int rank, const void* data) {
  return set_weight_impl(d, name, dtype, shape, rank, data, true);
}

int nd_denoiser_set_weight_q8(nd_denoiser* d, const char* name, const int64_t* shape, int rank,
                              const int8_t* q, int scale_dtype, const void* scales, int64_t quant_group) {
  using namespace nd;
  if (!d || !name || !shape || !q || !scales) return fail(ND_ERR_INVALID, "set_weight_q8: null argument");
  if (d->finalized) return fail(ND_ERR_STATE, "set_weight_q8: denoiser already finalized");
  auto it = d->index.find(name);
  if (it == d->index.end()) return fail(ND_ERR_INVALID, std::string("set_weight_q8: unknown tensor ") + name);
  WeightSlot& s = d->slots[it->second];
  if (!s.scales) return fail(ND_ERR_INVALID, std::string("set_weight_q8: ") + name + " is not stored as int8");
  if (rank != 2 || shape[0] != s.rows || shape[1] != s.cols)
    return fail(ND_ERR_INVALID, std::string("set_weight_q8: ") + name + " has the wrong shape");
  if ((scale_dtype == ND_F16) != d->qf16() || (quant_group > 0 ? quant_group : s.cols) != d->qgroup(s.cols))
    return fail(ND_ERR_INVALID, "set_weight_q8: scale type / group differ from the model's");
  DeviceGuard g(d->dev->ordinal);
  cudaStream_t st = d->dev->stream;
  const int64_t sc = s.cols / d->qgroup(s.cols);
  ND_CUDA(cudaMemcpyAsync(s.dst, q, static_cast<size_t>(s.rows * s.cols), cudaMemcpyHostToDevice, st));
  ND_CUDA(cudaMemcpyAsync(s.scales, scales, static_cast<size_t>(s.rows * sc) * (d->qf16() ? 2 : 4),
                          cudaMemcpyHostToDevice, st));
  ND_CUDA(cudaStreamSynchronize(st));
  s.set = true;
  return ND_OK;
}

int nd_denoiser_finalize(nd_denoiser* d) {
  if (!d) return nd::fail(ND_ERR_INVALID, "finalize: null denoiser");
  if (d->finalized) return ND_OK;
  for (const nd::WeightSlot& s : d->slots) {
    if (s.required && !s.set) return nd::fail(ND_ERR_MISSING_WEIGHT, "finalize: weight not set: " + s.name);
  }
  nd::DeviceGuard g(d->dev->ordinal);
  if (d->staging) {
    cudaFree(d->staging);
    d->staging = nullptr;
    d->staging_bytes = 0;
  }
  if (d->staging2) {
    cudaFree(d->staging2);
    d->staging2 = nullptr;
    d->staging2_bytes = 0;
  }
  int rc = d->prepare();
  if (rc) return rc;
  // One eager run outside capture: first-use setup (kernel attributes,
  // status word) happens here, and a broken configuration fails loudly now.
  rc = d->forward(d->dev->stream);
  if (rc) return rc;
  rc = nd::check_device_status(d->dev->stream);
  if (rc) return rc;
  d->finalized = true;
  return ND_OK;
}

int nd_denoiser::encode(const int32_t*, int, const float*, int, int, float*) {
  return nd::fail(ND_ERR_INVALID, "text_encode: this family is not a text tower");
}

int nd_text_encode(nd_denoiser* d, const int32_t* ids, int rows, const float* source, int source_rows,
                   int final_norm, float* out) {
  if (!d || !ids || !out) return nd::fail(ND_ERR_INVALID, "text_encode: null argument");
  if (!d->finalized) return nd::fail(ND_ERR_STATE, "text_encode: call nd_denoiser_finalize first");
  nd::DeviceGuard g(d->dev->ordinal);
  return d->encode(ids, rows, source, source_rows, final_norm, out);
}

int nd_denoiser_predict(nd_denoiser* d, const float* latent, double timestep, double sigma, int n_cond,
                        const nd_named_tensor* cond, float* out) {
  return run_predict(d, latent, timestep, sigma, n_cond, cond, out, false, nullptr);
}

int nd_denoiser_predict_device(nd_denoiser* d, const float* latent, double timestep, double sigma,
                               int n_cond, const nd_named_tensor* cond, float* out, void* stream) {
  return run_predict(d, latent, timestep, sigma, n_cond, cond, out, true, static_cast<cudaStream_t>(stream));
}

int nd_denoiser_profile(nd_denoiser* d, int steps, nd_kernel_time* out, int max_entries,
                        int* n_entries) {
  if (!d || !out || !n_entries || steps <= 0 || max_entries <= 0)
    return nd::fail(ND_ERR_INVALID, "profile: bad argument");
  if (!d->finalized) return nd::fail(ND_ERR_STATE, "profile: call nd_denoiser_finalize first");
  nd::DeviceGuard g(d->dev->ordinal);
  cudaStream_t st = d->dev->stream;
  // Run the step eagerly with an event pair recorded around every launch and
  // read the events. The host enqueues a step in a few milliseconds while the
  // GPU needs far longer, so after the first launches the queue runs ahead
  // and each pair brackets its kernel alone. (Event-record nodes inside a
  // captured graph were measured to add tens of microseconds per launch.)
  // Events are created once, two per launch.
  while (d->prof_pool.size() < 8192) {
    cudaEvent_t ev;
    ND_CUDA(cudaEventCreate(&ev));
    d->prof_pool.push_back(ev);
  }
  std::vector<double> ms;
  std::vector<nd_denoiser::ProfRecord> first;
  int rc = ND_OK;
  for (int i = 0; i < steps && rc == ND_OK; ++i) {
    d->prof.clear();
    d->prof_used = 0;
    d->profiling = true;
    rc = d->forward(st);
    d->profiling = false;
    if (rc) break;
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      rc = nd::cuda_fail(e, "profile: step");
      break;
    }
    if (i == 0) {
      first = d->prof;
      ms.assign(first.size(), 0.0);
    } else if (d->prof.size() != first.size()) {
      rc = nd::fail(ND_ERR_STATE, "profile: the step's launch list changed between runs");
      break;
    }
    for (size_t k = 0; k < d->prof.size() && rc == ND_OK; ++k) {
      float t = 0.f;
      e = cudaEventElapsedTime(&t, d->prof[k].start, d->prof[k].stop);
      if (e != cudaSuccess) {
        cudaGetLastError();  // not sticky: keep it from surfacing in a later call
        rc = nd::cuda_fail(e, (std::string("profile: event time of ") + d->prof[k].cls + " launch " +
                               std::to_string(k)).c_str());
        break;
      }
      ms[k] += t;
    }
  }
  if (rc) return rc;
  rc = nd::check_device_status(st);
  if (rc) return rc;
  int n = 0;
  for (size_t k = 0; k < first.size(); ++k) {
    const auto& r = first[k];
    int j = 0;
    while (j < n && std::strcmp(out[j].name, r.cls) != 0) ++j;
    if (j == n) {
      if (n == max_entries) continue;
      out[j] = nd_kernel_time{r.cls, 0, 0.0, 0.0, 0.0};
      ++n;
    }
    out[j].launches += 1;
    out[j].total_ms += ms[k] / steps;
    out[j].flops += r.flops;
    out[j].bytes += r.bytes;
  }
  *n_entries = n;
  return ND_OK;
}

int nd_denoiser_memory(const nd_denoiser* d, nd_memory* out) {
  if (!d || !out) return nd::fail(ND_ERR_INVALID, "memory: null argument");
  out->persistent_bytes = d->weight_bytes;
  out->streamed_bytes = 0;
  out->resident_bytes = d->weight_bytes;
  out->temporary_bytes = d->work_bytes;
  out->graph_count = d->exec ? 1 : 0;
  return ND_OK;
}

int nd_denoiser_destroy(nd_denoiser* d) {
  if (!d) return ND_OK;
  nd::DeviceGuard g(d->dev->ordinal);
  cudaStreamSynchronize(d->dev->stream);
  delete d;
  return ND_OK;
}

}  // extern "C"
