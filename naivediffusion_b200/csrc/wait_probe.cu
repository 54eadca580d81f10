// The library's device-timeout path, run on purpose: a kernel waits on an
// mbarrier through the same bounded mbar_wait every pipelined kernel here
// uses, with a caller-chosen limit. Unarmed, nothing ever arrives on the
// barrier, so the wait runs out, records kStatusTimeoutProbe in the device
// status word and the kernel returns; nd_op_sync then reports ND_ERR_TIMEOUT
// and clears the word, and the context stays usable. Armed, one thread
// arrives first and the wait completes at once.
//
// This is the library's stand-in for the reference's device-removed report
// (DeviceRemovedException, src/NaiveDiffusion/Dml/DeviceExceptions.cs:13-21,
// raised after a dispatch's fence wait in Dml/DmlDevice.cs:920-948): a stuck
// pipeline ends in a status code the host reads, not a hung GPU.
#include "nd_common.cuh"
#include "nd_internal.h"

namespace nd {
unsigned* device_status();
}  // namespace nd

namespace {

__global__ void wait_probe_kernel(uint64_t limit_ns, int armed, unsigned* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const uint32_t b = nd::smem_u32(&bar);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    nd::mbar_init(b, 1);
    nd::fence_barrier_init();
  }
  __syncthreads();
  if (armed && threadIdx.x == 0) nd::mbar_arrive(b);
  // Every thread waits for phase 0; with no arrival it never completes.
  nd::mbar_wait(b, 0, &abort_flag, status, nd::kStatusTimeoutProbe, limit_ns);
}

}  // namespace

extern "C" int nd_op_wait_probe(uint64_t limit_ns, int ctas, int armed, void* stream) {
  // At most 10 s: long enough for any test, short enough that a caller's
  // mistake cannot hold the GPU.
  if (ctas <= 0 || ctas > 4096 || limit_ns == 0 || limit_ns > 10000000000ull)
    return nd::fail(ND_ERR_INVALID, "nd_op_wait_probe: ctas must be 1..4096 and the limit 1 ns..10 s");
  unsigned* st = nd::device_status();
  if (!st) return nd::fail(ND_ERR_CUDA, "nd_op_wait_probe: no device status word");
  wait_probe_kernel<<<ctas, 64, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, armed ? 1 : 0, st);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}
