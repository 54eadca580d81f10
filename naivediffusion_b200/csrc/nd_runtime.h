// Per-device runtime state of libnd_denoise (status word, SM count).
#pragma once

#include <cuda_runtime.h>

namespace nd {

// The current device's status word: kernels write a nonzero code into it
// when a bounded wait runs out. Allocated on first use per device.
unsigned* device_status();

// Library-owned device scratch of at least `need` bytes for op-level entry
// points (grown with cudaMalloc when needed; reused by every call).
int op_scratch(size_t need, void** ptr, size_t* bytes);

// Read and clear the current device's status word (synchronizes `stream`).
int check_device_status(cudaStream_t stream);

// Whether launch_pdl() launches on this thread carry the programmatic
// stream serialization attribute. On for the SDXL UNet's step (over a
// thousand short launches: 2.4 % faster measured), off elsewhere: in the
// power-capped DiT steps the dependents' CTAs waiting early on every SM cost
// more SM clock than the launch gaps they hide (the cfg3 step measured 1.6 %
// slower at ~100 MHz lower clocks).
bool pdl_enabled();
struct PdlScope {  // enables the attribute for the scope's launches on this thread
  bool prev;
  explicit PdlScope(bool on);
  ~PdlScope();
};

// Launch `kernel` on `stream`, with programmatic stream serialization when
// pdl_enabled(): then it may be scheduled while the stream's previous kernel
// is still running, and waits for it (griddep_wait) before reading or writing
// global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace nd
