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

}  // namespace nd
