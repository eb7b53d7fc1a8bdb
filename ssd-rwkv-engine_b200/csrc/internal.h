// Host-side helpers shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

#include "rwkv_b200.h"

namespace rwkvb {

constexpr size_t kMaxSmem = 200 * 1024;

// Streaming multiprocessors on the current device (cached per device).
int device_sms();

inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return RWKVB_OK;
  cudaGetLastError();  // clear a non-sticky error so the next call starts clean
  return e == cudaErrorMemoryAllocation ? RWKVB_EALLOC : RWKVB_ECUDA;
}

// Raise a kernel's dynamic shared-memory limit to kMaxSmem once per device.
int allow_big_smem(const void* kernel);

}  // namespace rwkvb
