// Host-side helpers shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "rwkv_b200.h"

namespace rwkvb {

constexpr size_t kMaxSmem = 200 * 1024;

// Streaming multiprocessors on the current device (cached per device).
int device_sms();

inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return RWKVB_OK;
  if (std::getenv("RWKVB_DEBUG")) std::fprintf(stderr, "rwkvb: CUDA error %d: %s\n", (int)e, cudaGetErrorString(e));
  cudaGetLastError();  // clear a non-sticky error so the next call starts clean
  return e == cudaErrorMemoryAllocation ? RWKVB_EALLOC : RWKVB_ECUDA;
}

// Raise a kernel's dynamic shared-memory limit to kMaxSmem once per device.
int allow_big_smem(const void* kernel);

// Tiled TMA tensor map over a u8 array (dims innermost first, strides in bytes
// for dims 1..rank-1), no interleave, optional 128-byte swizzle, zero OOB fill.
// The driver entry point is resolved through the runtime (no libcuda link).
int encode_u8_map(CUtensorMap* out, int rank, const void* addr, const uint64_t* dims, const uint64_t* strides,
                  const uint32_t* box, bool swizzle128);

}  // namespace rwkvb
