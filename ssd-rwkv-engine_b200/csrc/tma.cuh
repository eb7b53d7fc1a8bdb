// Tensor-map TMA copies (cp.async.bulk.tensor) used to stream SG8 row tiles.
//
// A weight matrix W [rows][K] of u8 codes is described by a rank-3 tensor map
// with dimensions {128 bytes, rows, K/128} and strides {K, 128}: one box
// {128, 16, nb} lands 16 rows x (nb * 128) codes in shared memory as
// [nb column blocks][16 rows][128 bytes], 128-byte swizzled (16-byte chunk c of
// the line for row r is stored at chunk c ^ (r & 7)).  The (min, max) pairs of
// the same rows use a rank-2 map {gpr * 8 bytes, rows} with a box
// {nb * 128 / group * 8, 16}, no swizzle.  No copy uses cluster multicast.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace rwkvb {

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
      "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

// The same loads with an L2 cache policy (createpolicy; l2_evict_first for the weight stream).
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3, %4}], [%5], %6;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
      "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3}], [%4], %5;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))),
      "l"(pol)
      : "memory");
}

// Hint: bring a box into L2 ahead of its load.
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

}  // namespace rwkvb
