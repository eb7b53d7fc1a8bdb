// 5th-generation tensor cores (tcgen05) for sm_100a: TMEM allocation, the
// shared-memory matrix descriptor, the integer MMA (kind::i8), its commit to
// an mbarrier, and TMEM -> register loads.
//
// Descriptor and instruction-descriptor bit layouts follow the PTX ISA
// (tcgen05 "shared memory descriptor" and "instruction descriptor" tables).
// Every operand tile here is K-major with the 128-byte swizzle that a TMA box
// of 128-byte rows produces: rows of 128 bytes, 8-row atoms of 1024 bytes
// (stride byte offset 1024), 16-byte chunk c of row r stored at c ^ (r & 7).
#pragma once

#include <stdint.h>

#include "stream.cuh"

namespace rwkvb {

// ------------------------------------------------------------ TMEM alloc
// Whole warp; writes the TMEM base address to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ------------------------------------------------------------ ordering
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ------------------------------------------------------------ descriptors
// K-major, 128-byte swizzle: start address >> 4 in bits [0,14), leading byte
// offset 16 B (>> 4 = 1, unused by swizzled K-major layouts) in [16,30),
// stride byte offset 1024 B (>> 4 = 64) in [32,46), descriptor version 1 in
// [46,48), base offset 0, layout type 2 (SWIZZLE_128B) in [61,64).
// The tile base must be 1024-byte aligned; the k-th 32-byte slice of the
// 128-byte rows starts at base + 32 k.
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)64u << 32) | ((uint64_t)1u << 46) |
         ((uint64_t)2u << 61);
}

// Instruction descriptor, kind::i8: D s32 (c_format 2, bits [4,6)), A and B
// unsigned 8-bit (a_format / b_format 0), both K-major, N >> 3 in [17,23),
// M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_u8u8_s32(int m, int n) {
  return (2u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ------------------------------------------------------------ MMA
// D[tmem] (+)= A[smem] * B[smem]^T, issued by ONE thread.
__device__ __forceinline__ void umma_u8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------ TMEM loads
// 32 lanes x 32 bits: lane i of the warp reads TMEM lane (base lane + i); the
// warp's lane quarter is fixed by (warp id % 4).
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The destination registers of tcgen05.ld are defined only after
// tcgen05.wait::ld; these helpers issue the loads and the wait in ONE asm
// statement so that no use of a register can be scheduled before the wait.
__device__ __forceinline__ uint32_t tmem_ld1_sync(uint32_t taddr) {
  uint32_t r;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r)
      : "r"(taddr)
      : "memory");
  return r;
}

// One column (tq) and three 4-column loads (columns t0.., t1.., t2..), one wait.
__device__ __forceinline__ uint32_t tmem_ld1_4x3_sync(uint32_t tq, uint32_t t0, uint32_t t1, uint32_t t2,
                                                     uint32_t (&a)[4], uint32_t (&b)[4], uint32_t (&c)[4]) {
  uint32_t q;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%13];\n"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%1,%2,%3,%4}, [%14];\n"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%5,%6,%7,%8}, [%15];\n"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%9,%10,%11,%12}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(q), "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]),
        "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(tq), "r"(t0), "r"(t1), "r"(t2)
      : "memory");
  return q;
}

// Three 8-column loads (columns t0.., t1.., t2..) and one wait.
__device__ __forceinline__ void tmem_ld8x3_sync(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t (&a)[8],
                                                uint32_t (&b)[8], uint32_t (&c)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%24];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%25];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%26];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(b[0]),
        "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(c[0]), "=r"(c[1]),
        "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]), "=r"(c[7])
      : "r"(t0), "r"(t1), "r"(t2)
      : "memory");
}

// Three 16-column loads (columns t0.., t1.., t2..) and one wait.
__device__ __forceinline__ void tmem_ld16x3_sync(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t (&a)[16],
                                                 uint32_t (&b)[16], uint32_t (&c)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%48];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%49];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47}, "
      "[%50];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(a[8]),
        "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]), "=r"(b[0]),
        "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]),
        "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15]), "=r"(c[0]), "=r"(c[1]),
        "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]), "=r"(c[7]), "=r"(c[8]), "=r"(c[9]), "=r"(c[10]),
        "=r"(c[11]), "=r"(c[12]), "=r"(c[13]), "=r"(c[14]), "=r"(c[15])
      : "r"(t0), "r"(t1), "r"(t2)
      : "memory");
}

}  // namespace rwkvb
