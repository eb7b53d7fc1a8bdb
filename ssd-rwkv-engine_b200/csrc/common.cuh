// Shared device helpers for the sm_100a RWKV-7 packed-weight kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "rwkv_b200.h"

namespace rwkvb {

constexpr float kInv255 = 1.0f / 255.0f;   // f32(1/255), pack_codec.py:174
constexpr float kMagic23 = 8388608.0f;     // 2^23: u8 placed in a float mantissa

// Device-side view of one packed matrix (parsed on the host).
struct PackedView {
  const uint8_t* meta;     // SG8: f32 (min,max) pairs; LUT2: per-group records
  const uint8_t* payload;  // SG8: u8 codes; LUT2: 2-bit codes, LSB first
  uint32_t kind;           // RWKVB_KIND_*
  uint32_t group;          // elements per group (flattened row-major order)
  uint32_t rec;            // bytes per group record (8 for SG8 and TR2\x04/\x06)
  int32_t rows, cols;      // checkpoint shape
  int32_t lg;              // log2(group) when group is a power of two, else -1
};

__host__ inline PackedView make_view(const rwkvb_packed& p) {
  PackedView v;
  // the per-tensor LUT2's codebook (its one "group record") starts at byte 4
  v.meta = p.data + (p.kind == RWKVB_KIND_LUT2_TENSOR ? 4 : 8);
  v.kind = p.kind;
  v.group = p.group_size;
  uint64_t numel = (uint64_t)p.rows * (uint64_t)p.cols;
  uint64_t groups = (numel + p.group_size - 1) / p.group_size;
  v.rec = p.kind == RWKVB_KIND_SG8 ? 8u : rwkvb_lut2_record_bytes(p.kind);
  v.payload = v.meta + groups * v.rec;
  v.rows = p.rows;
  v.cols = p.cols;
  v.lg = -1;
  for (int l = 0; l < 32; ++l)
    if ((1u << l) == p.group_size) v.lg = l;
  return v;
}

// ---------------------------------------------------------------- loads
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t ldg_stream4(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float2 ldg_f2(const void* p) {
  return __ldg(reinterpret_cast<const float2*>(p));
}

// Bulk prefetch of [p, p+bytes) into L2 (p and bytes 16-byte aligned).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ------------------------------------------------------------ u8 -> f32
// Byte i of w as an exact float: 2^23 + q assembled with one byte permute,
// then 2^23 subtracted (exact).
template <int I>
__device__ __forceinline__ float u8_to_f(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | I)) - kMagic23;
}

template <int I>
__device__ __forceinline__ float u8_magic(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | I));
}

// sum_{b<4} byte_b(w) * x[b] with packed fp32x2 arithmetic.
__device__ __forceinline__ float2 dot4_u8(uint32_t w, float4 x, float2 acc) {
  const float2 m = make_float2(-kMagic23, -kMagic23);
  float2 q01 = __fadd2_rn(make_float2(u8_magic<0>(w), u8_magic<1>(w)), m);
  float2 q23 = __fadd2_rn(make_float2(u8_magic<2>(w), u8_magic<3>(w)), m);
  acc = __ffma2_rn(q01, make_float2(x.x, x.y), acc);
  acc = __ffma2_rn(q23, make_float2(x.z, x.w), acc);
  return acc;
}

// sum over 16 u8 codes times 16 consecutive floats at xs (16-byte aligned, shared memory).
__device__ __forceinline__ float dot16_u8(uint4 q, const float* xs) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float2 a = make_float2(0.f, 0.f);
  a = dot4_u8(q.x, x4[0], a);
  a = dot4_u8(q.y, x4[1], a);
  a = dot4_u8(q.z, x4[2], a);
  a = dot4_u8(q.w, x4[3], a);
  return a.x + a.y;
}

// Bit-exact SG8 dequant of one element: q * ((max - min) * f32(1/255)) + min,
// two separate roundings (pack_codec.py:174-176).
__device__ __forceinline__ float sg8_dequant(uint32_t q, float mn, float mx) {
  float delta = __fmul_rn(__fsub_rn(mx, mn), kInv255);
  return __fadd_rn(__fmul_rn((float)q, delta), mn);
}

// Element e of an SG8 view (any layout, any group straddling).
__device__ __forceinline__ float sg8_elem(const PackedView& w, uint64_t e) {
  uint64_t g = e / w.group;
  float2 s = ldg_f2(w.meta + g * 8);
  return sg8_dequant(__ldg(w.payload + e), s.x, s.y);
}

__device__ __forceinline__ float half_bits_to_f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// Element e (encoded logical order) of a grouped LUT2 view, residual applied.
__device__ __forceinline__ float lut2_elem(const PackedView& w, uint64_t e) {
  uint64_t g = e / w.group;
  uint32_t local = (uint32_t)(e - g * w.group);
  uint32_t code = (__ldg(w.payload + (e >> 2)) >> ((e & 3u) * 2u)) & 3u;
  const uint8_t* r = w.meta + g * w.rec;
  float v;
  if (w.kind == RWKVB_KIND_LUT2_F32 || w.kind == RWKVB_KIND_LUT2_TENSOR) {
    v = __ldg(reinterpret_cast<const float*>(r) + code);
  } else {
    v = half_bits_to_f(__ldg(reinterpret_cast<const unsigned short*>(r) + code));
  }
  if (w.kind == RWKVB_KIND_LUT2_RES || w.kind == RWKVB_KIND_LUT2_IN_RES) {
    uint32_t p0 = __ldg(r + 8), p1 = __ldg(r + 9);
    if (local == p0) {
      v = __fadd_rn(v, half_bits_to_f(__ldg(reinterpret_cast<const unsigned short*>(r + 10))));
    } else if (local == p1) {
      v = __fadd_rn(v, half_bits_to_f(__ldg(reinterpret_cast<const unsigned short*>(r + 12))));
    }
  }
  return v;
}

__device__ __forceinline__ bool lut2_input_major(uint32_t kind) {
  return kind == RWKVB_KIND_LUT2_IN_F16 || kind == RWKVB_KIND_LUT2_IN_RES;
}

// SG8 element e of a tensor below 2^32 elements whose group is a power of two.
__device__ __forceinline__ float sg8_elem_pow2(const PackedView& w, uint32_t e) {
  float2 s = ldg_f2(w.meta + (size_t)(e >> w.lg) * 8);
  return sg8_dequant(__ldg(w.payload + e), s.x, s.y);
}

// W[row, col] for any packed view.
__device__ __forceinline__ float packed_at(const PackedView& w, int row, int col) {
  if (w.kind == RWKVB_KIND_SG8) {
    uint64_t e = (uint64_t)row * w.cols + col;
    if (w.lg >= 0 && e < 0xffffffffull) return sg8_elem_pow2(w, (uint32_t)e);
    return sg8_elem(w, e);
  }
  uint64_t e = lut2_input_major(w.kind) ? (uint64_t)col * w.rows + row : (uint64_t)row * w.cols + col;
  return lut2_elem(w, e);
}

// ------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; `red` is shared scratch of >= 32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

}  // namespace rwkvb
