// Packed-weight GEMV building blocks (device functions) shared by the op-level
// entry points and the fused decode engine.
#pragma once

#include "common.cuh"

namespace rwkvb {

// Conditions for the vectorised row-major paths: rows start on a group
// boundary, groups are a power of two of at least 16 (SG8) / 64 (LUT2), and
// the code payload is 16-byte aligned.
__host__ inline bool is_pow2(uint32_t v) { return v && !(v & (v - 1)); }
__host__ inline int ilog2u(uint32_t v) { int l = 0; while ((1u << l) < v) ++l; return l; }

__host__ inline bool sg8_fast_ok(const PackedView& w) {
  return w.kind == RWKVB_KIND_SG8 && is_pow2(w.group) && w.group >= 16 && (w.cols % w.group) == 0 &&
         (reinterpret_cast<uintptr_t>(w.payload) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w.meta) & 7u) == 0;
}

__host__ inline bool lut2_fast_ok(const PackedView& w) {
  return w.kind == RWKVB_KIND_LUT2_F16 && is_pow2(w.group) && w.group >= 64 && (w.cols % w.group) == 0 &&
         (reinterpret_cast<uintptr_t>(w.payload) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w.meta) & 7u) == 0;
}

// Stage x[0..K) into shared memory (sx) and its 16-element chunk sums (sxc),
// where x[i] = f(i).  K % 16 == 0.  Ends with __syncthreads().
template <class F>
__device__ __forceinline__ void stage_input(int K, float* sx, float* sxc, F f) {
  for (int i = threadIdx.x; i < K; i += blockDim.x) sx[i] = f(i);
  __syncthreads();
  for (int c = threadIdx.x; c < (K >> 4); c += blockDim.x) {
    const float4* p = reinterpret_cast<const float4*>(sx + (c << 4));
    float4 a = p[0], b = p[1], d = p[2], e = p[3];
    sxc[c] = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w)) + ((d.x + d.y) + (d.z + d.w)) +
             ((e.x + e.y) + (e.z + e.w));
  }
  __syncthreads();
}

// Rows [r0, r1) of an SG8 W (fast-path layout) times the staged input.
// Each warp owns RPW consecutive rows at a time; lanes stride over 16-byte
// chunks of the row.  Per chunk:  acc += d_g * sum(q*x) + min_g * sum(x),
// d_g = (max_g - min_g) / 255 (the reference's per-group algebra,
// lut2_gather.c:344-381).  epi(row, value) consumes each finished row.
template <int RPW, class Epi>
__device__ __forceinline__ void sg8_rows(const PackedView& W, int lg, const float* sx, const float* sxc,
                                         int r0, int r1, Epi epi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int K = W.cols, nchunk = K >> 4;
  const int gshift = lg - 4;  // chunks per group = 2^gshift
  const int gpr = K >> lg;    // groups per row
  for (int rb = r0 + warp * RPW; rb < r1; rb += nw * RPW) {
    float acc[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) acc[i] = 0.f;
    const uint8_t* qrow[RPW];
    const float2* srow[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      int row = min(rb + i, r1 - 1);
      qrow[i] = W.payload + (size_t)row * K;
      srow[i] = reinterpret_cast<const float2*>(W.meta) + (size_t)row * gpr;
    }
    int c = lane;
    for (; c + 32 < nchunk; c += 64) {
      uint4 q0[RPW], q1[RPW];
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        q0[i] = ldg_stream16(qrow[i] + (c << 4));
        q1[i] = ldg_stream16(qrow[i] + ((c + 32) << 4));
      }
      const float xs0 = sxc[c], xs1 = sxc[c + 32];
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        float2 s0 = __ldg(srow[i] + (c >> gshift));
        float2 s1 = __ldg(srow[i] + ((c + 32) >> gshift));
        float d0 = (s0.y - s0.x) * kInv255, d1 = (s1.y - s1.x) * kInv255;
        acc[i] = fmaf(d0, dot16_u8(q0[i], sx + (c << 4)), fmaf(s0.x, xs0, acc[i]));
        acc[i] = fmaf(d1, dot16_u8(q1[i], sx + ((c + 32) << 4)), fmaf(s1.x, xs1, acc[i]));
      }
    }
    if (c < nchunk) {
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        uint4 q = ldg_stream16(qrow[i] + (c << 4));
        float2 s = __ldg(srow[i] + (c >> gshift));
        float d = (s.y - s.x) * kInv255;
        acc[i] = fmaf(d, dot16_u8(q, sx + (c << 4)), fmaf(s.x, sxc[c], acc[i]));
      }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      float v = warp_sum(acc[i]);
      if (lane == 0 && rb + i < r1) epi(rb + i, v);
    }
  }
}

// One fp16 centroid from a 4-entry record held as two words, by 2-bit code.
__device__ __forceinline__ float lut2_pick(uint32_t lo, uint32_t hi, uint32_t code) {
  uint32_t sel = (code & 1u) ? 0x3232u : 0x1010u;
  uint32_t word = (code & 2u) ? hi : lo;
  return __half2float(__ushort_as_half((unsigned short)(__byte_perm(word, 0u, sel) & 0xffffu)));
}

// PRMT selector for a nibble of codes (two 2-bit codes, LSB first): bytes
// 2c0, 2c0 + 1, 2c1, 2c1 + 1 of the 8-byte record {lo, hi}, i.e. centroids c0
// and c1 as one half2.  0x1010 + 0x22 * (c0 + 256 c1).
__host__ __device__ constexpr uint32_t lut2_nibble_sel(uint32_t n) {
  return 0x1010u + 0x22u * ((n & 3u) | ((n & 0xCu) << 6));
}

// Rows [r0, r1) of a TR2\x04 W (fast-path layout: group >= 64, power of two,
// row-aligned).  Lane l of a warp takes 32-bit code words u = l, l + 32, ...
// of the row (16 weights each; 128 contiguous bytes per warp load; four words
// per row in flight per lane) and the
// matching 16 inputs as four float4 (contiguous across lanes: no bank
// conflicts), reused for the warp's RPW rows.  Two codes at a time become a
// half2 of centroids with one byte permute (selector per nibble from a 16-entry
// shared table) and two FMAs in fp32; the centroids are the record's exact fp16
// values.
template <int RPW, class Epi>
__device__ __forceinline__ void lut2_rows(const PackedView& W, int lg, const float* sx, int r0, int r1,
                                          Epi epi) {
  __shared__ uint32_t s_sel[16];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane < 16) s_sel[lane] = lut2_nibble_sel((uint32_t)lane);  // every warp writes the same values
  __syncwarp();
  const int K = W.cols, nword = K >> 4;  // 16 weights per code word
  const int wshift = lg - 4;             // code words per group = 2^wshift
  const int gpr = K >> lg;
  const uint32_t* codes = reinterpret_cast<const uint32_t*>(W.payload);
  const uint2* recs = reinterpret_cast<const uint2*>(W.meta);
  const float4* sx4 = reinterpret_cast<const float4*>(sx);
  for (int rb = r0 + warp * RPW; rb < r1; rb += nw * RPW) {
    float acc0[RPW], acc1[RPW];
    int row[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      acc0[i] = acc1[i] = 0.f;
      row[i] = min(rb + i, r1 - 1);
    }
    // four code words per lane and row (u0, u0 + 32, u0 + 64, u0 + 96) are
    // loaded before any is used: 16 bytes per lane and row in flight
    for (int u0 = lane; u0 < nword; u0 += 128) {
      uint32_t w[RPW][4];
      uint2 rec[RPW][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = u0 + 32 * j;
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
          w[i][j] = 0u;
          rec[i][j] = make_uint2(0u, 0u);
          if (u < nword) {
            w[i][j] = ldg_stream4(codes + (size_t)row[i] * nword + u);
            rec[i][j] = __ldg(recs + (size_t)row[i] * gpr + (u >> wshift));
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = u0 + 32 * j;
        if (u >= nword) break;
        const float4 xa = sx4[4 * u], xb = sx4[4 * u + 1], xc = sx4[4 * u + 2], xd = sx4[4 * u + 3];
        const float xv[16] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w,
                              xc.x, xc.y, xc.z, xc.w, xd.x, xd.y, xd.z, xd.w};
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const uint32_t sel = s_sel[(w[i][j] >> (4 * p)) & 15u];
            const uint32_t h2 = __byte_perm(rec[i][j].x, rec[i][j].y, sel);
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
            acc0[i] = fmaf(f.x, xv[2 * p], acc0[i]);
            acc1[i] = fmaf(f.y, xv[2 * p + 1], acc1[i]);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const float v = warp_sum(acc0[i] + acc1[i]);
      if (lane == 0 && rb + i < r1) epi(rb + i, v);
    }
  }
}

// Any packed W, any layout: one warp per row, lanes over columns, x in shared memory.
template <class Epi>
__device__ __forceinline__ void generic_rows(const PackedView& W, const float* sx, int r0, int r1, Epi epi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int row = r0 + warp; row < r1; row += nw) {
    float acc = 0.f;
    for (int c = lane; c < W.cols; c += 32) acc = fmaf(packed_at(W, row, c), sx[c], acc);
    acc = warp_sum(acc);
    if (lane == 0) epi(row, acc);
  }
}

// Dispatch for rows [r0, r1): fast layouts when allowed, else the generic path.
// `lg` = log2(group) (ignored by the generic path).
template <class Epi>
__device__ __forceinline__ void packed_rows(const PackedView& W, int mode, int lg, const float* sx,
                                            const float* sxc, int r0, int r1, Epi epi) {
  if (mode == 1) {
    sg8_rows<2>(W, lg, sx, sxc, r0, r1, epi);
  } else if (mode == 2) {
    lut2_rows<3>(W, lg, sx, r0, r1, epi);
  } else {
    generic_rows(W, sx, r0, r1, epi);
  }
}

__host__ inline int gemv_mode(const PackedView& w) {
  if (sg8_fast_ok(w)) return 1;
  if (lut2_fast_ok(w)) return 2;
  return 0;
}

// Transposed partial product for a row-major W [R_in, C_out] (x @ W):
//   part[j] = sum_{i in [i0, i1)} x[i] * W[i, j]  for j in [j0, j1)
// Threads stride over j; rows are walked in order (coalesced bytes across j).
__device__ __forceinline__ void transposed_partial(const PackedView& W, const float* x, int i0, int i1, int j0,
                                                   int j1, float* out) {
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    float acc = 0.f;
    for (int i = i0; i < i1; ++i) acc = fmaf(x[i], packed_at(W, i, j), acc);
    out[j - j0] = acc;
  }
}

}  // namespace rwkvb
