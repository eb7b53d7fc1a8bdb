// SG8 dot products on the integer tensor cores (mma.sync m16n8k32, u8 x s8 -> s32).
//
// A (16 rows x 32 k) is the raw u8 weight codes: no conversion at all.
// B (32 k x 8 columns) carries the activation as three signed 8-bit digits in
// columns 0..2 (columns 3..7 are zero): per flush group f of FG columns
// (FG = min(group, 128)) the input is scaled by 2^-e_f (e_f = exponent of the
// group's largest |x|, so |x| 2^-e_f < 1) and written
//     x = c_f (X0 + X1/254 + X2/254^2),   c_f = 2^e_f / 127,   X0, X1, X2 in [-127, 127]
// (reconstruction error <= c_f / 2 / 254^2, i.e. below 6.2e-8 of the group's
// largest |x|).  The three integer sums D_n = sum q X_n are exact, and per
// flush group (weights (min, max), d = (max - min) / 255)
//     sum_k w_k x_k = min * sum_k x_k + d * c_f * (D0 + D1/254 + D2/254^2)
// which is the per-group algebra of the reference's SG8 row dot
// (rwkv_ssd/native/lut2_gather.c:344-381).
//
// k order inside one 32-wide k-step: lane (g, t) of a quad group reads the 8
// contiguous code bytes [8t, 8t+8) of its rows and feeds them as logical k
// {4t..4t+3} (register a0/a1) and {16+4t..16+4t+3} (a2/a3).  The B fragment of
// lane (n, t) is digit n of x[8t .. 8t+8) in the same order, so the product is
// the plain dot product; only the pairing inside the k-step is permuted.
#pragma once

#include "common.cuh"

namespace rwkvb {

constexpr float kInv254 = 1.0f / 254.0f;
constexpr float kInv254sq = 1.0f / 64516.0f;

__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// m16n8k16 form (A 16 x 16 u8: a0 row g, a1 row g + 8, k 4t..4t+3 each; B
// 16 x 8 s8: b0 = k 4t..4t+3 of column g; D as in m16n8k32).
__device__ __forceinline__ void imma_16816(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// Named barrier over the `n` consumer threads (barrier 0 is __syncthreads).
__device__ __forceinline__ void bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
}

// Digit form of one input vector.
//   xd[s*12 + n*4 + t] (uint2) = digit n of x[32s + 8t .. +8)   (k-step s, n < 3, t < 4)
//   xc[f] = 2^e_f / 127,  xsum[f] = sum of x over flush group f (FG columns)
struct XDigits {
  uint2* xd;
  float* xc;
  float* xsum;
};

// Digits of one item (x[8 it .. 8 it + 8) held in v) into X.  All 32 lanes of
// the warp call it together (shuffles): the flush-group maximum and sum (FG =
// 32 << lfk columns = 4 << lfk items on adjacent lanes) are reduced across
// lanes; `act` = this lane holds a real item.
__device__ __forceinline__ void emit_digits(const float (&v)[8], int it, bool act, int lfk, const XDigits& X) {
  const int gl = 4 << lfk;
  float m = 0.f, sum = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    m = fmaxf(m, fabsf(v[u]));
    sum += v[u];
  }
  for (int o = 1; o < gl; o <<= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  if (!act) return;
  // m = f 2^e with f in [0.5, 1), so |x| 2^-e < 1; e, 127 * 2^-e and
  // 2^e / 127 (= 2^e * f32(1/127) exactly: power-of-two scaling commutes with
  // rounding) from the float bits, the library calls kept for the ends
  int e = 0;
  if (m > 0.f) {
    const uint32_t be = __float_as_uint(m) >> 23;
    if (be != 0u) e = (int)be - 126;
    else frexpf(m, &e);  // subnormal m
  }
  const float inv = (e > -122 && e < 127) ? 127.0f * __uint_as_float((uint32_t)(127 - e) << 23) : ldexpf(127.0f, -e);
  if ((it & (gl - 1)) == 0) {
    X.xc[it >> (lfk + 2)] = (e > -127 && e < 128) ? __uint_as_float((uint32_t)(127 + e) << 23) * (1.0f / 127.0f)
                                                   : ldexpf(1.0f, e) / 127.0f;
    X.xsum[it >> (lfk + 2)] = sum;
  }
  // Rounding by the 1.5 * 2^23 shift: for |y| < 2^22, (y + 1.5 * 2^23) rounds y
  // to the nearest integer, ties to even (the rintf rule), into the low
  // mantissa bits, so the low byte of the sum's bit pattern is the digit's
  // two's-complement byte and subtracting the shift gives rintf(y) exactly.
  // |y0| <= 127 and |y1|, |y2| <= 127 here.  No float->int conversion.
  constexpr float kShift = 12582912.0f;
  uint32_t b0[8], b1[8], b2[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float y0 = v[u] * inv;
    const float s0 = __fadd_rn(y0, kShift);
    const float x0 = __fsub_rn(s0, kShift);
    const float y1 = (y0 - x0) * 254.0f;
    const float s1 = __fadd_rn(y1, kShift);
    const float x1 = __fsub_rn(s1, kShift);
    const float s2 = __fadd_rn((y1 - x1) * 254.0f, kShift);
    b0[u] = __float_as_uint(s0);
    b1[u] = __float_as_uint(s1);
    b2[u] = __float_as_uint(s2);
  }
  // byte 0 of each word, four words per 32-bit result
  auto pk = [](const uint32_t* w) {
    return __byte_perm(__byte_perm(w[0], w[1], 0x0040), __byte_perm(w[2], w[3], 0x0040), 0x5410);
  };
  const int s = it >> 2, t = it & 3;
  X.xd[s * 12 + t] = make_uint2(pk(b0), pk(b0 + 4));
  X.xd[s * 12 + 4 + t] = make_uint2(pk(b1), pk(b1 + 4));
  X.xd[s * 12 + 8 + t] = make_uint2(pk(b2), pk(b2 + 4));
}

// Build the digit form of x[0..K): item it = (k-step it / 4, quarter it % 4)
// covers x[8 it .. 8 it + 8); thread ct of the `nthreads` consumers takes
// items ct, ct + nthreads, ...; the loads of the next item are in flight while
// the current one is converted (get4(i) = x[i..i+4), i % 4 == 0).  The
// flush-group maximum and sum (FG = 32 << lfk columns = 4 << lfk items, on
// adjacent lanes) are reduced with shuffles.  K % FG == 0, nthreads % 32 == 0.
// Ends with the consumer barrier `bar_id`.
template <class Get4>
__device__ __forceinline__ void build_digits(int K, int lfk, Get4 get4, XDigits X, int ct, int nthreads, int bar_id) {
  const int items = K >> 3;
  float4 na = make_float4(0.f, 0.f, 0.f, 0.f), nb = na;
  if (ct < items) {
    na = get4(ct * 8);
    nb = get4(ct * 8 + 4);
  }
#pragma unroll 1
  for (int base = 0; base < items; base += nthreads) {
    const int it = base + ct;
    const float v[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
    const int nx = it + nthreads;
    if (nx < items) {
      na = get4(nx * 8);
      nb = get4(nx * 8 + 4);
    }
    emit_digits(v, it, it < items, lfk, X);
  }
  bar_sync(bar_id, nthreads);
}

// build_digits with every round's operands loaded before the first emit
// (K <= 8 * MAXR * nthreads): one memory round trip for the whole vector
// instead of one per round of `nthreads` items.
template <int MAXR, typename Get4>
__device__ __forceinline__ void build_digits_r1(int K, int lfk, Get4 get4, XDigits X, int ct, int nthreads,
                                                int bar_id) {
  const int items = K >> 3;
  float4 va[MAXR], vb[MAXR];
#pragma unroll
  for (int r = 0; r < MAXR; ++r) {
    const int it = r * nthreads + ct;
    va[r] = vb[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (it < items) {
      va[r] = get4(it * 8);
      vb[r] = get4(it * 8 + 4);
    }
  }
#pragma unroll
  for (int r = 0; r < MAXR; ++r) {
    if (r * nthreads < items) {  // uniform: every lane of the warp emits together
      const int it = r * nthreads + ct;
      const float v[8] = {va[r].x, va[r].y, va[r].z, va[r].w, vb[r].x, vb[r].y, vb[r].z, vb[r].w};
      emit_digits(v, it, it < items, lfk, X);
    }
  }
  bar_sync(bar_id, nthreads);
}

// A-operand row g of the mma is tile row 2 (g & 3) + (g >> 2) (and g + 8 ->
// 8 + that): with the 128-byte swizzle (tma.cuh: chunk c of row r stored at
// c ^ (r & 7)) each half-warp's 8-byte loads then hit 8 distinct 16-byte
// chunks.  acc0 / acc1 of lane (g, t) belong to tile rows imma_tile_row(g) and
// imma_tile_row(g) + 8.
__device__ __forceinline__ int imma_tile_row(int g) { return 2 * (g & 3) + (g >> 2); }

// Per-lane constants of the swizzled A loads.
struct ImmaLane {
  int ra;          // tile row of acc0 (acc1: ra + 8)
  uint32_t roff;   // ra * 128 + 8 * (t & 1)
  uint32_t c[4];   // chunk offset of k-step j of a 128-column block
};

__device__ __forceinline__ ImmaLane imma_lane() {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  ImmaLane L;
  L.ra = imma_tile_row(g);
  L.roff = (uint32_t)(L.ra * 128 + 8 * (t & 1));
#pragma unroll
  for (int j = 0; j < 4; ++j) L.c[j] = (uint32_t)(((2 * j + (t >> 1)) ^ (L.ra & 7)) << 4);
  return L;
}

// One warp: 16 rows x one 128-column block of a swizzled tile.
//   blk:    tile + block * 2048 (the block's 16 lines)
//   pa, pb: (min, max) pairs of rows ra and ra + 8 for the block's first flush
//           group; flush group f uses pa[f] (a flush group never spans two
//           weight groups: FG = min(group, 128))
//   ks:     whole-row k-step index of the block's first k-step
// LFK = log2(flush group in k-steps): 2 for 128-column groups, 1 for 64.
// Only lanes with t < 2 carry values (t == 0: min terms and digits 0, 1;
// t == 1: digit 2); sum lanes t = 0 and 1 for the row totals.
template <int LFK>
__device__ __forceinline__ void imma_block(const uint8_t* blk, const float2* pa, const float2* pb, int ks,
                                           const XDigits& X, const ImmaLane& L, float& acc0, float& acc1) {
  const int lane = threadIdx.x & 31, t = lane & 3;
  const uint8_t* base = blk + L.roff;
  const uint2* xb = X.xd + ks * 12 + lane;
  uint2 w0[4], w1[4], bb[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    w0[j] = *reinterpret_cast<const uint2*>(base + L.c[j]);
    w1[j] = *reinterpret_cast<const uint2*>(base + L.c[j] + 1024);
    bb[j] = lane < 12 ? xb[j * 12] : make_uint2(0u, 0u);
  }
  constexpr int KPF = 1 << LFK, NF = 4 >> LFK;
#pragma unroll
  for (int f = 0; f < NF; ++f) {
    int d[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = f * KPF; j < (f + 1) * KPF; ++j) imma_16832(d, w0[j].x, w1[j].x, w0[j].y, w1[j].y, bb[j].x, bb[j].y);
    // without branches: lane t = 0 holds digits 0 and 1, t = 1 digit 2 and
    // the zero column 3 (so d1 / d3 are 0 there), t >= 2 zero columns (their
    // sums are never stored); each lane does exactly the operations of its
    // case: t = 0  da (d0 + d1 / 254) + min x_sum,  t = 1  da / 254^2 d0
    const int fg = (ks >> LFK) + f;
    const float c = X.xc[fg], xs = X.xsum[fg];
    const float2 p0 = pa[f], p1 = pb[f];
    const float sc = t == 0 ? 1.0f : kInv254sq;
    const float da = (p0.y - p0.x) * kInv255 * c, db = (p1.y - p1.x) * kInv255 * c;
    const float m0 = t == 0 ? p0.x : 0.f, m1 = t == 0 ? p1.x : 0.f;
    acc0 = fmaf(t == 0 ? da : da * sc, fmaf((float)d[1], kInv254, (float)d[0]), fmaf(m0, xs, acc0));
    acc1 = fmaf(t == 0 ? db : db * sc, fmaf((float)d[3], kInv254, (float)d[2]), fmaf(m1, xs, acc1));
  }
}

}  // namespace rwkvb
