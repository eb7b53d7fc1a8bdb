// Batched SG8 GEMM on the 5th-generation tensor cores (tcgen05, kind::i8):
//     Y[b][n] = sum_k W[n][k] x[b][k]      (b < nb <= 64 sessions)
// for the batched decode step (r/k/v/o projections, FFN key/value, head).
//
// Operands, all exact integers:
//   A = the raw u8 weight codes of a 128-row x 128-column tile (TMA, 128-byte
//       swizzle), no conversion;
//   B = the activations as three unsigned 8-bit digit rows per session plus a
//       row of ones: per flush group f (FG = weight group, 64 or 128 columns)
//           x = c_f (X0 + X1/254 + X2/254^2),  c_f = 2^e_f / 127,
//       X_i in [-127, 127] stored as X_i + 127 in [0, 254]; rows
//       [0,bp) = digit 0, [bp,2bp) = digit 1, [2bp,3bp) = digit 2, 3bp = ones.
// The MMA (M 128, N = digit rows) accumulates D'_i = sum q (X_i + 127) and
// Q = sum q (the ones row) in TMEM; per flush group the epilogue recovers
// D_i = D'_i - 127 Q exactly and adds
//     min * sum_x + d * c_f * (D0 + D1/254 + D2/254^2),   d = (max - min) / 255
// which is the per-group algebra of the reference's SG8 row dot
// (rwkv_ssd/native/lut2_gather.c:344-381) for every session at once.
// |D_i| <= 128 * 255 * 127 < 2^22, so a D_i becomes a float exactly through
// the 1.5 * 2^23 bias (one integer add and one float subtract).
//
// Work split: the (tile, 128-column stage) pairs of all matrices of a launch
// are numbered in order and every CTA takes a contiguous, equal share, so
// each SM streams the same bytes.  A CTA writes the partial sums of each tile
// it touches into piece slot (cta - first cta of the tile); consumers add the
// pieces of a tile in slot order (deterministic).
//
// Roles (18 warps): warp 0 lane 0 issues the TMA loads into a ring of stages;
// warp 1 allocates TMEM (two accumulators of up to 256 columns) and lane 0
// issues the MMAs, one commit per flush group to the accumulator's "full"
// barrier and one per stage to the slot's "empty" barrier; warps 2..17 are the
// epilogue (TMEM lane quarter = warp % 4, 16 sessions per warp; 4 when the
// sessions pad to 16).
// Every wait is bounded: on a limit the CTA sets the error word, drains the
// copies it issued and returns.
#pragma once

#include <cuda.h>

#include "imma.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace rwkvb {

// Packed pairs of fp32 (Blackwell f32x2 arithmetic on 64-bit registers).
__device__ __forceinline__ uint64_t fx2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void fx2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

constexpr int kBgWarps = 18;
constexpr int kBgThreads = kBgWarps * 32;
constexpr int kBgMaxMats = 4;
constexpr int kBgMaxSessions = 64;
constexpr int kBgTileBytes = 128 * 128;  // A stage: 128 rows x 128 codes
constexpr int kBgTmemCols = 512;
constexpr int kBgAccStride = 256;        // TMEM columns between the two accumulators
constexpr int kBgMaxStages = 6;
constexpr int kBgBias = 0x4B400000;      // bits of 1.5 * 2^23
constexpr float kBgBiasF = 12582912.0f;  // 1.5 * 2^23

struct BgMat {
  const float2* pairs;  // (min, max) per (row, group): [rows][k / group]
  float* out;           // partial sums [pieces][nb][rows]
  int rows, k;          // N, K (multiples of 128)
  int lg;               // log2(group): 6 or 7
  int digits;           // digit matrix (B operand) index
  int tiles;            // rows / 128
  int stage0;           // first global stage index of this matrix
};

struct BgArgs {
  CUtensorMap amap[kBgMaxMats];   // codes {k, rows}, box {128, 128}, 128-byte swizzle
  CUtensorMap bmap[kBgMaxMats];   // digit rows {k, nrows}, box {128, nrows}, 128-byte swizzle
  BgMat mat[kBgMaxMats];
  const float* cs[kBgMaxMats];    // per digit matrix: c_f [k / group][bp] then sum_x (row + bp)
  int nmat;
  int total;                      // stages over all matrices
  int nb, bp, nrows;              // sessions, padded sessions, digit rows (= MMA N)
  int stages;                     // ring slots
  uint32_t idesc;
  int* err;
};

// CTA owning global stage x when `total` stages are split evenly over n CTAs
// (CTA c owns [floor(c total / n), floor((c+1) total / n))).
__host__ __device__ __forceinline__ int bg_cta_of(long long x, int total, int n) {
  return (int)(((x + 1) * (long long)n - 1) / total);
}
__host__ __device__ __forceinline__ int bg_range_lo(int c, int total, int n) {
  return (int)(((long long)c * total) / n);
}
// The same in 32-bit unsigned arithmetic for the kernels (a 64-bit division is
// a long software sequence at the start of every launch); exact while
// total * n < 2^31, which the launch setup checks.
__device__ __forceinline__ int bg_cta_of32(int x, int total, int n) {
  return (int)(((unsigned)(x + 1) * (unsigned)n - 1u) / (unsigned)total);
}
__device__ __forceinline__ int bg_range_lo32(int c, int total, int n) {
  return (int)(((unsigned)c * (unsigned)total) / (unsigned)n);
}

// One segment: stages [s0, s1) of tile t of matrix m, piece p.
struct BgSeg {
  int m, t, s0, s1, p;
};

// Next segment of [x, hi) (x < hi), in stage order.
__device__ __forceinline__ BgSeg bg_segment(const BgArgs& a, int x, int hi) {
  int m = 0;
#pragma unroll 1
  while (m + 1 < a.nmat && x >= a.mat[m + 1].stage0) ++m;
  const BgMat& M = a.mat[m];
  const int G = M.k >> 7;
  const int local = x - M.stage0;
  BgSeg s;
  s.m = m;
  s.t = local / G;
  s.s0 = local - s.t * G;
  const int tile_hi = M.stage0 + (s.t + 1) * G;
  s.s1 = s.s0 + (min(hi, tile_hi) - x);
  s.p = (int)blockIdx.x - bg_cta_of32(M.stage0 + s.t * G, a.total, gridDim.x);
  return s;
}

// Next ring slot; n counts the passes over the ring.
__device__ __forceinline__ void bg_advance(uint32_t& slot, uint32_t& n, uint32_t nstages) {
  if (++slot == nstages) {
    slot = 0;
    ++n;
  }
}

// Bounded wait by lane 0 of the calling warp, result broadcast to the warp
// (the whole warp calls it, so its lanes stay converged).
__device__ __forceinline__ bool bg_wait(uint64_t* bar, uint32_t parity, const BgArgs& a, volatile int* abort_flag) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) {
    if (!*abort_flag) {
      ok = mbar_wait_spin(bar, parity, kWaitLimitNs) ? 1 : 0;  // one polling lane per warp: prompt hand-offs
      if (!ok) {
        atomicOr(a.err, kErrTimeout);
        *abort_flag = 1;
      }
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__global__ void __maxnreg__(96) bgemm_kernel(const __grid_constant__ BgArgs a) {
  extern __shared__ __align__(1024) uint8_t bg_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(bg_smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = kBgTileBytes + a.nrows * 128;
  __shared__ __align__(8) uint64_t full[kBgMaxStages], empty[kBgMaxStages], tfull[2], tempty[2], done_bar;
  __shared__ uint32_t s_tbase;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lo = bg_range_lo32(blockIdx.x, a.total, gridDim.x);
  const int hi = bg_range_lo32(blockIdx.x + 1, a.total, gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kBgWarps - 2);
    }
    mbar_init(&done_bar, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tbase, kBgTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s_tbase;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    uint32_t use = 0;
    const uint32_t bytes = (uint32_t)stage_bytes;
    // The weight codes of the first `stages` stages go out before the grid
    // dependency wait (weights never depend on the previous kernel; under a
    // programmatic dependent launch they stream while it finishes); their
    // digit rows, written by the previous kernel, after it.  Weight codes are
    // read once per step: evict first, keep digit rows and constants in L2.
    uint32_t npre = 0;
    if (lane == 0) {
      for (int x = lo; x < hi && npre < (uint32_t)a.stages;) {
        const BgSeg sg = bg_segment(a, x, hi);
        for (int st = sg.s0; st < sg.s1 && npre < (uint32_t)a.stages; ++st, ++npre) {
          mbar_expect_tx(&full[npre], bytes);
          tma_load_2d_hint(smem + npre * stage_bytes, &a.amap[sg.m], st * 128, sg.t * 128, &full[npre],
                           l2_evict_first());
        }
        x += sg.s1 - sg.s0;
      }
    }
    npre = __shfl_sync(0xffffffffu, npre, 0);
    pdl_wait();
    pdl_launch_dependents();
    // ring slot and pass of stage `use`, advanced incrementally (no division
    // by the runtime depth on the issue path)
    uint32_t slot = 0, n = 0;
    const uint32_t nstages = (uint32_t)a.stages;
    for (int x = lo; x < hi;) {
      const BgSeg sg = bg_segment(a, x, hi);
      const BgMat& M = a.mat[sg.m];
      for (int st = sg.s0; st < sg.s1; ++st, ++use, bg_advance(slot, n, nstages)) {
        if (use < npre) {  // weights already issued; ring slot fresh
          if (lane == 0) tma_load_2d(smem + slot * stage_bytes + kBgTileBytes, &a.bmap[M.digits], st * 128, 0,
                                     &full[slot]);
          __syncwarp();
          continue;
        }
        if (!bg_wait(&empty[slot], (n & 1) ^ 1, a, &s_abort)) goto producer_drain;
        if (lane == 0) {
          uint8_t* sa = smem + slot * stage_bytes;
          mbar_expect_tx(&full[slot], bytes);
          tma_load_2d_hint(sa, &a.amap[sg.m], st * 128, sg.t * 128, &full[slot], l2_evict_first());
          tma_load_2d(sa + kBgTileBytes, &a.bmap[M.digits], st * 128, 0, &full[slot]);
        }
        __syncwarp();
      }
      x += sg.s1 - sg.s0;
    }
  producer_drain:
    // the copies still in flight are among the last min(stages, use) issues
    if (lane == 0)
      for (uint32_t u = use > (uint32_t)a.stages ? use - a.stages : 0; u < use; ++u)
        mbar_wait_suspend(&full[u % a.stages], (u / a.stages) & 1);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    pdl_launch_dependents();  // reads shared memory only (full barriers follow the producer's wait)
    uint32_t use = 0, fl = 0, slot = 0, n = 0;
    const uint32_t nstages = (uint32_t)a.stages;
    for (int x = lo; x < hi;) {
      const BgSeg sg = bg_segment(a, x, hi);
      const BgMat& M = a.mat[sg.m];
      const int nfl = 128 >> M.lg;  // flush groups per stage (1 or 2)
      const int kpf = 4 / nfl;      // 32-column k-steps per flush group
      for (int st = sg.s0; st < sg.s1; ++st, ++use, bg_advance(slot, n, nstages)) {
        if (!bg_wait(&full[slot], n & 1, a, &s_abort)) goto mma_done;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + slot * stage_bytes);
        const uint32_t sb = sa + kBgTileBytes;
        for (int f = 0; f < nfl; ++f, ++fl) {
          const uint32_t tb = fl & 1;
          if (!bg_wait(&tempty[tb], ((fl >> 1) & 1) ^ 1, a, &s_abort)) goto mma_done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t dt = tbase + tb * kBgAccStride;
            for (int j = 0; j < kpf; ++j) {
              const uint32_t ko = (uint32_t)((f * kpf + j) * 32);
              umma_u8(dt, sdesc_k128(sa + ko), sdesc_k128(sb + ko), a.idesc, j > 0 ? 1u : 0u);
            }
            umma_commit(&tfull[tb]);
          }
          __syncwarp();
        }
        if (lane == 0) umma_commit(&empty[slot]);
        __syncwarp();
      }
      x += sg.s1 - sg.s0;
    }
  mma_done:
    // every MMA issued so far has completed once done_bar's phase 0 ends
    if (lane == 0) {
      umma_commit(&done_bar);
      mbar_wait_suspend(&done_bar, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // per-session constants come from the previous kernel; outputs may be read by it
    pdl_launch_dependents();
    // warp w: TMEM lane quarter w % 4, sessions [16 ch, 16 ch + 16) with
    // ch = (w - 2) / 4; pairs of sessions go through packed f32x2 arithmetic.
    // With 16 padded sessions (narrow) every warp takes four, [4 ch, 4 ch + 4),
    // and one TMEM wait covers the ones column and the digits.
    const int q4 = warp & 3, ch = (warp - 2) >> 2;
    const bool narrow = a.bp == 16;
    const int sb = narrow ? 4 * ch : 16 * ch;  // the warp's first session
    const bool active = narrow || ch < (a.bp >> 4);
    const uint32_t tl = tbase + ((uint32_t)(q4 * 32) << 16);
    const uint64_t neg_bias = fx2(-kBgBiasF, -kBgBiasF), inv254 = fx2(kInv254, kInv254);
    uint32_t fl = 0;
    for (int x = lo; x < hi;) {
      const BgSeg sg = bg_segment(a, x, hi);
      const BgMat& M = a.mat[sg.m];
      const int row = sg.t * 128 + q4 * 32 + lane;
      const int gpr = M.k >> M.lg;
      const float2* prow = M.pairs + (size_t)row * gpr;
      const float* csm = a.cs[M.digits] + sb;
      const int nfl = 128 >> M.lg;
      uint64_t acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0ull;
      // (min, max) of this row's flush groups, loaded two groups ahead
      const int g_end = sg.s1 * nfl;
      float2 pr_a = __ldg(prow + sg.s0 * nfl);
      float2 pr_b = sg.s0 * nfl + 1 < g_end ? __ldg(prow + sg.s0 * nfl + 1) : make_float2(0.f, 0.f);
      for (int g = sg.s0 * nfl; g < g_end; ++g, ++fl) {
        const float2 pr = pr_a;
        pr_a = pr_b;
        if (g + 2 < g_end) pr_b = __ldg(prow + g + 2);
        const uint32_t tb = fl & 1;
        if (!bg_wait(&tfull[tb], (fl >> 1) & 1, a, &s_abort)) goto epi_done;
        tc_fence_after();
        if (narrow) {
          const uint32_t ta = tl + tb * kBgAccStride;
          uint32_t d0[4], d1[4], d2[4];
          const int q = (int)tmem_ld1_4x3_sync(ta + 3 * 16, ta + sb, ta + 16 + sb, ta + 2 * 16 + sb, d0, d1, d2);
          const int kq = kBgBias - 127 * q;
          const float dg = (pr.y - pr.x) * kInv255;
          const uint64_t dg2 = fx2(dg, dg), mn2 = fx2(pr.x, pr.x);
          const float* cg = csm + (size_t)g * 2 * 16;  // c_f of the warp's sessions; sum_x at + bp
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const uint64_t c2 = *reinterpret_cast<const uint64_t*>(cg + 2 * s);
            const uint64_t x2 = *reinterpret_cast<const uint64_t*>(cg + 16 + 2 * s);
            const uint64_t f0 = fadd2(
                fx2(__int_as_float((int)d0[2 * s] + kq), __int_as_float((int)d0[2 * s + 1] + kq)), neg_bias);
            const uint64_t f1 = fadd2(
                fx2(__int_as_float((int)d1[2 * s] + kq), __int_as_float((int)d1[2 * s + 1] + kq)), neg_bias);
            const uint64_t f2 = fadd2(
                fx2(__int_as_float((int)d2[2 * s] + kq), __int_as_float((int)d2[2 * s + 1] + kq)), neg_bias);
            const uint64_t t = ffma2(ffma2(f2, inv254, f1), inv254, f0);
            acc[s] = ffma2(fmul2(dg2, c2), t, ffma2(mn2, x2, acc[s]));
          }
        } else if (active) {
          const uint32_t ta = tl + tb * kBgAccStride;
          const int q = (int)tmem_ld1_sync(ta + 3 * a.bp);
          const int kq = kBgBias - 127 * q;
          const float dg = (pr.y - pr.x) * kInv255;
          const uint64_t dg2 = fx2(dg, dg), mn2 = fx2(pr.x, pr.x);
          const float* cg = csm + (size_t)g * 2 * a.bp;  // c_f of the chunk's sessions; sum_x at + bp
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {  // two rounds of 8 sessions (register budget)
            const uint32_t co = (uint32_t)(sb + hf * 8);
            uint32_t d0[8], d1[8], d2[8];
            tmem_ld8x3_sync(ta + co, ta + a.bp + co, ta + 2 * a.bp + co, d0, d1, d2);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
              const int sp = hf * 4 + s;  // session pair
              const uint64_t c2 = *reinterpret_cast<const uint64_t*>(cg + 2 * sp);
              const uint64_t x2 = *reinterpret_cast<const uint64_t*>(cg + a.bp + 2 * sp);
              const uint64_t f0 = fadd2(
                  fx2(__int_as_float((int)d0[2 * s] + kq), __int_as_float((int)d0[2 * s + 1] + kq)), neg_bias);
              const uint64_t f1 = fadd2(
                  fx2(__int_as_float((int)d1[2 * s] + kq), __int_as_float((int)d1[2 * s + 1] + kq)), neg_bias);
              const uint64_t f2 = fadd2(
                  fx2(__int_as_float((int)d2[2 * s] + kq), __int_as_float((int)d2[2 * s + 1] + kq)), neg_bias);
              const uint64_t t = ffma2(ffma2(f2, inv254, f1), inv254, f0);
              acc[sp] = ffma2(fmul2(dg2, c2), t, ffma2(mn2, x2, acc[sp]));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[tb]);
      }
      if (active) {
        float* out = M.out + (size_t)sg.p * a.nb * M.rows + row;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          if (narrow && s >= 2) break;
          float lo_v, hi_v;
          fx2_unpack(acc[s], lo_v, hi_v);
          const int b = sb + 2 * s;
          if (b < a.nb) out[(size_t)b * M.rows] = lo_v;
          if (b + 1 < a.nb) out[(size_t)(b + 1) * M.rows] = hi_v;
        }
      }
      x += sg.s1 - sg.s0;
    }
  epi_done:;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kBgTmemCols);
  }
}

// Digits of one flush group (1 << lfk = 64 or 128 columns, `per` = 2 or 4
// values per lane in v) for session b: the whole warp calls it.  Writes the
// three digit bytes (X + 127) of its values at column `col` of rows b, bp + b
// and 2 bp + b of dig [rows][k], c_f to cs[g][0][b] and sum_x to cs[g][1][b]
// (cs viewed as float [k / group][2][bp]).
__device__ __forceinline__ void bg_emit_group(const float (&v)[4], int per, uint8_t* dig, float2* cs, size_t k,
                                              size_t col, int b, int bp, int g) {
  const int lane = threadIdx.x & 31;
  float m = 0.f, sum = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    m = fmaxf(m, fabsf(v[u]));
    sum += v[u];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  int e = 0;
  if (m > 0.f) frexpf(m, &e);  // |x| 2^-e < 1
  const float inv = ldexpf(127.0f, -e);
  // rintf by the 1.5 * 2^23 shift (ties to even, |y| <= 127): the low byte of
  // the sum's bits is the integer's two's-complement byte; no float->int
  // conversion.  Stored digits are offset by 127 (u8).
  constexpr float kShift = 12582912.0f;
  uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float y0 = v[u] * inv;
    const float s0 = __fadd_rn(y0, kShift);
    const float x0 = __fsub_rn(s0, kShift);
    const float y1 = (y0 - x0) * 254.0f;
    const float s1 = __fadd_rn(y1, kShift);
    const float x1 = __fsub_rn(s1, kShift);
    const float s2 = __fadd_rn((y1 - x1) * 254.0f, kShift);
    w0 |= ((__float_as_uint(s0) + 127u) & 0xffu) << (8 * u);
    w1 |= ((__float_as_uint(s1) + 127u) & 0xffu) << (8 * u);
    w2 |= ((__float_as_uint(s2) + 127u) & 0xffu) << (8 * u);
  }
  if (per == 4) {
    *reinterpret_cast<uint32_t*>(dig + (size_t)b * k + col) = w0;
    *reinterpret_cast<uint32_t*>(dig + (size_t)(bp + b) * k + col) = w1;
    *reinterpret_cast<uint32_t*>(dig + (size_t)(2 * bp + b) * k + col) = w2;
  } else {
    *reinterpret_cast<uint16_t*>(dig + (size_t)b * k + col) = (uint16_t)w0;
    *reinterpret_cast<uint16_t*>(dig + (size_t)(bp + b) * k + col) = (uint16_t)w1;
    *reinterpret_cast<uint16_t*>(dig + (size_t)(2 * bp + b) * k + col) = (uint16_t)w2;
  }
  if (lane == 0) {
    float* cg = reinterpret_cast<float*>(cs) + (size_t)g * 2 * bp;
    cg[b] = ldexpf(1.0f, e) / 127.0f;
    cg[bp + b] = sum;
  }
}

// Digit rows of nb input vectors (row b of x at x + b * ldx, k columns) for
// flush groups of 1 << lfk columns (64 or 128): one warp per (session, group).
__global__ void __launch_bounds__(256) bg_digits_kernel(uint8_t* dig, float2* cs, const float* x, int ldx, int k,
                                                        int nb, int bp, int lfk) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int G = k >> lfk;
  if (gw >= nb * G) return;
  const int b = gw / G, g = gw - b * G;
  const int per = 1 << (lfk - 5);  // 2 or 4 values per lane
  const float* src = x + (size_t)b * ldx + ((size_t)g << lfk) + lane * per;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (per == 4) {
    const float4 t = *reinterpret_cast<const float4*>(src);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  } else {
    const float2 t = *reinterpret_cast<const float2*>(src);
    v[0] = t.x, v[1] = t.y;
  }
  bg_emit_group(v, per, dig, cs, (size_t)k, ((size_t)g << lfk) + lane * per, b, bp, g);
}

// y[b][n] = sum over the pieces of n's tile of part[p][b][n], in piece order.
__global__ void bg_reduce_kernel(float* y, const float* part, int nb, int rows, int stage0, int G, int total,
                                 int ncta) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * rows) return;
  const int b = i / rows, n = i - b * rows;
  const int t = n >> 7;
  const long long first = stage0 + (long long)t * G;
  const int np = bg_cta_of(first + G - 1, total, ncta) - bg_cta_of(first, total, ncta) + 1;
  float s = 0.f;
  for (int p = 0; p < np; ++p) s += part[((size_t)p * nb + b) * rows + n];
  y[i] = s;
}

}  // namespace rwkvb
