// Batched LUT2 (TR2\x04) GEMM on the 5th-generation tensor cores (tcgen05,
// kind::f16):
//     Y[b][n] = sum_k W[n][k] x[b][k]      (b < nb <= 64 sessions)
// for the batched decode step of engines whose projections and head are LUT2
// (the reference's per-row product is trinity_grouped_lut2_gemv_f32,
// rwkv_ssd/native/lut2_gather.c:269-335).
//
// Operands:
//   A = the weights: every weight IS one of its group's four fp16 codebook
//       values, so the 2-bit codes decode to an exact fp16 tile (128 rows x
//       64 columns = one code group per row, 128-byte swizzled rows);
//   B = the activations as the engine's three digit rows per session
//       (x = c_g (X0 + X1/254 + X2/254^2) per 64-column group g, X_i stored
//       as X_i + 127), each turned into an fp16 plane
//           P_i = r_g (X_i - 127),   r_g = c_g / S,
//       S = the largest c_g of the session over the segment's K range: r_g is
//       a power of two <= 1 and X_i - 127 an integer in [-127, 127], so every
//       P_i is exact in fp16 (one byte permute builds 1024 + X_i + 127 as an
//       fp16, one HFMA2 applies r_g and the offset); rows [i bp, (i+1) bp)
//       hold plane i.
// The MMA (M 128, N 3 bp, K 16) accumulates D_i = sum W P_i in fp32 TMEM over
// the whole segment -- the codebook values are the weights, so nothing is
// flushed per group -- and the epilogue writes S (D0 + D1/254 + D2/254^2),
// the digit algebra of the SG8 GEMM with fp16 weights.
//
// Work split: (tile, 64-column stage) pairs of all matrices of a launch are
// numbered in order and every CTA takes a contiguous, equal share (as the SG8
// GEMM); the partial sums of a tile's CTA go to piece slot (cta - first cta of
// the tile) of [pieces][nb][rows], which consumers add in slot order.
//
// Roles (22 warps): warp 0 lane 0 issues the raw copies of a stage (codes,
// codebook records, digit rows, group scales) into a deep ring that the decode
// warps release as soon as they have read a slot, so copies run up to eight
// stages ahead whatever the MMAs are doing; the decode warps write the A and B
// tiles into a short operand ring that the MMAs release; warp 1 allocates
// TMEM (two accumulators of up to 192 columns) and lane 0 issues the MMAs; warps
// 2..5 are the epilogue (TMEM lane quarter = warp % 4, one row per lane);
// warps 6..21 decode the raw stage into the A and B operand tiles.  Every wait
// is bounded: on a limit the CTA sets the error word, drains the copies it
// issued and returns.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "bgemm.cuh"
#include "imma.cuh"
#include "stream.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace rwkvb {

constexpr int kLmWarps = 22;
constexpr int kLmThreads = kLmWarps * 32;
constexpr int kLmBuildWarps = 16;  // warps 6..21
constexpr int kLmMaxMats = 3;
constexpr int kLmMaxRaw = 8;  // raw-copy ring slots (codes, records, digit rows, scales)
constexpr int kLmOps = 4;     // operand ring slots (A and B tiles)
constexpr int kLmAccStride = 256;  // TMEM columns between the two accumulators
constexpr int kLmTmemCols = 512;
constexpr int kLmATile = 128 * 128;  // A: 128 rows x 64 fp16

// Instruction descriptor, kind::f16: D f32 (c_format 1, bits [4,6)), A and B
// f16 (a_format / b_format 0), both K-major, N >> 3 in [17,23), M >> 4 in
// [24,29).
__host__ __device__ constexpr uint32_t idesc_f16f16_f32(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T in fp16 with fp32 accumulation, issued by
// ONE thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Generic-proxy shared-memory writes made visible to the async proxy (the
// tensor cores read the operand tiles the decode warps wrote).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

struct LmMat {
  float* out;    // partial sums [pieces][nb][rows]
  const float* cs;  // group scales of the digit rows: c_g at cs[g * 2 bp + b]
  int rows, k;   // N, K (rows % 128 == 0, k % 128 == 0)
  int tiles;     // rows / 128
  int stage0;    // first global stage index of this matrix
};

struct LmArgs {
  CUtensorMap cmap[kLmMaxMats];  // codes, bytes {k / 4, rows}, box {16, 128}
  CUtensorMap rmap[kLmMaxMats];  // records, bytes {k / 8, rows}, box {16, 128} (two groups)
  CUtensorMap dmap[kLmMaxMats];  // digit rows, bytes {k, nrows}, box {64, 3 bp}
  LmMat mat[kLmMaxMats];
  int nmat, total;               // matrices, stages over all matrices
  int nb, bp;                    // sessions, padded sessions (MMA N = 3 bp)
  int rstages;                   // raw ring slots (<= kLmMaxRaw)
  int raw_bytes;                 // raw slot stride (multiple of 128): codes | records | digit rows | scales
  int op_bytes;                  // operand slot stride (multiple of 1024): A | B (3 bp rows)
  int r_dig, r_cs;               // digit rows / scales offsets in a raw slot (codes at 0, records at 2048)
  uint32_t tx_bytes;             // bytes of the raw copies of one stage
  uint32_t idesc;
  int* err;
};

// One segment: stages [s0, s1) of tile t of matrix m, piece p.
struct LmSeg {
  int m, t, s0, s1, p;
};

__device__ __forceinline__ LmSeg lm_segment(const LmArgs& a, int x, int hi) {
  int m = 0;
#pragma unroll 1
  while (m + 1 < a.nmat && x >= a.mat[m + 1].stage0) ++m;
  const LmMat& M = a.mat[m];
  const int G = M.k >> 6;
  const int local = x - M.stage0;
  LmSeg s;
  s.m = m;
  s.t = local / G;
  s.s0 = local - s.t * G;
  const int tile_hi = M.stage0 + (s.t + 1) * G;
  s.s1 = s.s0 + (min(hi, tile_hi) - x);
  s.p = (int)blockIdx.x - bg_cta_of32(M.stage0 + s.t * G, a.total, gridDim.x);
  return s;
}

__device__ __forceinline__ bool lm_wait(uint64_t* bar, uint32_t parity, const LmArgs& a, volatile int* abort_flag) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) {
    if (!*abort_flag) {
      ok = mbar_wait_suspend(bar, parity) ? 1 : 0;
      if (!ok) {
        atomicOr(a.err, kErrTimeout);
        *abort_flag = 1;
      }
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Largest group scale c_g of session b over groups [g0, g1), the groups split
// over `n` cooperating lanes (lane index i of n, adjacent lanes of one warp);
// 1 for padded sessions.  Order-independent, so every caller gets the same S.
__device__ __forceinline__ float lm_scale(const LmArgs& a, const LmMat& M, int b, int g0, int g1, int i, int n) {
  float s = 0.f;
  if (b < a.nb) {
    const float* p = M.cs + b;
    const size_t st = (size_t)2 * a.bp;
    int g = g0 + i;
    for (; g + 3 * n < g1; g += 4 * n) {  // four loads in flight
      const float v0 = __ldcg(p + g * st), v1 = __ldcg(p + (g + n) * st);
      const float v2 = __ldcg(p + (g + 2 * n) * st), v3 = __ldcg(p + (g + 3 * n) * st);
      s = fmaxf(s, fmaxf(fmaxf(v0, v1), fmaxf(v2, v3)));
    }
    for (; g < g1; g += n) s = fmaxf(s, __ldcg(p + g * st));
  }
  for (int o = 1; o < n; o <<= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
  return s > 0.f ? s : 1.f;
}

// PRMT selector of a nibble of codes (two 2-bit codes, LSB first): bytes
// 2 c0, 2 c0 + 1, 2 c1, 2 c1 + 1 of the 8-byte record {lo, hi}, i.e. the two
// fp16 codebook values as one half2.
__device__ __forceinline__ uint32_t lm_sel(uint32_t n) { return 0x1010u + 0x22u * ((n & 3u) | ((n & 0xCu) << 6)); }

__global__ void __launch_bounds__(kLmThreads, 1) l2mma_kernel(const __grid_constant__ LmArgs a) {
  extern __shared__ __align__(1024) uint8_t lm_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(lm_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem + kLmOps * a.op_bytes;
  __shared__ __align__(8) uint64_t rfull[kLmMaxRaw], rempty[kLmMaxRaw], built[kLmOps], oempty[kLmOps], tfull[2],
      tempty[2], done_bar;
  __shared__ uint32_t s_tbase;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lo = bg_range_lo32(blockIdx.x, a.total, gridDim.x);
  const int hi = bg_range_lo32(blockIdx.x + 1, a.total, gridDim.x);
  const uint32_t R = (uint32_t)a.rstages;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < R; ++i) {
      mbar_init(&rfull[i], 1);
      mbar_init(&rempty[i], kLmBuildWarps);
    }
    for (int i = 0; i < kLmOps; ++i) {
      mbar_init(&built[i], kLmBuildWarps);
      mbar_init(&oempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(&done_bar, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tbase, kLmTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s_tbase;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Codes and records of the first R stages go out before the grid
    // dependency wait (weights never depend on the previous kernel); digit
    // rows and group scales, written by the previous kernel, after it.
    uint32_t npre = 0;
    if (lane == 0) {
      for (int x = lo; x < hi && npre < R;) {
        const LmSeg sg = lm_segment(a, x, hi);
        for (int st = sg.s0; st < sg.s1 && npre < R; ++st, ++npre) {
          uint8_t* slot = raw + npre * a.raw_bytes;
          mbar_expect_tx(&rfull[npre], a.tx_bytes);
          tma_load_2d_hint(slot, &a.cmap[sg.m], st * 16, sg.t * 128, &rfull[npre], l2_evict_first());
          tma_load_2d_hint(slot + 2048, &a.rmap[sg.m], (st >> 1) * 16, sg.t * 128, &rfull[npre], l2_evict_first());
        }
        x += sg.s1 - sg.s0;
      }
    }
    npre = __shfl_sync(0xffffffffu, npre, 0);
    pdl_wait();
    pdl_launch_dependents();
    uint32_t use = 0;
    for (int x = lo; x < hi;) {
      const LmSeg sg = lm_segment(a, x, hi);
      const LmMat& M = a.mat[sg.m];
      for (int st = sg.s0; st < sg.s1; ++st, ++use) {
        const uint32_t ri = use % R, n = use / R;
        uint8_t* slot = raw + ri * a.raw_bytes;
        if (use >= npre) {
          if (!lm_wait(&rempty[ri], (n & 1) ^ 1, a, &s_abort)) goto producer_drain;
          if (lane == 0) {
            mbar_expect_tx(&rfull[ri], a.tx_bytes);
            tma_load_2d_hint(slot, &a.cmap[sg.m], st * 16, sg.t * 128, &rfull[ri], l2_evict_first());
            tma_load_2d_hint(slot + 2048, &a.rmap[sg.m], (st >> 1) * 16, sg.t * 128, &rfull[ri], l2_evict_first());
          }
        }
        if (lane == 0) {
          tma_load_2d(slot + a.r_dig, &a.dmap[sg.m], st * 64, 0, &rfull[ri]);
          bulk_g2s(slot + a.r_cs, M.cs + (size_t)st * 2 * a.bp, (uint32_t)(4 * a.bp), &rfull[ri]);
        }
        __syncwarp();
      }
      x += sg.s1 - sg.s0;
    }
  producer_drain:
    // the copies still in flight are among the last min(R, use) issues
    if (lane == 0)
      for (uint32_t u = use > R ? use - R : 0; u < use; ++u)
        mbar_wait_suspend(&rfull[u % R], (u / R) & 1);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    pdl_launch_dependents();  // reads shared memory only
    uint32_t use = 0, seg = 0;
    for (int x = lo; x < hi; ++seg) {
      const LmSeg sg = lm_segment(a, x, hi);
      const uint32_t tb = seg & 1;
      if (!lm_wait(&tempty[tb], ((seg >> 1) & 1) ^ 1, a, &s_abort)) goto mma_done;
      tc_fence_after();
      const uint32_t dt = tbase + tb * kLmAccStride;
      for (int st = sg.s0; st < sg.s1; ++st, ++use) {
        const uint32_t oi = use % kLmOps, n = use / kLmOps;
        if (!lm_wait(&built[oi], n & 1, a, &s_abort)) goto mma_done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = smem_u32(smem + oi * a.op_bytes);
          const uint32_t sb = sa + (uint32_t)kLmATile;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            umma_f16(dt, sdesc_k128(sa + 32 * j), sdesc_k128(sb + 32 * j), a.idesc,
                     (st > sg.s0 || j > 0) ? 1u : 0u);
          umma_commit(&oempty[oi]);
          if (st + 1 == sg.s1) umma_commit(&tfull[tb]);
        }
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
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // group scales come from the previous kernel; outputs may be read by it
    pdl_launch_dependents();
    const int q4 = warp & 3;
    const uint32_t tl = tbase + ((uint32_t)(q4 * 32) << 16);
    uint32_t seg = 0;
    for (int x = lo; x < hi; ++seg) {
      const LmSeg sg = lm_segment(a, x, hi);
      const LmMat& M = a.mat[sg.m];
      // S of sessions lane and lane + 32 (the decode warps derive the same values)
      const float s_a = lm_scale(a, M, lane, sg.s0, sg.s1, 0, 1);
      const float s_b = lm_scale(a, M, lane + 32, sg.s0, sg.s1, 0, 1);
      const uint32_t tb = seg & 1;
      if (!lm_wait(&tfull[tb], (seg >> 1) & 1, a, &s_abort)) goto epi_done;
      tc_fence_after();
      const int row = sg.t * 128 + q4 * 32 + lane;
      float* out = M.out + (size_t)sg.p * a.nb * M.rows + row;
      const uint32_t ta = tl + tb * kLmAccStride;
      for (int c0 = 0; c0 < a.bp; c0 += 16) {
        uint32_t d0[16], d1[16], d2[16];
        tmem_ld16x3_sync(ta + c0, ta + a.bp + c0, ta + 2 * a.bp + c0, d0, d1, d2);
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          const int b = c0 + s;
          const float sc = __shfl_sync(0xffffffffu, b < 32 ? s_a : s_b, b & 31);
          const float y = fmaf(fmaf(__uint_as_float(d2[s]), kInv254, __uint_as_float(d1[s])), kInv254,
                               __uint_as_float(d0[s]));
          if (b < a.nb) out[(size_t)b * M.rows] = sc * y;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[tb]);
      x += sg.s1 - sg.s0;
    }
  epi_done:;
  } else {
    // ------------------------------------------------------------ decode warps
    // A: thread t decodes code word t & 3 (16 weights, two 16-byte chunks) of
    // row t >> 2; B: thread t builds session t >> 3, columns 8 (t & 7) ..+7
    // (one 16-byte chunk of each of the three planes).  Consecutive lanes read consecutive
    // staging bytes and write distinct swizzled chunks: no bank conflicts.  A
    // raw slot is read into registers and released before the operand slot is
    // awaited.
    pdl_wait();
    pdl_launch_dependents();
    const int t = threadIdx.x - 6 * 32;
    const int ar = t >> 2, aw = t & 3;
    const int bb = t >> 3, bq = t & 7;
    const bool live = bb < a.nb;
    uint32_t use = 0;
    for (int x = lo; x < hi;) {
      const LmSeg sg = lm_segment(a, x, hi);
      const LmMat& M = a.mat[sg.m];
      // 1 / S: r_g = c_g / S is then a power of two to within one rounding
      // (both are 2^e / 127 in fp32; S is undone by the epilogue's multiply)
      const float inv_s = __frcp_rn(lm_scale(a, M, bb, sg.s0, sg.s1, bq, 8));
      for (int st = sg.s0; st < sg.s1; ++st, ++use) {
        const uint32_t ri = use % R, nr = use / R;
        const uint32_t oi = use % kLmOps, no = use / kLmOps;
        if (!lm_wait(&rfull[ri], nr & 1, a, &s_abort)) goto build_done;
        const uint8_t* slot = raw + ri * a.raw_bytes;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(slot + ar * 16 + 4 * aw);
        const uint2 rec = *reinterpret_cast<const uint2*>(slot + 2048 + ar * 16 + 8 * (st & 1));
        uint2 d0 = make_uint2(0u, 0u), d1 = d0, d2 = d0;
        float cf = 0.f;
        if (live) {
          const uint8_t* dg = slot + a.r_dig + 8 * bq;
          d0 = *reinterpret_cast<const uint2*>(dg + (size_t)bb * 64);
          d1 = *reinterpret_cast<const uint2*>(dg + (size_t)(a.bp + bb) * 64);
          d2 = *reinterpret_cast<const uint2*>(dg + (size_t)(2 * a.bp + bb) * 64);
          cf = reinterpret_cast<const float*>(slot + a.r_cs)[bb];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[ri]);
        uint32_t h2[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) h2[p] = __byte_perm(rec.x, rec.y, lm_sel((w >> (4 * p)) & 15u));
        // planes: (1024 + byte) as fp16 by one permute per pair, then
        // r (1024 + X + 127) - 1151 r = r X exactly by one HFMA2
        const float ratio = live ? cf * inv_s : 0.f;
        const __half2 r2 = __float2half2_rn(ratio), o2 = __float2half2_rn(-1151.f * ratio);
        uint32_t pv[3][4];
        const uint2 dd[3] = {d0, d1, d2};
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t hb = __byte_perm(j < 2 ? dd[i].x : dd[i].y, 0x64646464u, (j & 1) ? 0x4342u : 0x4140u);
            const __half2 v = __hfma2(*reinterpret_cast<const __half2*>(&hb), r2, o2);
            pv[i][j] = *reinterpret_cast<const uint32_t*>(&v);
          }
        if (!lm_wait(&oempty[oi], (no & 1) ^ 1, a, &s_abort)) goto build_done;
        uint8_t* op = smem + oi * a.op_bytes;
        uint8_t* arow = op + ar * 128;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int chunk = 2 * aw + c;
          *reinterpret_cast<uint4*>(arow + ((chunk ^ (ar & 7)) << 4)) =
              make_uint4(h2[4 * c], h2[4 * c + 1], h2[4 * c + 2], h2[4 * c + 3]);
        }
        if (bb < a.bp) {
          const int sw = (bq ^ (bb & 7)) << 4;  // rows i bp + bb share (row & 7)
#pragma unroll
          for (int i = 0; i < 3; ++i)
            *reinterpret_cast<uint4*>(op + kLmATile + (size_t)(i * a.bp + bb) * 128 + sw) =
                make_uint4(pv[i][0], pv[i][1], pv[i][2], pv[i][3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&built[oi]);
      }
      x += sg.s1 - sg.s0;
    }
  build_done:;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kLmTmemCols);
  }
}

}  // namespace rwkvb
