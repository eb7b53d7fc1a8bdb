// Persistent decode kernel: every layer of every token of a decode call in
// one cooperative launch, one CTA per SM, warp-specialised.
//
//   warps 0..9  (consumers): activations, integer-MMA SG8 GEMV (imma.cuh),
//                            WKV7, LayerNorms, grid barriers
//   warp 10     (producer):  streams this CTA's weight tiles, in consumption
//                            order, through a ring of shared-memory slots with
//                            tensor-map TMA (tma.cuh); gated only by the
//                            slots' "empty" barriers, so HBM keeps streaming
//                            across the grid barriers of the data flow.
//
// Work split.  A big projection (r, k, v, o, ffn key, ffn value, head) is cut
// into units of 16 rows x KC = nb * 128 columns; every CTA owns a contiguous,
// balanced range of units (whole tiles when units are too few), so each CTA
// streams the same number of bytes.  A CTA adds its partial row sums of a tile
// into a zeroed fp32 accumulator with one atomic add per row; ranges are cut so
// that no row receives more than two contributions, which keeps the sum
// independent of arrival order (a + b == b + a).  Adapter first stages (x @ W1)
// are split by rows across CTAs and accumulated in 2^-32 fixed point (int64
// atomics: order-independent).  Accumulators are zeroed by CTA slices in a
// later phase, at least one grid barrier after their last read and before
// their next write, and once more at the start of every launch.
//
// Phases per layer (packed_block_forward.py:76-166, rwkv7_linear.py:125-435):
//   A  ln1 + token-shift mixes; r/k/v rows; adapter first stages
//   B  one CTA per head: adapter second stages (tiles streamed through the
//      ring), kk-normalize, decay, WKV7 state update, GroupNorm, bonus, gate
//   C  output projection                      (att_x[l] <- ln1 slice)
//   D  x += att; ln2 + mix; ffn key rows
//   E  relu^2; ffn value rows                 (ffn_x[l] <- ln2 slice)
// then the head (ln_out, logits) and a two-barrier first-maximum argmax.
//
// Every wait is bounded (slot barriers, grid barrier).  A timeout sets the
// engine's error word and the shared abort flag; consumers stop waiting and
// run to the next grid barrier, the producer stops issuing and drains its
// in-flight copies, and the kernel returns.
//
// Included by engine.cu after LayerDev / Bufs / Dims.
#pragma once

#include <cuda.h>

#include "imma.cuh"
#include "tma.cuh"
#include "wkv7.cuh"

namespace rwkvb {

constexpr int kDW = 10;                // consumer warps
constexpr int kDT = kDW * 32;          // consumer threads
constexpr int kDThreads = kDT + 32;    // + producer warp
constexpr int kDMaxSt = 8;             // ring slots (upper bound)
constexpr int kDBar = 1;               // named barrier of the consumers
constexpr int kDMaxItems = 8;          // adapter first-stage items per CTA
constexpr int kDMaxPieces = 8;         // adapter second-stage tile pieces per layer
constexpr int kDMisc = 2560;           // misc shared floats
constexpr float kFix = 4294967296.0f;  // 2^32 fixed-point scale of adapter partials
constexpr float kUnfix = 1.0f / 4294967296.0f;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long v;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(v));
  return v;
}

__device__ __forceinline__ unsigned d_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One LayerNorm output element; the single definition keeps the value stored
// for the next token's shift bit-identical to the one mixed now.
__device__ __forceinline__ float ln_val(float x, float mean, float rstd, float w, float b) {
  return fmaf(__fmul_rn(__fsub_rn(x, mean), rstd), w, b);
}

// Tensor maps of one layer: r, k, v, o, ffn key, ffn value (codes, pairs) and
// the four adapter second stages w2, a2, g2, v2 (64-column tiles, pairs).
struct DLayerMaps {
  CUtensorMap q[6], p[6], aq[4], ap[4];
};

struct DRange {
  int u0, u1, nch;  // units [u0, u1), chunks per 16-row tile
};

struct DArgs {
  const LayerDev* layers;
  const DLayerMaps* lmaps;       // [L]
  const CUtensorMap* head_maps;  // [2] codes, pairs
  PackedView emb;
  const float *ln0_w, *ln0_b, *lnout_w, *lnout_b;
  Bufs b;
  Dims d;
  int nb, kc, pr;    // 128-column blocks per chunk, chunk columns, pairs per chunk row
  int lg, fg;        // log2 group of the big matrices, flush group columns
  int nst, pf_dist;  // ring slots, L2 prefetch distance in stages
  uint32_t slot, code_b, pair_b;
  int abr[4];  // adapter second stage: box rows per matrix
  int alg[4];  // adapter second stage: log2 group
  int ntok, mode, first_tok;  // mode 0 greedy (step 0 consumes first_tok, -1: *tok), 1 forced tokens
  const int* forced;
  unsigned* gbar;
  uint32_t spin_limit;
  int emb_fast;
  unsigned long long* trace;
  int trace_cap;
  uint32_t o_dig, o_x, o_xb, o_t, o_p, o_part, o_misc, smem_total;
  uint32_t dig_set;  // bytes of one digit set of width C
};

struct DTable {
  DRange r[5];    // r/k/v (3C rows), o, ffn key, ffn value, head
  int nitem[2];   // adapter first-stage items: layer 0 (no v1), other layers
  int item[kDMaxItems];
  int npc[2];     // adapter second-stage pieces: layer 0 (no v2), other layers; 0 unless a head CTA
  int pm[kDMaxPieces], pr0[kDMaxPieces];
  int zc0, zc1, zf0, zf1, z3c0, z3c1, zv0, zv1, zr0, zr1;  // zeroing slices (C, F, 3C, V, rtot)
};

__device__ __forceinline__ void d_split(int n, int parts, int i, int* a, int* b) {
  *a = (int)((long long)n * i / parts);
  *b = (int)((long long)n * (i + 1) / parts);
}

__device__ __forceinline__ void d_range(int tiles, int nch, int G, int b, DRange& R) {
  const int U = tiles * nch;
  R.nch = nch;
  if (U / G >= nch - 1) {  // every range spans >= nch - 1 units: a tile meets at most two CTAs
    d_split(U, G, b, &R.u0, &R.u1);
  } else {  // whole tiles
    int t0, t1;
    d_split(tiles, G, b, &t0, &t1);
    R.u0 = t0 * nch;
    R.u1 = t1 * nch;
  }
}

__device__ __forceinline__ int d_rank(const Dims& d, int m) {
  return m == 0 ? d.rw : (m == 1 ? d.ra : (m == 2 ? d.rg : d.rv));
}

__device__ __forceinline__ int d_rank_off(const Dims& d, int m) {
  return m == 0 ? 0 : (m == 1 ? d.rw : (m == 2 ? d.rw + d.ra : d.rw + d.ra + d.rg));
}

__device__ void d_build_table(const DArgs& a, DTable& T) {
  const int G = gridDim.x, bx = blockIdx.x, C = a.d.C, F = a.d.F;
  const int nc = C / a.kc, nf = F / a.kc;
  d_range(3 * C / 16, nc, G, bx, T.r[0]);
  d_range(C / 16, nc, G, bx, T.r[1]);
  d_range(F / 16, nc, G, bx, T.r[2]);
  d_range(C / 16, nf, G, bx, T.r[3]);
  d_range((a.d.V + 15) / 16, nc, G, bx, T.r[4]);
  const int items3 = 3 * a.d.adp_splits, items4 = 4 * a.d.adp_splits;
  T.nitem[0] = T.nitem[1] = 0;
  for (int it = bx; it < items4 && T.nitem[1] < kDMaxItems; it += G) {
    T.item[T.nitem[1]++] = it;
    if (it < items3) T.nitem[0] = T.nitem[1];
  }
  T.npc[0] = T.npc[1] = 0;
  if (bx < a.d.H) {
    int n = 0;
    for (int m = 0; m < 4; ++m) {
      if (m == 3) T.npc[0] = n;
      const int R = d_rank(a.d, m);
      for (int r0 = 0; r0 < R && n < kDMaxPieces; r0 += a.abr[m]) {
        T.pm[n] = m;
        T.pr0[n] = r0;
        ++n;
      }
    }
    T.npc[1] = n;
  }
  d_split(C, G, bx, &T.zc0, &T.zc1);
  d_split(F, G, bx, &T.zf0, &T.zf1);
  d_split(3 * C, G, bx, &T.z3c0, &T.z3c1);
  d_split(a.d.V, G, bx, &T.zv0, &T.zv1);
  d_split(a.d.rtot, G, bx, &T.zr0, &T.zr1);
}

// ------------------------------------------------------------- producer
// The stage sequence of one CTA, exactly as the consumers consume it: per
// token, per layer [r/k/v units, adapter items, adapter-2 pieces, o units,
// ffn key units, ffn value units], then the head units (every token in greedy
// mode, the last one in forced mode).
struct DWalk {
  int tok, l, ph, i;  // ph: 0 r/k/v, 1 items, 2 pieces, 3 o, 4 ffn key, 5 ffn value, 6 head
};

__device__ __forceinline__ int d_phase_len(const DArgs& a, const DTable& T, const DWalk& w) {
  switch (w.ph) {
    case 0: return T.r[0].u1 - T.r[0].u0;
    case 1: return T.nitem[w.l == 0 ? 0 : 1];
    case 2: return T.npc[w.l == 0 ? 0 : 1];
    case 3: return T.r[1].u1 - T.r[1].u0;
    case 4: return T.r[2].u1 - T.r[2].u0;
    case 5: return T.r[3].u1 - T.r[3].u0;
    default: return (a.mode == 0 || w.tok == a.ntok - 1) ? T.r[4].u1 - T.r[4].u0 : 0;
  }
}

// Move `w` to the first stage at or after it; false at the end of the launch.
__device__ __forceinline__ bool d_norm(const DArgs& a, const DTable& T, DWalk& w) {
  while (w.tok < a.ntok) {
    if (w.i < d_phase_len(a, T, w)) return true;
    w.i = 0;
    if (w.ph < 5) {
      ++w.ph;
    } else if (w.ph == 5) {
      if (w.l + 1 < a.d.L) {
        ++w.l;
        w.ph = 0;
      } else {
        w.ph = 6;
      }
    } else {
      ++w.tok;
      w.l = 0;
      w.ph = 0;
    }
  }
  return false;
}

// Issue stage `w` into a slot (bar != nullptr: expect its bytes, then copy),
// or only bring it into L2 (bar == nullptr).
__device__ void d_stage(const DArgs& a, const DTable& T, const DWalk& w, uint8_t* dst, uint64_t* bar) {
  const int C = a.d.C, bx = blockIdx.x;
  if (w.ph == 1) {  // adapter first-stage item: rows [i0, i1) of W1 [C][R] and their pairs
    const LayerDev& Ly = a.layers[w.l];
    const int item = T.item[w.i];
    const int m = item / a.d.adp_splits, sp = item - m * a.d.adp_splits;
    const PackedView& W = m == 0 ? Ly.w1 : (m == 1 ? Ly.a1 : (m == 2 ? Ly.g1 : Ly.v1));
    const int R = W.cols;
    const int i0 = sp * a.d.adp_rows, i1 = min(C, i0 + a.d.adp_rows);
    const uint32_t qb = (uint32_t)((i1 - i0) * R);
    const uint32_t g0 = (uint32_t)(((uint64_t)i0 * R) >> W.lg) & ~1u;
    const uint32_t g1 = ((uint32_t)((((uint64_t)i1 * R - 1) >> W.lg) + 1) + 1u) & ~1u;
    const uint32_t sb = (g1 - g0) * 8u;
    if (bar) {
      mbar_expect_tx(bar, qb + sb);
      bulk_g2s(dst, W.payload + (size_t)i0 * R, qb, bar);
      bulk_g2s(dst + ((qb + 15u) & ~15u), W.meta + (size_t)g0 * 8, sb, bar);
    } else {
      prefetch_l2_bulk(W.payload + (size_t)i0 * R, qb);
      prefetch_l2_bulk(W.meta + (size_t)g0 * 8, sb);
    }
    return;
  }
  if (w.ph == 2) {  // adapter second-stage piece of this CTA's head
    const DLayerMaps& M = a.lmaps[w.l];
    const int m = T.pm[w.i], br = a.abr[m], r0 = T.pr0[w.i];
    const int px = (((bx * 64) >> a.alg[m]) & ~1) * 8;
    if (bar) {
      mbar_expect_tx(bar, (uint32_t)br * 80u);
      tma_load_2d(dst, &M.aq[m], bx * 64, r0, bar);
      tma_load_2d(dst + br * 64, &M.ap[m], px, r0, bar);
    } else {
      tma_prefetch_2d(&M.aq[m], bx * 64, r0);
      tma_prefetch_2d(&M.ap[m], px, r0);
    }
    return;
  }
  // GEMV unit: 16 rows x one chunk
  const DRange& R = T.r[w.ph == 0 ? 0 : (w.ph == 6 ? 4 : w.ph - 2)];
  const int u = R.u0 + w.i;
  const int tile = u / R.nch, chunk = u - tile * R.nch;
  const CUtensorMap* q;
  const CUtensorMap* p;
  int row0;
  if (w.ph == 6) {
    q = a.head_maps;
    p = q + 1;
    row0 = tile * 16;
  } else {
    const DLayerMaps& M = a.lmaps[w.l];
    const int ct = C / 16;
    const int m = w.ph == 0 ? tile / ct : w.ph;  // phases 3, 4, 5 are matrices o, ffn key, ffn value
    q = &M.q[m];
    p = &M.p[m];
    row0 = (w.ph == 0 ? tile - (tile / ct) * ct : tile) * 16;
  }
  if (bar) {
    mbar_expect_tx(bar, a.code_b + a.pair_b);
    tma_load_3d(dst, q, 0, row0, chunk * a.nb, bar);
    tma_load_2d(dst + a.code_b, p, chunk * a.pr * 8, row0, bar);
  } else {
    tma_prefetch_3d(q, 0, row0, chunk * a.nb);
    tma_prefetch_2d(p, chunk * a.pr * 8, row0);
  }
}

// Lane 0 of the producer warp: fill the ring in sequence order, gated by the
// slots' empty barriers, and keep an L2 prefetch cursor `pf_dist` stages ahead.
__device__ void d_producer(const DArgs& a, const DTable& T, uint8_t* ring, uint64_t* full, uint64_t* empty,
                           volatile int* abort_flag) {
  int seq = 0, pseq = 0;
  DWalk w{0, 0, 0, 0}, pf{0, 0, 0, 0};
  bool have = d_norm(a, T, w), pf_have = d_norm(a, T, pf);
  while (have) {
    const int slot = seq % a.nst;
    if (seq >= a.nst) {
      const uint32_t par = (uint32_t)((seq / a.nst - 1) & 1);
      uint32_t i = 0;
      bool ok = true;
      while (!mbar_try_wait(&empty[slot], par)) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        if (++i > a.spin_limit) {
          atomicOr(a.b.err, kErrTimeout);
          *abort_flag = 1;
          ok = false;
          break;
        }
      }
      if (!ok) break;
    }
    d_stage(a, T, w, ring + (size_t)slot * a.slot, &full[slot]);
    ++seq;
    ++w.i;
    have = d_norm(a, T, w);
    while (pf_have && pseq < seq + a.pf_dist) {
      if (pseq >= seq) d_stage(a, T, pf, nullptr, nullptr);
      ++pseq;
      ++pf.i;
      pf_have = d_norm(a, T, pf);
    }
  }
  // every issued copy has landed before the CTA may exit
  for (int s = seq > a.nst ? seq - a.nst : 0; s < seq; ++s)
    mbar_wait_bounded(&full[s % a.nst], (uint32_t)((s / a.nst) & 1), 1u << 20);
}

// --------------------------------------------------------------- kernel
template <int LFK>
__global__ void __launch_bounds__(kDThreads, 1) decode_kernel(DArgs a) {
  extern __shared__ __align__(1024) uint8_t d_smraw[];
  uint8_t* sm = d_smraw + ((1024u - (smem_u32(d_smraw) & 1023u)) & 1023u);
  __shared__ DTable T;
  __shared__ uint64_t full[kDMaxSt], empty[kDMaxSt];
  __shared__ float red[32];
  __shared__ int s_flag, s_tok;
  __shared__ volatile int s_abort;
  __shared__ float s_bv[kDW];
  __shared__ int s_bi[kDW];
  __shared__ float s_stat[4];  // mean / rstd of ln1 and ln2

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (t == 0) {
    d_build_table(a, T);
    for (int i = 0; i < a.nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kDW);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  if (warp == kDW) {
    if (lane == 0) d_producer(a, T, sm, full, empty, &s_abort);
    return;
  }

  // ------------------------------------------------------------ consumers
  const int C = a.d.C, F = a.d.F, H = a.d.H, G = gridDim.x, bx = blockIdx.x;
  float* X = reinterpret_cast<float*>(sm + a.o_x);    // layer input (residual stream)
  float* XB = reinterpret_cast<float*>(sm + a.o_xb);  // after attention
  float* TV = reinterpret_cast<float*>(sm + a.o_t);   // normalised vector
  float* PV = reinterpret_cast<float*>(sm + a.o_p);   // previous-token vector
  float* part = reinterpret_cast<float*>(sm + a.o_part);
  float* misc = reinterpret_cast<float*>(sm + a.o_misc);
  uint8_t* dig = sm + a.o_dig;
  const ImmaLane L = imma_lane();
  int seq = 0, pbuf = 0;
  bool dead = false;
  unsigned target = 0;
  int tr = 0;
  const int trow = bx == 0 ? 0 : (bx == G - 1 ? 1 : -1);
  auto mark = [&]() {
    if (a.trace && trow >= 0 && t == 0 && tr < a.trace_cap) a.trace[(size_t)trow * a.trace_cap + tr] = global_ns();
    ++tr;
  };
  auto csync = [&]() { bar_sync(kDBar, kDT); };
  auto csum = [&](float v) -> float {
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    csync();
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < kDW; ++w) r += red[w];
    csync();
    return r;
  };
  // grid barrier of the consumers; false (CTA-uniform) when it gave up or another wait failed
  auto gsync = [&]() -> bool {
    csync();
    target += G;
    if (t == 0) {
      bool ok = !s_abort;
      if (ok) {
        __threadfence();
        atomicAdd(a.gbar, 1u);
        ok = false;
        for (uint32_t i = 0; i < a.spin_limit; ++i) {
          if (d_ld_acquire(a.gbar) >= target) {
            ok = true;
            break;
          }
          __nanosleep(32);
        }
        if (!ok) {
          atomicOr(a.b.err, kErrTimeout);
          s_abort = 1;
        }
      }
      s_flag = ok ? 0 : 1;
    }
    csync();
    return s_flag == 0;
  };
  auto zero = [&](float* p, int i0, int i1) {
    for (int i = i0 + t; i < i1; i += kDT) p[i] = 0.f;
  };
  // dst = LayerNorm(src) over C (eps 1e-5, F.layer_norm); optionally keep mean / rstd
  auto layer_norm = [&](float* dst, const float* src, const float* w, const float* bb, float* stat) {
    float s = 0.f;
    for (int i = t; i < C; i += kDT) s += src[i];
    const float mean = csum(s) / (float)C;
    float q = 0.f;
    for (int i = t; i < C; i += kDT) {
      const float dv = src[i] - mean;
      q += dv * dv;
    }
    const float rstd = rsqrtf(csum(q) / (float)C + 1e-5f);
    for (int i = t; i < C; i += kDT) dst[i] = ln_val(src[i], mean, rstd, __ldg(w + i), __ldg(bb + i));
    if (stat && t == 0) {
      stat[0] = mean;
      stat[1] = rstd;
    }
    csync();
  };
  auto ln_at = [&](const float* src, int i, const float* stat, const float* w, const float* bb) {
    return ln_val(src[i], stat[0], stat[1], __ldg(w + i), __ldg(bb + i));
  };
  auto digits_at = [&](uint32_t off, int K) -> XDigits {
    uint8_t* base = dig + off;
    XDigits Xd;
    Xd.xd = reinterpret_cast<uint2*>(base);
    Xd.xc = reinterpret_cast<float*>(base + (size_t)K * 3);
    Xd.xsum = Xd.xc + (K >> (LFK + 5));
    return Xd;
  };
  auto build = [&](uint32_t off, int K, auto get4) { build_digits(K, LFK, get4, digits_at(off, K), t, kDT, kDBar); };
  auto f4 = [](const float* p, int i) { return *reinterpret_cast<const float4*>(p + i); };
  auto mix4 = [](float4 z, float4 p, float4 m) {
    return make_float4(z.x + (p.x - z.x) * m.x, z.y + (p.y - z.y) * m.y, z.z + (p.z - z.z) * m.z,
                       z.w + (p.w - z.w) * m.w);
  };
  // wait for the next ring slot; a warp whose wait gives up stops waiting for good
  auto slot_wait = [&]() -> const uint8_t* {
    const int slot = seq % a.nst;
    if (!dead) {
      const bool got = mbar_wait_bounded(&full[slot], (uint32_t)((seq / a.nst) & 1), a.spin_limit);
      if (!__all_sync(0xffffffffu, got)) {
        dead = true;
        if (lane == 0) {
          atomicOr(a.b.err, kErrTimeout);
          s_abort = 1;
        }
      }
    }
    return sm + (size_t)slot * a.slot;
  };
  auto slot_release = [&]() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[seq % a.nst]);
    ++seq;
  };
  // GEMV units of one phase: rows of `out` (rows_total) += W[rows, :] @ x;
  // xs[tile / per_set] is the input of a tile (per_set = 0: one input)
  auto run_units = [&](const DRange& R, const XDigits* xs, int per_set, float* out, int rows_total) {
    float acc0 = 0.f, acc1 = 0.f;
    const int kch = a.kc >> 5;
    for (int u = R.u0; u < R.u1; ++u) {
      const int tile = u / R.nch, chunk = u - tile * R.nch;
      const uint8_t* sl = slot_wait();
      if (!dead && warp < a.nb) {
        const float2* pp = reinterpret_cast<const float2*>(sl + a.code_b) + L.ra * a.pr + ((warp << 7) >> a.lg);
        imma_block<LFK>(sl + warp * 2048, pp, pp + 8 * a.pr, chunk * kch + warp * 4, xs[per_set ? tile / per_set : 0], L,
                        acc0, acc1);
      }
      slot_release();
      if (chunk == R.nch - 1 || u == R.u1 - 1) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        float* pt = part + pbuf * (kDW * 16);
        if ((lane & 3) == 0) {
          pt[warp * 16 + L.ra] = acc0;
          pt[warp * 16 + L.ra + 8] = acc1;
        }
        acc0 = acc1 = 0.f;
        csync();
        if (t < 16) {
          float v = 0.f;
          for (int w = 0; w < a.nb; ++w) v += pt[w * 16 + t];
          const int row = tile * 16 + t;
          if (row < rows_total && !dead) atomicAdd(out + row, v);
        }
        pbuf ^= 1;
      }
    }
  };

  float* acc_rkv = a.b.rkv;
  float* acc_ao = a.b.ao;
  float* acc_hk = a.b.h;
  float* acc_fo = a.b.fo;
  unsigned long long* acc_adp = a.b.adp64;
  float* logits = a.b.logits;

  // accumulators start from zero in every launch (a failed launch may leave partial sums)
  zero(acc_rkv, T.z3c0, T.z3c1);
  zero(acc_hk, T.zf0, T.zf1);
  zero(acc_ao, T.zc0, T.zc1);
  zero(acc_fo, T.zc0, T.zc1);
  zero(logits, T.zv0, T.zv1);
  for (int i = T.zr0 + t; i < T.zr1; i += kDT) acc_adp[i] = 0ull;
  int tok = a.mode == 0 ? (a.first_tok >= 0 ? a.first_tok : __ldcg(a.b.tok)) : __ldg(a.forced);
  bool alive = gsync();
  for (int step = 0; step < a.ntok && alive; ++step) {
    const bool head = a.mode == 0 || step == a.ntok - 1;
    if (a.mode == 1) tok = __ldg(a.forced + step);
    if (tok < 0 || tok >= a.d.V) {
      if (t == 0) atomicOr(a.b.err, kErrToken);
      tok = 0;
    }
    mark();  // token start
    // ---- embedding + ln0 (every CTA)
    {
      const PackedView& E = a.emb;
      if (a.emb_fast) {
        const int gpr = C >> E.lg;
        uint8_t* q = reinterpret_cast<uint8_t*>(TV);
        float2* sc = reinterpret_cast<float2*>(PV);
        for (int o = t * 16; o < C; o += kDT * 16) cp_async16(q + o, E.payload + (size_t)tok * C + o);
        for (int o = t * 16; o < gpr * 8; o += kDT * 16)
          cp_async16(reinterpret_cast<uint8_t*>(sc) + o, E.meta + (size_t)tok * gpr * 8 + o);
        cp_async_commit();
        cp_async_wait_all();
        csync();
        for (int i = t; i < C; i += kDT) {
          const float2 s = sc[i >> E.lg];
          X[i] = sg8_dequant(q[i], s.x, s.y);
        }
      } else {
        for (int i = t; i < C; i += kDT) X[i] = packed_at(E, tok, i);
      }
      csync();
      layer_norm(X, X, a.ln0_w, a.ln0_b, nullptr);
    }

    for (int l = 0; l < a.d.L && alive; ++l) {
      const LayerDev& Ly = a.layers[l];
      const float* prev_att = a.b.att_x + (size_t)l * C;
      const float* prev_ffn = a.b.ffn_x + (size_t)l * C;
      if (l > 0) {
        if (!gsync()) {
          alive = false;
          break;
        }
        for (int i = t; i < C; i += kDT) X[i] = XB[i] + __ldcg(acc_fo + i);
        csync();
      }
      mark();  // A start
      // ================= A: ln1, mixes, r/k/v rows, adapter first stages
      layer_norm(TV, X, Ly.ln1_w, Ly.ln1_b, s_stat);
      for (int i = t; i < C; i += kDT) PV[i] = __ldcg(prev_att + i);
      csync();
      build(0, C, [&](int i) { return mix4(f4(TV, i), f4(PV, i), ldg4(Ly.x_r + i)); });
      build(a.dig_set, C, [&](int i) { return mix4(f4(TV, i), f4(PV, i), ldg4(Ly.x_k + i)); });
      build(2 * a.dig_set, C, [&](int i) { return mix4(f4(TV, i), f4(PV, i), ldg4(Ly.x_v + i)); });
      mark();  // A prep done
      {
        const XDigits xs3[3] = {digits_at(0, C), digits_at(a.dig_set, C), digits_at(2 * a.dig_set, C)};
        run_units(T.r[0], xs3, C / 16, acc_rkv, 3 * C);
      }
      mark();  // A units done
      for (int k = 0; k < T.nitem[l == 0 ? 0 : 1]; ++k) {
        const int item = T.item[k];
        const int m = item / a.d.adp_splits, sp = item - m * a.d.adp_splits;
        const PackedView& W = m == 0 ? Ly.w1 : (m == 1 ? Ly.a1 : (m == 2 ? Ly.g1 : Ly.v1));
        const float* mix = m == 0 ? Ly.x_w : (m == 1 ? Ly.x_a : (m == 2 ? Ly.x_g : Ly.x_v));
        const int R = W.cols, wlg = W.lg;
        const int i0 = sp * a.d.adp_rows, i1 = min(C, i0 + a.d.adp_rows), nr = i1 - i0;
        float* xm = misc;          // [adp_rows]
        float* pacc = misc + 256;  // [nrg][R]
        for (int i = t; i < nr; i += kDT) xm[i] = TV[i0 + i] + (PV[i0 + i] - TV[i0 + i]) * __ldg(mix + i0 + i);
        csync();
        const uint8_t* sl = slot_wait();
        const int nrg = R < kDT ? kDT / R : 1;
        if (!dead) {
          const uint8_t* cq = sl;
          const uint32_t qb = (uint32_t)(nr * R);
          const float2* cs = reinterpret_cast<const float2*>(sl + ((qb + 15u) & ~15u));
          const uint32_t g0 = (uint32_t)(((uint64_t)i0 * R) >> wlg) & ~1u;
          for (int jw = t; jw < nrg * R; jw += kDT) {
            const int j = jw % R, rg = jw / R;
            float acc = 0.f;
            for (int i = rg; i < nr; i += nrg) {
              const uint32_t e = (uint32_t)(i0 + i) * (uint32_t)R + (uint32_t)j;
              const float2 sc = cs[(e >> wlg) - g0];
              acc = fmaf(xm[i], sg8_dequant(cq[i * R + j], sc.x, sc.y), acc);
            }
            pacc[rg * R + j] = acc;
          }
        }
        slot_release();
        csync();
        if (!dead) {
          const int off = d_rank_off(a.d, m);
          for (int j = t; j < R; j += kDT) {
            float v = 0.f;
            for (int rg = 0; rg < nrg; ++rg) v += pacc[rg * R + j];
            atomicAdd(acc_adp + off + j, (unsigned long long)__float2ll_rn(v * kFix));
          }
        }
        csync();
      }
      mark();  // A done
      // ================= B: one CTA per head
      const bool is_head = bx < H;
      float* S = reinterpret_cast<float*>(dig);  // [64][64] (digit sets are dead in B)
      float* mid = S + 4096;                     // [rtot]
      float* vec = mid + ((a.d.rtot + 3) & ~3);  // [4][64]
      float* sr = vec + 256;
      float* sd = sr + 64;
      float* sk = sd + 64;
      float* sv = sk + 64;
      float* skk = sv + 64;
      float* ska = skk + 64;
      float* sy = ska + 64;
      float* Sg = a.b.wkv + ((size_t)l * H + bx) * 4096;
      if (is_head) {
        for (int u = t; u < 1024; u += kDT) cp_async16(S + u * 4, Sg + u * 4);
        cp_async_commit();
      }
      if (!gsync()) {
        alive = false;
        break;
      }
      mark();  // B barrier
      zero(acc_hk, T.zf0, T.zf1);
      if (l == 0) zero(logits, T.zv0, T.zv1);
      if (is_head) {
        const int h = bx;
        const int nm = l == 0 ? 3 : 4;
        const int used = l == 0 ? a.d.rw + a.d.ra + a.d.rg : a.d.rtot;
        for (int j = t; j < used; j += kDT) {
          float v = (float)(long long)__ldcg(acc_adp + j) * kUnfix;
          if (j < a.d.rw) v = tanhf(v);
          else if (j >= a.d.rw + a.d.ra && j < a.d.rw + a.d.ra + a.d.rg) v = sigmoidf_(v);
          mid[j] = v;
        }
        float r = 0.f, k = 0.f, v = 0.f, vf = 0.f;
        if (t < 64) {
          const int ch = h * 64 + t;
          r = __ldcg(acc_rkv + ch);
          k = __ldcg(acc_rkv + C + ch);
          v = __ldcg(acc_rkv + 2 * C + ch);
          if (l != 0) vf = __ldcg(a.b.v_first + ch);
        }
        float* vp = misc;  // [5][4][64] per-thread partials
        for (int i = t; i < 5 * 256; i += kDT) vp[i] = 0.f;
        cp_async_wait_all();
        csync();
        {
          const int c = t & 63, q = t >> 6;  // 5 row phases x 64 columns
          for (int pc = 0; pc < T.npc[l == 0 ? 0 : 1]; ++pc) {
            const uint8_t* sl = slot_wait();
            if (!dead) {
              const int m = T.pm[pc], br = a.abr[m], r0 = T.pr0[pc];
              const int nr = min(br, d_rank(a.d, m) - r0);
              const float2* pairs = reinterpret_cast<const float2*>(sl + br * 64);
              const int sel = ((h * 64) >> a.alg[m]) & 1;
              const float* mm = mid + d_rank_off(a.d, m) + r0;
              float acc = 0.f;
              for (int i = q; i < nr; i += 5) {
                const float2 pq = pairs[i * 2 + sel];
                acc = fmaf(mm[i], sg8_dequant(sl[i * 64 + c], pq.x, pq.y), acc);
              }
              vp[(q * 4 + m) * 64 + c] += acc;
            }
            slot_release();
          }
        }
        csync();
        if (t < 256) {
          const int m = t >> 6, c = t & 63;
          float s = 0.f;
          if (m < nm)
            for (int q = 0; q < 5; ++q) s += vp[(q * 4 + m) * 64 + c];
          vec[m * 64 + c] = s;
        }
        csync();
        const float kkv = t < 64 ? k * __ldg(Ly.k_k + h * 64 + t) : 0.f;
        const float nrm = sqrtf(csum(kkv * kkv));
        if (t < 64) {
          const int ch = h * 64 + t;
          const float aa = sigmoidf_(__ldg(Ly.a0 + ch) + vec[64 + t]);
          const float kk = kkv / fmaxf(nrm, 1e-12f);
          const float kn = k * (1.0f + (aa - 1.0f) * __ldg(Ly.k_a + ch));
          if (l == 0) a.b.v_first[ch] = v;
          else v = v + (vf - v) * sigmoidf_(__ldg(Ly.v0 + ch) + vec[192 + t]);
          sr[t] = r;
          sd[t] = expf(-0.606531f * sigmoidf_(__ldg(Ly.w0 + ch) + vec[t]));
          sk[t] = kn;
          sv[t] = v;
          skk[t] = kk;
          ska[t] = kk * aa;
        }
        csync();
        if (t < 256) wkv7_head64(S, sr, sd, sk, sv, skk, ska, sy);
        csync();
        for (int u = t; u < 1024; u += kDT) reinterpret_cast<float4*>(Sg)[u] = reinterpret_cast<const float4*>(S)[u];
        const float yv = t < 64 ? sy[t] : 0.f;
        const float mean = csum(yv) / 64.f;
        const float dv = t < 64 ? yv - mean : 0.f;
        const float var = csum(dv * dv) / 64.f;
        const float bon = t < 64 ? sr[t] * sk[t] * __ldg(Ly.r_k + h * 64 + t) : 0.f;
        const float bonus = csum(bon);
        if (t < 64) {
          const int ch = h * 64 + t;
          float o = dv * rsqrtf(var + 64e-5f) * __ldg(Ly.lnx_w + ch) + __ldg(Ly.lnx_b + ch);
          o = o + bonus * sv[t];
          a.b.att_y[ch] = o * vec[128 + t];
        }
      }
      mark();  // B done
      if (!gsync()) {
        alive = false;
        break;
      }
      mark();  // C barrier
      // ================= C: output projection; att_x[l] <- ln1 slice
      zero(acc_fo, T.zc0, T.zc1);
      for (int i = T.zc0 + t; i < T.zc1; i += kDT)
        a.b.att_x[(size_t)l * C + i] = ln_at(X, i, s_stat, Ly.ln1_w, Ly.ln1_b);
      build(0, C, [&](int i) { return ldcg4(a.b.att_y + i); });
      mark();  // C prep done
      {
        const XDigits x1 = digits_at(0, C);
        run_units(T.r[1], &x1, 0, acc_ao, C);
      }
      mark();  // C done
      if (!gsync()) {
        alive = false;
        break;
      }
      mark();  // D barrier
      // ================= D: x += att; ln2 + mix; ffn key rows
      zero(acc_rkv, T.z3c0, T.z3c1);
      for (int i = T.zr0 + t; i < T.zr1; i += kDT) acc_adp[i] = 0ull;
      for (int i = t; i < C; i += kDT) {
        XB[i] = X[i] + __ldcg(acc_ao + i);
        PV[i] = __ldcg(prev_ffn + i);
      }
      csync();
      layer_norm(TV, XB, Ly.ln2_w, Ly.ln2_b, s_stat + 2);
      build(0, C, [&](int i) { return mix4(f4(TV, i), f4(PV, i), ldg4(Ly.ffn_x_k + i)); });
      mark();  // D prep done
      {
        const XDigits x1 = digits_at(0, C);
        run_units(T.r[2], &x1, 0, acc_hk, F);
      }
      mark();  // D done
      if (!gsync()) {
        alive = false;
        break;
      }
      mark();  // E barrier
      // ================= E: relu^2; ffn value rows; ffn_x[l] <- ln2 slice
      zero(acc_ao, T.zc0, T.zc1);
      for (int i = T.zc0 + t; i < T.zc1; i += kDT)
        a.b.ffn_x[(size_t)l * C + i] = ln_at(XB, i, s_stat + 2, Ly.ln2_w, Ly.ln2_b);
      build(0, F, [&](int i) {
        const float4 v = ldcg4(acc_hk + i);
        return make_float4(v.x > 0.f ? v.x * v.x : 0.f, v.y > 0.f ? v.y * v.y : 0.f, v.z > 0.f ? v.z * v.z : 0.f,
                           v.w > 0.f ? v.w * v.w : 0.f);
      });
      mark();  // E prep done
      {
        const XDigits x1 = digits_at(0, F);
        run_units(T.r[3], &x1, 0, acc_fo, C);
      }
      mark();  // E done
    }
    if (!alive) break;
    if (!head) continue;
    // ================= head: ln_out, logits, argmax (first maximum)
    if (!gsync()) {
      alive = false;
      break;
    }
    mark();  // head barrier
    zero(acc_hk, T.zf0, T.zf1);
    for (int i = t; i < C; i += kDT) PV[i] = XB[i] + __ldcg(acc_fo + i);
    csync();
    layer_norm(TV, PV, a.lnout_w, a.lnout_b, nullptr);
    build(0, C, [&](int i) { return f4(TV, i); });
    mark();  // head prep done
    {
      const XDigits x1 = digits_at(0, C);
      run_units(T.r[4], &x1, 0, logits, a.d.V);
    }
    mark();  // head done
    if (!gsync()) {
      alive = false;
      break;
    }
    zero(acc_fo, T.zc0, T.zc1);
    {
      float best = -INFINITY;
      int besti = 0x7fffffff;
      for (int i = T.zv0 + t; i < T.zv1; i += kDT) {
        const float v = __ldcg(logits + i);
        if (v > best) {
          best = v;
          besti = i;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) {
          best = ov;
          besti = oi;
        }
      }
      if (lane == 0) {
        s_bv[warp] = best;
        s_bi[warp] = besti;
      }
      csync();
      if (t == 0) {
        float cb = -INFINITY;
        int ci = 0x7fffffff;
        for (int w = 0; w < kDW; ++w)
          if (s_bv[w] > cb || (s_bv[w] == cb && s_bi[w] < ci)) {
            cb = s_bv[w];
            ci = s_bi[w];
          }
        a.b.amax_v[bx] = cb;
        a.b.amax_i[bx] = ci;
      }
    }
    if (!gsync()) {
      alive = false;
      break;
    }
    if (t < 32) {
      float gb = -INFINITY;
      int gi = 0x7fffffff;
      for (int c = lane; c < G; c += 32) {
        const float v = __ldcg(a.b.amax_v + c);
        const int i = __ldcg(a.b.amax_i + c);
        if (v > gb || (v == gb && i < gi)) {
          gb = v;
          gi = i;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, gb, o);
        const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
        if (ov > gb || (ov == gb && oi < gi)) {
          gb = ov;
          gi = oi;
        }
      }
      if (t == 0) s_tok = gi == 0x7fffffff ? 0 : gi;
    }
    csync();
    tok = s_tok;
    if (bx == 0 && t == 0) {
      a.b.hist[step % a.d.hist_cap] = tok;
      *a.b.tok = tok;
    }
  }
}

}  // namespace rwkvb
