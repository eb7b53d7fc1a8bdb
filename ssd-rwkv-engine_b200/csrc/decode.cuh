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
// FFN value rows in column-chunk order (the default): E's units are numbered
// chunk by chunk, so each CTA's range covers one or two KC-column chunks and
// it builds the digits of only those chunks of relu^2(k) instead of the whole
// FFN-wide vector; a row then receives one partial per chunk, accumulated in
// 2^-32 fixed point with 64-bit integer adds (exact: independent of order).
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
constexpr int kDRingDefault = 3;       // ring slots unless the engine flags ask for more
constexpr int kDBar = 1;               // named barrier of the consumers
constexpr int kDMaxItems = 8;          // adapter first-stage items per CTA
constexpr int kDPartTiles = 16;        // GEMV tiles whose per-warp partial sums are buffered per CTA reduction
constexpr uint32_t kDPartBytes = kDPartTiles * kDW * 16 * 4 + 128;  // the partial sums, then their tile indices
constexpr int kDMaxPieces = 8;         // adapter second-stage tile pieces per layer
constexpr int kDPieceSteps = 2;        // preload mode: 32-row k-steps per phase-B tensor-core task
constexpr int kDMaxChunks = 16;        // preload mode: k-step chunks over the four adapters
constexpr int kDMisc = 2560;           // misc shared floats
static_assert((kDW / 2) * 4 * 64 <= kDMisc, "phase-B adapter partials [warps / 2][4][64] live in misc");
static_assert(256 + 4 * kDT <= kDMisc, "adapter item inputs and row-group partials live in misc");
constexpr int kMidPer = (2048 + kDT - 1) / kDT;  // first-adapter sums per consumer thread (rtot <= 2048)
// Preload-mode phase B keeps in misc: the min-term partials of the 8-row
// items (rt / 8 floats), the digit blocks of the four adapters (3.25 bytes per
// row), the task partials [4 nchunk][16], the adapter biases [4].
__host__ __device__ constexpr int d_pieces_misc_floats(int rt, int nchunk) { return rt / 8 + rt * 13 / 16 + 64 * nchunk + 4; }
constexpr float kFix = 4294967296.0f;  // 2^32 fixed-point scale of adapter partials
constexpr float kUnfix = 1.0f / 4294967296.0f;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long v;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(v));
  return v;
}

__device__ __forceinline__ int d_ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void d_st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Fire-and-forget 64-bit integer add (the fixed-point accumulators).
__device__ __forceinline__ void red_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
// Grid-barrier arrival: the release orders every write this CTA made before
// its preceding CTA barrier ahead of the count.
__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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
  // streaming copy (null: load through the tensor maps): r/k/v (one region of
  // 3C rows), o, ffn key, ffn value, each unit-major, a unit stored as the
  // shared-memory image of its ring slot
  const uint8_t* su[4];
  // preload mode: this layer's adapter second-stage images, one per head
  // (adp_b0 bytes on layer 0, adp_b1 on later layers): per adapter m (w, a,
  // g, v) its R_m rows of the head's 64 columns, then the rows' two (min, max)
  // pairs around those columns ([R_m][64] codes, [R_m][2] float2)
  const uint8_t* ai;
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
  int nst;  // ring slots
  uint32_t slot, code_b, pair_b;
  int abr[4];  // adapter second stage: box rows per matrix
  int alg[4];  // adapter second stage: log2 group
  int ntok, mode, first_tok;  // mode 0 greedy (step 0 consumes first_tok, -1: *tok), 1 forced tokens
  const int* forced;
  unsigned* gbar;
  uint32_t spin_limit;
  int emb_fast;
  int l2_first;  // weight stream loaded with the L2 evict-first policy
  unsigned long long* trace;
  int trace_cap;
  uint32_t o_dig, o_x, o_xb, o_t, o_p, o_part, o_misc, smem_total;
  uint32_t dig_set;  // bytes of one digit set of width C
  // streamed greedy decode (mode 0; all null otherwise): mapped pinned host
  // memory that receives each step's id (ring_ids[step], then ring_count =
  // step + 1) and holds the host's cancel word, read between tokens
  int* ring_ids;
  unsigned* ring_count;
  const int* ring_cancel;
  const uint8_t* head_su;  // streaming copy of the head (null with the tensor maps)
  // preload mode (pre != 0): the phase-B adapter image (head CTAs) and the
  // adapter first-stage item (at most one per CTA) of each layer land in
  // dedicated shared memory at the start of the layer instead of ring slots
  int pre;
  uint32_t o_adp, o_item, adp_b0, adp_b1;
  // preload images of the adapter second stages, per adapter m (w, a, g, v):
  // codes transposed, [64 columns][aps[m] bytes] (row = one output column,
  // its apr[m] = rank rounded up to 32 codes, zero-padded), then the rows'
  // (min, max) pair of pairs [apr[m]][16 B]
  int aps[4], apr[4];
  // FFN value rows in column-chunk order with fixed-point accumulation (0:
  // row order, fp32 atomics)
  int ecm;
};

struct DTable {
  DRange r[5];    // r/k/v (3C rows), o, ffn key, ffn value, head
  int nitem[2];   // adapter first-stage items: layer 0 (no v1), other layers
  int item[kDMaxItems];
  int npc[2];     // adapter second-stage pieces: layer 0 (no v2), other layers; 0 unless a head CTA
  int pm[kDMaxPieces], pr0[kDMaxPieces];
  // preload mode: phase B's k-step chunks (adapter, first k-step), v last
  int nck[2];     // layer 0 (no v2), other layers
  int ckm[kDMaxChunks], cks[kDMaxChunks];
  int zc0, zc1, zf0, zf1, z3c0, z3c1, zv0, zv1, zr0, zr1;  // zeroing slices (C, F, 3C, V, rtot)
  int ech0, ech1;  // chunk-ordered E: first and last column chunk of this CTA's units
  uint32_t aneed;  // bit m: this CTA has r/k/v units of matrix m (r, k, v), so phase A builds its digits
};

// [a, b) = part i of [0, n) split into `parts` (n * parts < 2^32).
__device__ __noinline__ void d_split(int n, int parts, int i, int* a, int* b) {
  *a = (int)((unsigned)n * (unsigned)i / (unsigned)parts);
  *b = (int)((unsigned)n * (unsigned)(i + 1) / (unsigned)parts);
}

__device__ __forceinline__ void d_range(int tiles, int nch, int G, int b, DRange& R, bool whole = false) {
  const int U = tiles * nch;
  R.nch = nch;
  if (!whole && U / G >= nch - 1) {  // every range spans >= nch - 1 units: a tile meets at most two CTAs
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

// Adapter (0 w, 1 a, 2 g, 3 v) of first-stage item `item`.
__device__ __forceinline__ int d_item_mat(const Dims& d, int item) {
  int m = 0;
  while (m < 3 && item >= d.abase[m + 1]) ++m;
  return m;
}

__device__ __forceinline__ int d_rank_off(const Dims& d, int m) {
  return m == 0 ? 0 : (m == 1 ? d.rw : (m == 2 ? d.rw + d.ra : d.rw + d.ra + d.rg));
}

__device__ void d_build_table(const DArgs& a, DTable& T) {
  const int G = gridDim.x, bx = blockIdx.x, C = a.d.C, F = a.d.F;
  const int nc = C / a.kc, nf = F / a.kc;
  d_range(3 * C / 16, nc, G, bx, T.r[0]);
  d_range(C / 16, nc, G, bx, T.r[1]);
  T.aneed = 0u;
  for (int u = T.r[0].u0; u < T.r[0].u1; ++u) T.aneed |= 1u << (u / nc / (C / 16));
  d_range(F / 16, nc, G, bx, T.r[2]);
  if (a.ecm) {  // chunk order: equal contiguous shares of the chunk-major unit numbering
    T.r[3].nch = nf;
    d_split(C / 16 * nf, G, bx, &T.r[3].u0, &T.r[3].u1);
    T.ech0 = T.r[3].u0 / (C / 16);
    T.ech1 = T.r[3].u1 > T.r[3].u0 ? (T.r[3].u1 - 1) / (C / 16) : T.ech0;
  } else {
    d_range(C / 16, nf, G, bx, T.r[3]);
    T.ech0 = 0;
    T.ech1 = nf - 1;
  }
  d_range((a.d.V + 15) / 16, nc, G, bx, T.r[4]);
  const int items3 = a.d.abase[3], items4 = a.d.abase[4];
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
  {
    int n = 0;
    T.nck[0] = 0;
    for (int m = 0; m < 4; ++m) {
      if (m == 3) T.nck[0] = n;
      for (int s0 = 0; s0 < a.apr[m] / 32 && n < kDMaxChunks; s0 += kDPieceSteps) {
        T.ckm[n] = m;
        T.cks[n] = s0;
        ++n;
      }
    }
    T.nck[1] = n;
  }
  d_split(C, G, bx, &T.zc0, &T.zc1);
  d_split(F, G, bx, &T.zf0, &T.zf1);
  d_split(3 * C, G, bx, &T.z3c0, &T.z3c1);
  d_split(a.d.V, G, bx, &T.zv0, &T.zv1);
  d_split(a.d.rtot, G, bx, &T.zr0, &T.zr1);
}

// ------------------------------------------------------------- producer
// Bring layer l's small operands into L2: its fp32 vectors, this layer's rows
// of the token-shift state and (head CTAs) this CTA's WKV state.  They are
// read after the weight stream has evicted them, on the latency-bound path
// between phases.
__device__ void d_prefetch_layer(const DArgs& a, int l) {
  const LayerDev& Ly = a.layers[l];
  const uint32_t vb = (uint32_t)a.d.C * 4u;
  const float* vecs[19] = {Ly.ln1_w, Ly.ln1_b, Ly.ln2_w, Ly.ln2_b, Ly.x_r, Ly.x_w, Ly.x_k, Ly.x_v, Ly.x_a, Ly.x_g,
                           Ly.w0,    Ly.a0,    Ly.v0,    Ly.k_k,   Ly.k_a, Ly.r_k, Ly.lnx_w, Ly.lnx_b, Ly.ffn_x_k};
  for (int i = 0; i < 19; ++i)
    if (vecs[i] && (i != 12 || l > 0)) prefetch_l2_bulk(vecs[i], vb);
  prefetch_l2_bulk(a.b.att_x + (size_t)l * a.d.C, vb);
  prefetch_l2_bulk(a.b.ffn_x + (size_t)l * a.d.C, vb);
  if ((int)blockIdx.x < a.d.H) prefetch_l2_bulk(a.b.wkv + ((size_t)l * a.d.H + blockIdx.x) * 4096, 16384u);
}

__device__ __forceinline__ void d_prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// Producer: the ring slot of stage `seq` once it is free; -1 when the launch
// is aborting (another wait gave up) or this wait gave up.
__device__ __noinline__ int d_acquire(const DArgs& a, uint64_t* empty, volatile int* abort_flag, int seq) {
  const int slot = seq % a.nst;
  if (seq >= a.nst) {
    const uint32_t par = (uint32_t)((seq / a.nst - 1) & 1);
    if (mbar_try_wait_hint(&empty[slot], par, 20000u)) return slot;  // no wall-clock read on the common path
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait_hint(&empty[slot], par, 20000u)) {  // suspended, not spinning, while the ring is full
      if (*abort_flag) return -1;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(a.b.err, kErrTimeout);
        *abort_flag = 1;
        return -1;
      }
    }
  }
  return slot;
}

__device__ __forceinline__ void d_issued(const DArgs& a, int& seq) {
  if (a.trace && blockIdx.x == 0 && 3 * seq + 2 < 2 * a.trace_cap) a.trace[2 * (size_t)a.trace_cap + 3 * seq] = global_ns();
  ++seq;
}

// Producer: GEMV units [R.u0, R.u1); per_map > 0: tile t uses map t / per_map
// (the r, k, v maps of phase A), row (t % per_map) * 16.  Every argument the
// loop needs is copied to registers first (the loop stores to shared memory,
// so reads through `a` would be repeated each iteration).
// su != null: unit u is one bulk copy of its slot image from the streaming
// copy (a single TMA operation per unit instead of a code box and a pair box).
__device__ __noinline__ bool d_issue_units(const DArgs& a, const DRange& R, const CUtensorMap* q, const CUtensorMap* p,
                                           int per_map, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                           volatile int* abort_flag, int& seq_io, const uint8_t* su, int tiles_cm) {
  const int nst = a.nst, nb = a.nb, pr8 = a.pr * 8, u0 = R.u0, u1 = R.u1, nch = R.nch;
  const uint32_t slot_b = a.slot, code_b = a.code_b, bytes = a.code_b + a.pair_b;
  unsigned long long* tr = (a.trace && blockIdx.x == 0) ? a.trace + 2 * (size_t)a.trace_cap : nullptr;
  const int tr_n = 2 * a.trace_cap;
  int seq = seq_io;
  const bool hint = a.l2_first != 0;
  const uint64_t pol = l2_evict_first();
  // unit u: (tile, chunk) = (u / nch, u % nch), or chunk-major (u % tiles_cm, u / tiles_cm)
  int tile = tiles_cm ? u0 % tiles_cm : u0 / nch, chunk = tiles_cm ? u0 / tiles_cm : u0 - tile * nch;
  int mi = per_map ? tile / per_map : 0, row0 = (tile - mi * per_map) * 16;
  bool ok = true;
  // ring position of stage seq, advanced incrementally: a division by the
  // runtime depth per unit is a long dependent chain on the issue path
  int slot = seq % nst;
  uint32_t par = (uint32_t)((seq / nst - 1) & 1);  // parity of the release this stage waits for
#pragma unroll 1
  for (int u = u0; u < u1; ++u) {
    if (seq >= nst) {
      uint64_t t0 = 0;  // the wall clock is read only once a wait has not ended at the first poll
      while (!mbar_try_wait_hint(&empty[slot], par, 20000u)) {
        if (t0 == 0) t0 = globaltimer_ns();
        if (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs) {
          if (!*abort_flag) {
            atomicOr(a.b.err, kErrTimeout);
            *abort_flag = 1;
          }
          ok = false;
          break;
        }
      }
      if (!ok) break;
    }
    uint8_t* dst = ring + (size_t)slot * slot_b;
    mbar_expect_tx(&full[slot], bytes);
    if (su) {
      const uint8_t* src = su + (size_t)(tile * nch + chunk) * bytes;  // images are stored tile by tile
      if (hint) bulk_g2s_hint(dst, src, bytes, &full[slot], pol);
      else bulk_g2s(dst, src, bytes, &full[slot]);
    } else if (hint) {
      tma_load_3d_hint(dst, q + mi, 0, row0, chunk * nb, &full[slot], pol);
      tma_load_2d_hint(dst + code_b, p + mi, chunk * pr8, row0, &full[slot], pol);
    } else {
      tma_load_3d(dst, q + mi, 0, row0, chunk * nb, &full[slot]);
      tma_load_2d(dst + code_b, p + mi, chunk * pr8, row0, &full[slot]);
    }
    if (tr && 3 * seq + 2 < tr_n) tr[3 * seq] = global_ns();
    ++seq;
    if (++slot == nst) {
      slot = 0;
      par ^= 1u;
    }
    if (tiles_cm) {
      row0 += 16;
      if (++tile == tiles_cm) {
        tile = 0;
        row0 = 0;
        ++chunk;
      }
    } else if (++chunk == nch) {
      chunk = 0;
      ++tile;
      row0 += 16;
      if (per_map && row0 == per_map * 16) {
        row0 = 0;
        ++mi;
      }
    }
  }
  seq_io = seq;
  return ok;
}

// One adapter first-stage item (rows [i0, i1) of W1 [C][R] and the (min, max)
// pairs of the groups they touch) into `dst`, completing on `bar`.
__device__ __noinline__ void d_issue_item(const DArgs& a, const LayerDev& Ly, int item, uint8_t* dst, uint64_t* bar) {
  const int m = d_item_mat(a.d, item);
  const PackedView& W = m == 0 ? Ly.w1 : (m == 1 ? Ly.a1 : (m == 2 ? Ly.g1 : Ly.v1));
  const int R = W.cols, C = a.d.C;
  const int i0 = (item - a.d.abase[m]) * a.d.arow[m], i1 = min(C, i0 + a.d.arow[m]);
  const uint32_t qb = (uint32_t)((i1 - i0) * R);
  const uint32_t g0 = (uint32_t)(((uint64_t)i0 * R) >> W.lg) & ~1u;
  const uint32_t g1 = ((uint32_t)((((uint64_t)i1 * R - 1) >> W.lg) + 1) + 1u) & ~1u;
  const uint32_t sb = (g1 - g0) * 8u;
  // the item's slice of its token-shift mix vector follows the pairs, so the
  // consumers mix the item's inputs from shared memory only
  const float* mix = m == 0 ? Ly.x_w : (m == 1 ? Ly.x_a : (m == 2 ? Ly.x_g : Ly.x_v));
  const uint32_t xb = (uint32_t)(i1 - i0) * 4u;
  const uint32_t xo = ((qb + 15u) & ~15u) + sb;
  mbar_expect_tx(bar, qb + sb + xb);
  if (a.l2_first) {
    const uint64_t pol = l2_evict_first();
    bulk_g2s_hint(dst, W.payload + (size_t)i0 * R, qb, bar, pol);
    bulk_g2s_hint(dst + ((qb + 15u) & ~15u), W.meta + (size_t)g0 * 8, sb, bar, pol);
  } else {
    bulk_g2s(dst, W.payload + (size_t)i0 * R, qb, bar);
    bulk_g2s(dst + ((qb + 15u) & ~15u), W.meta + (size_t)g0 * 8, sb, bar);
  }
  bulk_g2s(dst + xo, mix + i0, xb, bar);  // re-read every token: default L2 policy
}

// Producer: wait until the consumers released load n - 1 of a dedicated
// buffer (its "empty" barrier); false when the launch aborts or the wait
// gives up.
__device__ __noinline__ bool d_pre_acquire(const DArgs& a, uint64_t* empty, int n, volatile int* abort_flag) {
  if (n == 0) return true;
  const uint32_t par = (uint32_t)((n - 1) & 1);
  if (mbar_try_wait_hint(empty, par, 20000u)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_hint(empty, par, 20000u)) {
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(a.b.err, kErrTimeout);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// Lane 0 of the producer warp: fill the ring in the consumers' order (per
// token, per layer: r/k/v units, adapter items, adapter-2 pieces, o units,
// ffn key units, ffn value units; then the head units), gated by the slots'
// empty barriers.  When it starts a layer it prefetches the next layer's small
// operands and this layer's tensor maps.
__device__ void d_producer(const DArgs& a, const DTable& T, uint8_t* ring, uint64_t* full, uint64_t* empty,
                           volatile int* abort_flag, uint64_t* pbar) {
  int seq = 0;
  int nadp = 0, nitm = 0;  // dedicated-buffer loads issued (preload mode)
  const bool hint = a.l2_first != 0;
  const uint64_t pol = l2_evict_first(), keep = l2_evict_last();
  auto acquire = [&]() -> int { return d_acquire(a, empty, abort_flag, seq); };
  auto issued = [&]() { d_issued(a, seq); };
  auto layer_start = [&](int l) {
    const DLayerMaps& M = a.lmaps[l];
    for (int m = 0; m < 6; ++m) {
      d_prefetch_map(&M.q[m]);
      d_prefetch_map(&M.p[m]);
    }
    if ((int)blockIdx.x < a.d.H)
      for (int m = 0; m < 4; ++m) {
        d_prefetch_map(&M.aq[m]);
        d_prefetch_map(&M.ap[m]);
      }
    d_prefetch_layer(a, l + 1 < a.d.L ? l + 1 : 0);
  };
  d_prefetch_layer(a, 0);
  {
    const int C = a.d.C, ct = C / 16, bx = blockIdx.x;
    bool ok = true;
    auto units = [&](const DRange& R, const CUtensorMap* q, const CUtensorMap* p, int per_map,
                     const uint8_t* su, int tiles_cm = 0) -> bool {
      return d_issue_units(a, R, q, p, per_map, ring, full, empty, abort_flag, seq, su, tiles_cm);
    };
    for (int tok = 0; tok < a.ntok && ok; ++tok) {
      const bool head = a.mode == 0 || tok == a.ntok - 1;
      for (int l = 0; l < a.d.L && ok; ++l) {
        const DLayerMaps& M = a.lmaps[l];
        const LayerDev& Ly = a.layers[l];
        layer_start(l);
        if (a.pre) {
          // phase-B image and the item first: they land while phase A runs
          if (bx < a.d.H) {
            ok = d_pre_acquire(a, &pbar[1], nadp, abort_flag);
            if (ok) {
              const uint32_t b = l == 0 ? a.adp_b0 : a.adp_b1;
              mbar_expect_tx(&pbar[0], b);
              if (hint) bulk_g2s_hint(ring + a.o_adp, M.ai + (size_t)bx * b, b, &pbar[0], pol);
              else bulk_g2s(ring + a.o_adp, M.ai + (size_t)bx * b, b, &pbar[0]);
              ++nadp;
            }
          }
          if (ok && T.nitem[l == 0 ? 0 : 1] > 0) {
            ok = d_pre_acquire(a, &pbar[3], nitm, abort_flag);
            if (ok) {
              d_issue_item(a, Ly, T.item[0], ring + a.o_item, &pbar[2]);
              ++nitm;
            }
          }
        }
        if (ok) ok = units(T.r[0], M.q, M.p, ct, M.su[0]);
        for (int k = 0; ok && !a.pre && k < T.nitem[l == 0 ? 0 : 1]; ++k) {
          const int item = T.item[k];
          const int m = d_item_mat(a.d, item);
          const PackedView& W = m == 0 ? Ly.w1 : (m == 1 ? Ly.a1 : (m == 2 ? Ly.g1 : Ly.v1));
          const int R = W.cols;
          const int i0 = (item - a.d.abase[m]) * a.d.arow[m], i1 = min(C, i0 + a.d.arow[m]);
          const uint32_t qb = (uint32_t)((i1 - i0) * R);
          const uint32_t g0 = (uint32_t)(((uint64_t)i0 * R) >> W.lg) & ~1u;
          const uint32_t g1 = ((uint32_t)((((uint64_t)i1 * R - 1) >> W.lg) + 1) + 1u) & ~1u;
          const uint32_t sb = (g1 - g0) * 8u;
          const int slot = acquire();
          ok = slot >= 0;
          if (ok) {
            uint8_t* dst = ring + (size_t)slot * a.slot;
            mbar_expect_tx(&full[slot], qb + sb);
            if (hint) {
              bulk_g2s_hint(dst, W.payload + (size_t)i0 * R, qb, &full[slot], pol);
              bulk_g2s_hint(dst + ((qb + 15u) & ~15u), W.meta + (size_t)g0 * 8, sb, &full[slot], pol);
            } else {
              bulk_g2s(dst, W.payload + (size_t)i0 * R, qb, &full[slot]);
              bulk_g2s(dst + ((qb + 15u) & ~15u), W.meta + (size_t)g0 * 8, sb, &full[slot]);
            }
            issued();
          }
        }
        for (int k = 0; ok && !a.pre && k < T.npc[l == 0 ? 0 : 1]; ++k) {
          const int m = T.pm[k], br = a.abr[m];
          const int slot = acquire();
          ok = slot >= 0;
          if (ok) {
            uint8_t* dst = ring + (size_t)slot * a.slot;
            mbar_expect_tx(&full[slot], (uint32_t)br * 80u);
            const int px = (((bx * 64) >> a.alg[m]) & ~1) * 8;
            if (hint) {  // phase B waits on these: keep them in L2 across tokens
              tma_load_2d_hint(dst, &M.aq[m], bx * 64, T.pr0[k], &full[slot], keep);
              tma_load_2d_hint(dst + br * 64, &M.ap[m], px, T.pr0[k], &full[slot], keep);
            } else {
              tma_load_2d(dst, &M.aq[m], bx * 64, T.pr0[k], &full[slot]);
              tma_load_2d(dst + br * 64, &M.ap[m], px, T.pr0[k], &full[slot]);
            }
            issued();
          }
        }
        if (ok) ok = units(T.r[1], M.q + 3, M.p + 3, 0, M.su[1]);
        if (ok) ok = units(T.r[2], M.q + 4, M.p + 4, 0, M.su[2]);
        if (ok) ok = units(T.r[3], M.q + 5, M.p + 5, 0, M.su[3], a.ecm ? C / 16 : 0);
      }
      if (ok && head) {
        d_prefetch_map(a.head_maps);
        d_prefetch_map(a.head_maps + 1);
        ok = units(T.r[4], a.head_maps, a.head_maps + 1, 0, a.head_su);
      }
    }
  }
  // every issued copy has landed before the CTA may exit
  for (int s = seq > a.nst ? seq - a.nst : 0; s < seq; ++s)
    mbar_wait_bounded(&full[s % a.nst], (uint32_t)((s / a.nst) & 1), 1u << 20);
  if (nadp > 0) mbar_wait_bounded(&pbar[0], (uint32_t)((nadp - 1) & 1), 1u << 20);
  if (nitm > 0) mbar_wait_bounded(&pbar[2], (uint32_t)((nitm - 1) & 1), 1u << 20);
}

// ------------------------------------------------------------ consumers
// The consumer side is a set of non-inlined subroutines shared by all phases
// (one digit builder, one GEMV unit loop, one LayerNorm, ...), so the code a
// layer executes stays small enough to remain in the instruction caches while
// the weight stream sweeps L2.

// Consumer state shared by the subroutines: one copy per consumer warp in
// shared memory (the same values on every lane).  Kept in local memory it
// would be re-read from L2 after every phase: the carve-out leaves the SM a
// small L1, which the phase's vector loads sweep.
struct DCons {
  uint8_t* sm;  // 1024-aligned dynamic shared memory (ring at offset 0)
  uint64_t* full;
  uint64_t* empty;
  float* red;  // [32] reduction scratch
  volatile int* abort;
  int* flag;
  int seq, pbuf, dead, tr, trow;
  unsigned target;
  uint64_t* pbar;  // preload mode: adp full/empty, item full/empty
  int nadp, nitm;  // dedicated-buffer loads consumed
};

// Warp-uniform update of a field of the warp's DCons: every lane reads the
// old value (the argument) before lane 0 stores the new one.
template <typename T>
__device__ __forceinline__ void d_wset(T& f, T v) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) f = v;
  __syncwarp();
}

// Consumers: wait for a dedicated-buffer load (all threads); a failed wait
// marks this CTA dead like a ring wait.
__device__ __forceinline__ void d_pre_wait(const DArgs& a, DCons& c, uint64_t* full, int n) {
  if (c.dead) return;
  const bool got = mbar_wait_suspend(full, (uint32_t)(n & 1));
  if (!__all_sync(0xffffffffu, got)) {
    c.dead = 1;
    if ((threadIdx.x & 31) == 0) {
      atomicOr(a.b.err, kErrTimeout);
      *c.abort = 1;
    }
  }
}

__device__ __forceinline__ void d_csync() { bar_sync(kDBar, kDT); }

__device__ __forceinline__ void d_mark(const DArgs& a, DCons& c) {
  if (a.trace && c.trow >= 0 && threadIdx.x == 0 && c.tr < a.trace_cap)
    a.trace[(size_t)c.trow * a.trace_cap + c.tr] = global_ns();
  d_wset(c.tr, c.tr + 1);
}

// Sum over the consumer threads (all of them get the result).
__device__ __noinline__ float d_csum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  d_csync();
  float r = 0.f;
#pragma unroll
  for (int w = 0; w < kDW; ++w) r += red[w];
  d_csync();
  return r;
}

// Sums over the 64 threads of warps 0 and 1 only (a head's channels): warp
// shuffles, one 64-thread named barrier; `red` gets two (or four) fresh
// floats per call so that successive calls do not race.
constexpr int kDBar64 = 3;  // named barrier of warps 0-1
__device__ __forceinline__ float d_sum64(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  bar_sync(kDBar64, 64);
  return red[0] + red[1];
}
__device__ __forceinline__ float2 d_sum64x2(float v, float w, float* red) {
  v = warp_sum(v);
  w = warp_sum(w);
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = v;
    red[2 + (threadIdx.x >> 5)] = w;
  }
  bar_sync(kDBar64, 64);
  return make_float2(red[0] + red[1], red[2] + red[3]);
}

// Grid barrier of the consumers; false (CTA-uniform) when it gave up or an
// earlier wait of this CTA failed.
__device__ __noinline__ bool d_gsync(const DArgs& a, DCons& c) {
  d_csync();
  d_wset(c.target, c.target + gridDim.x);
  if (threadIdx.x == 0) {
    bool ok = !*c.abort;
    if (ok) {
      red_release_add_u32(a.gbar, 1u);
      ok = false;
      for (uint32_t i = 0; i < a.spin_limit; ++i) {
        if (d_ld_acquire(a.gbar) >= c.target) {
          ok = true;
          break;
        }
        __nanosleep(32);
      }
      if (!ok) {
        atomicOr(a.b.err, kErrTimeout);
        *c.abort = 1;
      }
    }
    *c.flag = ok ? 0 : 1;
  }
  d_csync();
  return *c.flag == 0;
}

__device__ __forceinline__ void d_zero(float* p, int i0, int i1) {
  #pragma unroll 1
  for (int i = i0 + (int)threadIdx.x; i < i1; i += kDT) p[i] = 0.f;
}

// dst = LayerNorm(src) over C (eps 1e-5, F.layer_norm); stat (optional) <- mean, rstd
__device__ __noinline__ void d_layer_norm(float* dst, const float* src, const float* w, const float* bb, int C,
                                          float* stat, float* red) {
  const int t = threadIdx.x;
  float s = 0.f;
  #pragma unroll 1
  for (int i = t; i < C; i += kDT) s += src[i];
  const float mean = d_csum(s, red) / (float)C;
  float q = 0.f;
  #pragma unroll 1
  for (int i = t; i < C; i += kDT) {
    const float dv = src[i] - mean;
    q += dv * dv;
  }
  const float rstd = rsqrtf(d_csum(q, red) / (float)C + 1e-5f);
  #pragma unroll 1
  for (int i = t; i < C; i += kDT) dst[i] = ln_val(src[i], mean, rstd, __ldg(w + i), __ldg(bb + i));
  if (stat && t == 0) {
    stat[0] = mean;
    stat[1] = rstd;
  }
  d_csync();
}

__device__ __forceinline__ XDigits d_digits_at(uint8_t* base, int K, int lfk) {
  XDigits Xd;
  Xd.xd = reinterpret_cast<uint2*>(base);
  Xd.xc = reinterpret_cast<float*>(base + (size_t)K * 3);
  Xd.xsum = Xd.xc + (K >> (lfk + 5));
  return Xd;
}

// Input of a digit build: kind 0  z + (p - z) * mix (z, p shared, mix global);
// 1  z (shared); 2  g (global, read through L2); 3  relu(g)^2.
struct DSrc {
  int kind;
  const float* z;
  const float* p;
  const float* g;
};

template <int LFK>
__device__ __noinline__ void d_build(int kind, const float* z, const float* p, const float* g, int K, uint8_t* base) {
  const DSrc S{kind, z, p, g};
  auto get4 = [&](int i) -> float4 {
    if (S.kind == 0) {
      const float4 z = *reinterpret_cast<const float4*>(S.z + i), p = *reinterpret_cast<const float4*>(S.p + i);
      const float4 m = ldg4(S.g + i);
      return make_float4(z.x + (p.x - z.x) * m.x, z.y + (p.y - z.y) * m.y, z.z + (p.z - z.z) * m.z,
                         z.w + (p.w - z.w) * m.w);
    }
    if (S.kind == 1) return *reinterpret_cast<const float4*>(S.z + i);
    const float4 v = ldcg4(S.g + i);
    if (S.kind == 2) return v;
    return make_float4(v.x > 0.f ? v.x * v.x : 0.f, v.y > 0.f ? v.y * v.y : 0.f, v.z > 0.f ? v.z * v.z : 0.f,
                       v.w > 0.f ? v.w * v.w : 0.f);
  };
  // up to 4 items per thread (K <= 10240): all loads in flight at once
  if (K <= 32 * kDT)
    build_digits_r1<4>(K, LFK, get4, d_digits_at(base, K, LFK), threadIdx.x, kDT, kDBar);
  else
    build_digits(K, LFK, get4, d_digits_at(base, K, LFK), threadIdx.x, kDT, kDBar);
}

__device__ __forceinline__ void ld8(float (&v)[8], const float* p) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ldg8(float (&v)[8], const float* p) {
  const float4 a = ldg4(p), b = ldg4(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ldcg8(float (&v)[8], const float* p) {
  const float4 a = ldcg4(p), b = ldcg4(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
// Eight 2^-32 fixed-point values (one rounding each to fp32).
__device__ __forceinline__ float unfix(unsigned long long v) { return __ll2float_rn((long long)v) * kUnfix; }
__device__ __forceinline__ void ldcg8_fix(float (&v)[8], const unsigned long long* p) {
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const ulonglong2 w = __ldcg(reinterpret_cast<const ulonglong2*>(p) + h);
    v[2 * h] = unfix(w.x);
    v[2 * h + 1] = unfix(w.y);
  }
}
__device__ __forceinline__ void st8(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// Operands of one fused LayerNorm + token-shift prep (d_ln_mix).
struct DLnMix {
  const float* xs;   // shared input vector
  const float* add;  // global vector added to it (nullptr: none)
  const unsigned long long* add64;  // or a 2^-32 fixed-point vector added to it (nullptr: none)
  float* xo;         // shared copy of the sum (nullptr: not kept)
  const float *w, *b;  // LayerNorm weight, bias (global)
  const float* prev;   // previous-token vector (global; nullptr: mixes are the LayerNorm output itself)
  float* pv;           // shared copy of prev (nullptr: not kept)
  const float* mix[3];  // token-shift mixes (global), one digit set each
  int nmix;
  uint32_t need;  // bit m: emit the digits of mix m (the others are not used by this CTA)
  float* ln;     // shared LayerNorm output
  float* stat;   // mean, rstd (nullptr: not kept)
};

// The warp's shared-memory copy of a prep's operands (stored by lane 0), so
// the prep reads them from shared memory rather than from the stack.
__device__ __forceinline__ const DLnMix& d_warp_copy(DLnMix& dst, const DLnMix& q) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) dst = q;
  __syncwarp();
  return dst;
}

// y = LayerNorm(xs + add); for each mix m: digits of y + (prev - y) * mix_m
// into dig + m * stride.  One item of 8 columns per consumer thread (C <= 8 *
// kDT): every global operand of the phase is loaded in one round.
template <int LFK>
__device__ __noinline__ void d_ln_mix(const DArgs& a, DCons& c, const DLnMix& q, uint8_t* dig, uint32_t stride) {
  const int t = threadIdx.x, C = a.d.C, items = C >> 3;
  const bool act = t < items;
  const int i0 = act ? t * 8 : 0;
  float x[8], w[8], b[8], pv[8], mx[3][8];
  ld8(x, q.xs + i0);
  if (q.add) {
    float ad[8];
    ldcg8(ad, q.add + i0);
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] += ad[u];
  }
  if (q.add64) {
    float ad[8];
    ldcg8_fix(ad, q.add64 + i0);
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] += ad[u];
  }
  ldg8(w, q.w + i0);
  ldg8(b, q.b + i0);
  if (q.prev) ldcg8(pv, q.prev + i0);
#pragma unroll
  for (int m = 0; m < 3; ++m)  // only the mixes whose digits this CTA emits (every CTA reads them: L2-bound)
    if (m < q.nmix && q.mix[m] && ((q.need >> m) & 1u)) ldg8(mx[m], q.mix[m] + i0);
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u) s += act ? x[u] : 0.f;
  const float mean = d_csum(s, c.red) / (float)C;
  float qq = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float dv = x[u] - mean;
    qq += act ? dv * dv : 0.f;
  }
  const float rstd = rsqrtf(d_csum(qq, c.red) / (float)C + 1e-5f);
  float y[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) y[u] = ln_val(x[u], mean, rstd, w[u], b[u]);
  if (act) {
    if (q.xo) st8(q.xo + i0, x);
    st8(q.ln + i0, y);
    if (q.pv && q.prev) st8(q.pv + i0, pv);
  }
  if (q.stat && t == 0) {
    q.stat[0] = mean;
    q.stat[1] = rstd;
  }
#pragma unroll
  for (int m = 0; m < 3; ++m) {
    if (m < q.nmix && ((q.need >> m) & 1u)) {  // CTA-uniform
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = q.prev ? y[u] + (pv[u] - y[u]) * mx[m][u] : y[u];
      emit_digits(v, t, act, LFK, d_digits_at(dig + (size_t)m * stride, C, LFK));
    }
  }
  d_csync();
}

// Wait for the next ring slot; a warp whose wait gives up stops waiting for good.
__device__ __forceinline__ const uint8_t* d_slot_wait(const DArgs& a, DCons& c) {
  const int slot = c.seq % a.nst;
  if (!c.dead) {
    const bool got = mbar_wait_suspend(&c.full[slot], (uint32_t)((c.seq / a.nst) & 1));
    if (!__all_sync(0xffffffffu, got)) {
      c.dead = 1;
      if ((threadIdx.x & 31) == 0) {
        atomicOr(a.b.err, kErrTimeout);
        *c.abort = 1;
      }
    }
  }
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 0 && 3 * c.seq + 2 < 2 * a.trace_cap)
    a.trace[2 * (size_t)a.trace_cap + 3 * c.seq + 1] = global_ns();
  return c.sm + (size_t)slot * a.slot;
}

__device__ __forceinline__ void d_slot_release(const DArgs& a, DCons& c) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&c.empty[c.seq % a.nst]);
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 0 && 3 * c.seq + 2 < 2 * a.trace_cap)
    a.trace[2 * (size_t)a.trace_cap + 3 * c.seq + 2] = global_ns();
  d_wset(c.seq, c.seq + 1);
}

// GEMV units of one phase: out[row] += W[row, :] @ x for this CTA's units.
// The input of tile `tile` is the digit set at dig + (tile / per_set) * stride
// (per_set = 0: one input).  Arguments and ring counters live in registers
// for the loop (it stores to shared memory, so reads through `a` or `c` would
// be repeated each iteration).
template <int LFK>
// tiles_cm > 0: units in chunk-major order (tiles_cm tiles per chunk; every
// unit ends a tile), the digits built for chunks [ch0, ..] only, row sums
// added to the 2^-32 fixed-point `out64` instead of `out`.
__device__ __noinline__ void d_units(const DArgs& a, DCons& c, const DRange& R, uint8_t* dig, uint32_t stride, int K,
                                     int per_set, float* out, int rows_total, int tiles_cm = 0, int ch0 = 0,
                                     unsigned long long* out64 = nullptr) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const ImmaLane L = imma_lane();
  const int nst = a.nst, nb = a.nb, pr = a.pr, lg = a.lg, kch = a.kc >> 5, u0 = R.u0, u1 = R.u1, nch = R.nch;
  const uint32_t slot_b = a.slot, code_b = a.code_b;
  uint8_t* const sm = c.sm;
  uint64_t* const full = c.full;
  uint64_t* const empty = c.empty;
  float* const part = reinterpret_cast<float*>(sm + a.o_part);
  unsigned long long* tr = (a.trace && blockIdx.x == 0 && t == 0) ? a.trace + 2 * (size_t)a.trace_cap : nullptr;
  const int tr_n = 2 * a.trace_cap;
  int seq = c.seq;
  int slot = seq % nst;
  uint32_t ph = (uint32_t)((seq / nst) & 1);
  bool dead = c.dead;
  const int pofs = L.ra * pr + ((warp << 7) >> lg);
  float acc0 = 0.f, acc1 = 0.f;
  int cur_set = -1;
  XDigits X{};
  int tile = tiles_cm ? u0 % tiles_cm : u0 / nch, chunk = tiles_cm ? u0 / tiles_cm : u0 - tile * nch;
  int nt = 0;  // tiles buffered in `part`
  int* ptile = reinterpret_cast<int*>(part + kDPartTiles * kDW * 16);  // their tile indices
  // digit set of the current tile (tile / per_set), advanced with the tile
  int set = per_set ? tile / per_set : 0, set_end = per_set ? (set + 1) * per_set : 0x7fffffff;
#pragma unroll 1
  for (int u = u0; u < u1; ++u) {
    if (tile >= set_end) {
      ++set;
      set_end += per_set;
    }
    if (set != cur_set) {
      X = d_digits_at(dig + (size_t)set * stride, K, LFK);
      cur_set = set;
    }
    const uint8_t* sl = sm + (size_t)slot * slot_b;
    if (!dead) {
      bool got = mbar_try_wait(&full[slot], ph);  // usually already there: no timer, no suspend
      if (!got) got = mbar_wait_suspend(&full[slot], ph);
      if (!__all_sync(0xffffffffu, got)) {
        dead = true;
        if (lane == 0) {
          atomicOr(a.b.err, kErrTimeout);
          *c.abort = 1;
        }
      }
    }
    if (tr && 3 * seq + 2 < tr_n) tr[3 * seq + 1] = global_ns();
    if (!dead && warp < nb) {
      const float2* pp = reinterpret_cast<const float2*>(sl + code_b) + pofs;
      imma_block<LFK>(sl + warp * 2048, pp, pp + 8 * pr, (chunk - ch0) * kch + warp * 4, X, L, acc0, acc1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (tr && 3 * seq + 2 < tr_n) tr[3 * seq + 2] = global_ns();
    ++seq;
    if (++slot == nst) {
      slot = 0;
      ph ^= 1u;
    }
    if (tiles_cm || chunk == nch - 1 || u == u1 - 1) {
      // tile end: this warp's partial sums of the tile's 16 rows go to the
      // buffer; the CTA sums them over warps (in warp order) and adds each row
      // to `out` once per kDPartTiles tiles instead of meeting at every tile
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
      float* pt = part + nt * (kDW * 16);
      if ((lane & 3) == 0) {
        pt[warp * 16 + L.ra] = acc0;
        pt[warp * 16 + L.ra + 8] = acc1;
      }
      if (t == 0) ptile[nt] = tile;
      acc0 = acc1 = 0.f;
      if (++nt == kDPartTiles || u == u1 - 1) {
        d_csync();
#pragma unroll 1
        for (int i = t; i < nt * 16; i += kDT) {
          const float* q = part + (i >> 4) * (kDW * 16) + (i & 15);
          float v = 0.f;
          for (int w = 0; w < nb; ++w) v += q[w * 16];
          const int row = ptile[i >> 4] * 16 + (i & 15);
          if (row < rows_total && !dead) {
            if (out64) red_add_u64(out64 + row, (unsigned long long)__float2ll_rn(v * kFix));
            else red_add_f32(out + row, v);
          }
        }
        d_csync();  // the buffer is rewritten next
        nt = 0;
      }
    }
    if (tiles_cm) {
      if (++tile == tiles_cm) {
        tile = 0;
        ++chunk;
      }
    } else if (++chunk == nch) {
      chunk = 0;
      ++tile;
    }
  }
  __syncwarp();
  if (lane == 0) {
    c.seq = seq;
    c.dead = dead;
  }
  __syncwarp();
}

// Adapter first stages of this CTA (rows [i0, i1) of W1 [C][R] times the
// mixed input), accumulated in 2^-32 fixed point.
__device__ __noinline__ void d_items(const DArgs& a, DCons& c, const DTable& T, int l, const LayerDev& Ly,
                                     const float* TV, const float* PV, float* misc) {
  const int t = threadIdx.x, C = a.d.C;
  for (int k = 0; k < T.nitem[l == 0 ? 0 : 1]; ++k) {
    const int item = T.item[k];
    const int m = d_item_mat(a.d, item);
    const PackedView& W = m == 0 ? Ly.w1 : (m == 1 ? Ly.a1 : (m == 2 ? Ly.g1 : Ly.v1));
    const float* mix = m == 0 ? Ly.x_w : (m == 1 ? Ly.x_a : (m == 2 ? Ly.x_g : Ly.x_v));
    const int R = W.cols, wlg = W.lg;
    const int i0 = (item - a.d.abase[m]) * a.d.arow[m], i1 = min(C, i0 + a.d.arow[m]), nr = i1 - i0;
    float* xm = misc;          // [arow[m] <= 256]
    float* pacc = misc + 256;  // [nrg][R]
    const uint8_t* sl;
    if (a.pre) {  // the mix slice came with the item (d_issue_item)
      d_pre_wait(a, c, &c.pbar[2], c.nitm);
      sl = c.sm + a.o_item;
      const uint32_t qb0 = (uint32_t)(nr * R);
      const uint32_t g00 = (uint32_t)(((uint64_t)i0 * R) >> wlg) & ~1u;
      const uint32_t g10 = ((uint32_t)((((uint64_t)i1 * R - 1) >> wlg) + 1) + 1u) & ~1u;
      const float* mx = reinterpret_cast<const float*>(sl + ((qb0 + 15u) & ~15u) + (g10 - g00) * 8u);
      #pragma unroll 1
      for (int i = t; i < nr; i += kDT) xm[i] = TV[i0 + i] + (PV[i0 + i] - TV[i0 + i]) * mx[i];
      d_csync();
    } else {
      #pragma unroll 1
      for (int i = t; i < nr; i += kDT) xm[i] = TV[i0 + i] + (PV[i0 + i] - TV[i0 + i]) * __ldg(mix + i0 + i);
      d_csync();
      sl = d_slot_wait(a, c);
    }
    // four columns per thread (one 32-bit code word; a group holds whole
    // quads: R % 16 == 0, group >= 4), rows split over `nrg` row groups; per
    // row the scale is folded into the input: x (q d + mn) = (x d) q + x mn
    const int q4 = R >> 2;
    const int nrg = q4 < kDT ? kDT / q4 : 1;
    const uint32_t qb = (uint32_t)(nr * R);
    const float2* cs = reinterpret_cast<const float2*>(sl + ((qb + 15u) & ~15u));
    const uint32_t g0 = (uint32_t)(((uint64_t)i0 * R) >> wlg) & ~1u;
    #pragma unroll 1
    for (int jw = t; !c.dead && jw < nrg * q4; jw += kDT) {
      const int j = (jw % q4) * 4, rg = jw / q4;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, bs = 0.f;
      #pragma unroll 4
      for (int i = rg; i < nr; i += nrg) {
        const uint32_t e = (uint32_t)(i0 + i) * (uint32_t)R + (uint32_t)j;
        const float2 sc = cs[(e >> wlg) - g0];
        const float xv = xm[i];
        const float ad = xv * __fmul_rn(__fsub_rn(sc.y, sc.x), kInv255);
        bs = fmaf(xv, sc.x, bs);
        const uint32_t w4 = *reinterpret_cast<const uint32_t*>(sl + i * R + j);
        // code byte b as a float: bits 0x4B0000qq = 2^23 + q, minus 2^23 (exact)
        a0 = fmaf(ad, __uint_as_float(__byte_perm(w4, 0x4B000000u, 0x7440)) - 8388608.0f, a0);
        a1 = fmaf(ad, __uint_as_float(__byte_perm(w4, 0x4B000000u, 0x7441)) - 8388608.0f, a1);
        a2 = fmaf(ad, __uint_as_float(__byte_perm(w4, 0x4B000000u, 0x7442)) - 8388608.0f, a2);
        a3 = fmaf(ad, __uint_as_float(__byte_perm(w4, 0x4B000000u, 0x7443)) - 8388608.0f, a3);
      }
      *reinterpret_cast<float4*>(pacc + rg * R + j) = make_float4(a0 + bs, a1 + bs, a2 + bs, a3 + bs);
    }
    if (!a.pre) d_slot_release(a, c);
    d_csync();
    if (a.pre) {
      if (t == 0) mbar_arrive(&c.pbar[3]);  // the item buffer may be refilled
      d_wset(c.nitm, c.nitm + 1);
    }
    if (!c.dead) {
      const int off = d_rank_off(a.d, m);
      #pragma unroll 1
      for (int j = t; j < R; j += kDT) {
        float v = 0.f;
        for (int rg = 0; rg < nrg; ++rg) v += pacc[rg * R + j];
        red_add_u64(a.b.adp64 + off + j, (unsigned long long)__float2ll_rn(v * kFix));
      }
    }
    d_csync();
  }
}

// Phase B, preload mode: the four adapter second stages of head h on the
// integer tensor cores.  Output column c of adapter m is
//     sum_r mid_r (q[r][c] d_r + min_r) = sum_r x'_r q[r][c] + sum_r mid_r min_r,
// x'_r = mid_r d_r (d, min of row r's weight group, which holds all 64 columns
// of the head): a GEMV whose activation x' is split into three digits per
// 32-row flush group (emit_digits) and whose A operand is the transposed code
// image ([64 columns][rank]).  Tasks (chunk of kDPieceSteps k-steps, 16-column
// tile) go round-robin to the warps; partials are summed in chunk order.
// Writes vec[m * 64 + c] for the layer's adapters; ends with the consumer
// barrier.
__device__ __noinline__ void d_pieces_mma(const DArgs& a, DCons& c, const DTable& T, int l, const float* mid,
                                          float* misc, float* vec) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, g = lane >> 2, tq = lane & 3, h = blockIdx.x;
  const int nm = l == 0 ? 3 : 4, nck = T.nck[l == 0 ? 0 : 1];
  d_pre_wait(a, c, &c.pbar[0], c.nadp);
  const uint8_t* img = c.sm + a.o_adp;
  uint32_t boff[4];
  int roff[5];
  {
    uint32_t o = 0;
    int r = 0;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      boff[m] = o;
      roff[m] = r;
      o += 64u * (uint32_t)a.aps[m] + 16u * (uint32_t)a.apr[m];
      r += a.apr[m];
    }
    roff[4] = r;
  }
  const int rt = roff[4], nit = rt >> 3;
  float* bpart = misc;                                         // [nit] sum over an item's rows of mid * min
  uint8_t* dgb = reinterpret_cast<uint8_t*>(misc + nit);       // digit blocks, 3.25 bytes per row
  float* part = misc + nit + rt * 13 / 16;                     // [4 nck][16]
  float* bias = part + 64 * nck;                               // [4]
  auto adapter_of = [&](int j) { return j >= roff[3] ? 3 : (j >= roff[2] ? 2 : (j >= roff[1] ? 1 : 0)); };
  auto digits_of = [&](int m) {
    XDigits X;
    uint8_t* b = dgb + (size_t)roff[m] * 13 / 4;
    X.xd = reinterpret_cast<uint2*>(b);
    X.xc = reinterpret_cast<float*>(b + 3 * a.apr[m]);
    X.xsum = X.xc + a.apr[m] / 32;
    return X;
  };
  // one 8-row item per lane: x'_r = mid_r d_r of its rows, their digits (32-row
  // flush groups: four adjacent lanes), and the item's sum of mid_r min_r
  if (w * 32 < nit) {
    const int it = w * 32 + lane;
    const bool act = it < nit && !c.dead;
    const int m = it < nit ? adapter_of(it * 8) : 0;
    const int R = d_rank(a.d, m), sel = ((h * 64) >> a.alg[m]) & 1;
    const float2* pairs = reinterpret_cast<const float2*>(img + boff[m] + 64u * (uint32_t)a.aps[m]);
    const float* md = mid + d_rank_off(a.d, m);
    float v[8], bs = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = it * 8 + u - roff[m];
      v[u] = 0.f;
      if (act && m < nm && r < R) {
        const float2 pq = pairs[r * 2 + sel];
        v[u] = md[r] * __fmul_rn(__fsub_rn(pq.y, pq.x), kInv255);
        bs = fmaf(md[r], pq.x, bs);
      }
    }
    if (act) bpart[it] = bs;
    emit_digits(v, act ? it - roff[m] / 8 : 0, act, 0, digits_of(m));
  }
  d_csync();
  if (w < nm) {  // the adapter's min term, its items in order
    float sb = 0.f;
    for (int i = roff[w] / 8 + lane; i < roff[w + 1] / 8; i += 32) sb += bpart[i];
    sb = warp_sum(sb);
    if (lane == 0) bias[w] = sb;
  }
#pragma unroll 1
  for (int tau = w; !c.dead && tau < 4 * nck; tau += kDW) {
    const int k = tau >> 2, tile = tau & 3, m = T.ckm[k], s0 = T.cks[k];
    const int s1 = min(s0 + kDPieceSteps, a.apr[m] / 32);
    const XDigits X = digits_of(m);
    const uint8_t* rowa = img + boff[m] + (uint32_t)(tile * 16 + g) * (uint32_t)a.aps[m] + 8 * tq;
    const uint8_t* rowb = rowa + 8 * a.aps[m];
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
    for (int ks = s0; ks < s1; ++ks) {
      const uint2 w0 = *reinterpret_cast<const uint2*>(rowa + ks * 32);
      const uint2 w1 = *reinterpret_cast<const uint2*>(rowb + ks * 32);
      const uint2 bb = lane < 12 ? X.xd[ks * 12 + lane] : make_uint2(0u, 0u);
      int d[4] = {0, 0, 0, 0};
      imma_16832(d, w0.x, w1.x, w0.y, w1.y, bb.x, bb.y);
      // lanes without branches (as in imma_block): tq = 1 holds digit 2 and
      // the zero column 3, tq >= 2 zero columns whose sums are never stored
      const float cs = X.xc[ks];
      const float cq = tq == 0 ? cs : cs * kInv254sq;
      acc0 = fmaf(cq, fmaf((float)d[1], kInv254, (float)d[0]), acc0);
      acc1 = fmaf(cq, fmaf((float)d[3], kInv254, (float)d[2]), acc1);
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    if (tq == 0) {
      part[tau * 16 + g] = acc0;
      part[tau * 16 + g + 8] = acc1;
    }
  }
  d_csync();
  if (t < 256) {
    const int m = t >> 6, cc = t & 63, tile = cc >> 4, r = cc & 15;
    if (m < nm) {
      float sacc = bias[m];
      for (int k = 0; k < nck; ++k)
        if (T.ckm[k] == m) sacc += part[(k * 4 + tile) * 16 + r];
      vec[m * 64 + cc] = sacc;
    }
  }
  d_csync();
}

// Phase B for head h = blockIdx.x: adapter second stages, kk-normalize, decay,
// WKV7 update of S (already in shared memory), GroupNorm, bonus, gate.
__device__ __noinline__ void d_head_wkv(const DArgs& a, DCons& c, const DTable& T, int l, const LayerDev& Ly,
                                        float* S, float* misc) {
  const int t = threadIdx.x, C = a.d.C, H = a.d.H, h = blockIdx.x;
  float* mid = S + 4096;                     // [rtot]
  float* vec = mid + ((a.d.rtot + 3) & ~3);  // [4][64]
  float* sr = vec + 256;
  float* sd = sr + 64;
  float* sk = sd + 64;
  float* sv = sk + 64;
  float* skk = sv + 64;
  float* ska = skk + 64;
  float* sy = ska + 64;
  float* Sg = a.b.wkv + ((size_t)l * H + h) * 4096;
  const int nm = l == 0 ? 3 : 4;
  const int used = l == 0 ? a.d.rw + a.d.ra + a.d.rg : a.d.rtot;
  // every global operand of the head in one round: the first-adapter sums
  // (up to kMidPer per thread) and the head's per-channel vectors are loaded
  // together, then used
  unsigned long long mq[kMidPer];
#pragma unroll
  for (int q = 0; q < kMidPer; ++q) {
    const int j = t + q * kDT;
    mq[q] = j < used ? __ldcg(a.b.adp64 + j) : 0ull;
  }
  float r = 0.f, k = 0.f, v = 0.f, vf = 0.f, kk_w = 0.f, a0 = 0.f, ka = 0.f, v0 = 0.f, w0 = 0.f, rk = 0.f, lw = 0.f,
        lb = 0.f;
  if (t < 64) {
    const int ch = h * 64 + t;
    r = __ldcg(a.b.rkv + ch);
    k = __ldcg(a.b.rkv + C + ch);
    v = __ldcg(a.b.rkv + 2 * C + ch);
    if (l != 0) {
      vf = __ldcg(a.b.v_first + ch);
      v0 = __ldg(Ly.v0 + ch);
    }
    kk_w = __ldg(Ly.k_k + ch);
    a0 = __ldg(Ly.a0 + ch);
    ka = __ldg(Ly.k_a + ch);
    w0 = __ldg(Ly.w0 + ch);
    rk = __ldg(Ly.r_k + ch);
    lw = __ldg(Ly.lnx_w + ch);
    lb = __ldg(Ly.lnx_b + ch);
  }
#pragma unroll
  for (int q = 0; q < kMidPer; ++q) {
    const int j = t + q * kDT;
    if (j < used) {
      float mv = (float)(long long)mq[q] * kUnfix;
      if (j < a.d.rw) mv = tanhf(mv);
      else if (j >= a.d.rw + a.d.ra && j < a.d.rw + a.d.ra + a.d.rg) mv = sigmoidf_(mv);
      mid[j] = mv;
    }
  }
  float* vp = misc;  // [kDW / 2 warp pairs][4 matrices][64 columns] partials
  cp_async_wait_all();
  d_csync();
  if (a.pre) {
    d_pieces_mma(a, c, T, l, mid, misc, vec);
    if (t == 0) mbar_arrive(&c.pbar[1]);  // the head image buffer may be refilled
    d_wset(c.nadp, c.nadp + 1);
  } else {
    // 16 lanes per tile row, 4 columns each (one 32-bit code word); the two
    // half-warps take alternate rows: row phase rp of 20.  Per row the scale
    // is folded into the input: mid * (q * d + mn) = (mid * d) * q + mid * mn.
    const int lane = t & 31, w = t >> 5, cg = lane & 15, rp = w * 2 + (lane >> 4);
    float acc4[4][5];  // per adapter: this lane's four column partials and its min term
#pragma unroll
    for (int mm = 0; mm < 4; ++mm)
#pragma unroll
      for (int u = 0; u < 5; ++u) acc4[mm][u] = 0.f;
    const int npc = T.npc[l == 0 ? 0 : 1];
    for (int pc = 0; pc < npc; ++pc) {
      const uint8_t* sl = d_slot_wait(a, c);
      if (!c.dead) {
        const int m = T.pm[pc];
        const int br = a.abr[m], r0 = T.pr0[pc];
        const int nr = min(br, d_rank(a.d, m) - r0);
        const float2* pairs = reinterpret_cast<const float2*>(sl + br * 64);
        const int sel = ((h * 64) >> a.alg[m]) & 1;
        const float* mm = mid + d_rank_off(a.d, m) + r0;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, bs = 0.f;
        #pragma unroll 4
        for (int i = rp; i < nr; i += 2 * kDW) {
          const float2 pq = pairs[i * 2 + sel];
          const float am = mm[i];
          const float ad = am * __fmul_rn(__fsub_rn(pq.y, pq.x), kInv255);
          bs = fmaf(am, pq.x, bs);
          const uint32_t q4 = *reinterpret_cast<const uint32_t*>(sl + i * 64 + 4 * cg);
          // code byte k as a float: bits 0x4B0000qq = 2^23 + q, minus 2^23 (exact)
          a0 = fmaf(ad, __uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7440)) - 8388608.0f, a0);
          a1 = fmaf(ad, __uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7441)) - 8388608.0f, a1);
          a2 = fmaf(ad, __uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7442)) - 8388608.0f, a2);
          a3 = fmaf(ad, __uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7443)) - 8388608.0f, a3);
        }
        // lanes l and l ^ 16 hold the same columns (alternate rows)
        a0 += __shfl_xor_sync(0xffffffffu, a0, 16);
        a1 += __shfl_xor_sync(0xffffffffu, a1, 16);
        a2 += __shfl_xor_sync(0xffffffffu, a2, 16);
        a3 += __shfl_xor_sync(0xffffffffu, a3, 16);
        bs += __shfl_xor_sync(0xffffffffu, bs, 16);
#pragma unroll
        for (int mm = 0; mm < 4; ++mm)
          if (mm == m) {  // warp-uniform
            acc4[mm][0] += a0;
            acc4[mm][1] += a1;
            acc4[mm][2] += a2;
            acc4[mm][3] += a3;
            acc4[mm][4] += bs;
          }
      }
      d_slot_release(a, c);
    }
    // fixed-order fold of the warps' partials: warp w + kDW/2 stores, warp w adds
    // its own, then the sum over the kDW/2 pairs (below) in pair order
    constexpr int kHalf = kDW / 2;
    if (w >= kHalf && lane < 16)
#pragma unroll
      for (int mm = 0; mm < 4; ++mm)
        *reinterpret_cast<float4*>(vp + ((w - kHalf) * 4 + mm) * 64 + 4 * cg) =
            make_float4(acc4[mm][0] + acc4[mm][4], acc4[mm][1] + acc4[mm][4], acc4[mm][2] + acc4[mm][4],
                        acc4[mm][3] + acc4[mm][4]);
    d_csync();
    if (w < kHalf && lane < 16)
#pragma unroll
      for (int mm = 0; mm < 4; ++mm) {
        float4* dst = reinterpret_cast<float4*>(vp + (w * 4 + mm) * 64 + 4 * cg);
        float4 v4 = *dst;
        v4.x += acc4[mm][0] + acc4[mm][4];
        v4.y += acc4[mm][1] + acc4[mm][4];
        v4.z += acc4[mm][2] + acc4[mm][4];
        v4.w += acc4[mm][3] + acc4[mm][4];
        *dst = v4;
      }
    d_csync();
    if (t < 256) {
      const int m = t >> 6, cc = t & 63;
      float s = 0.f;
      if (m < nm)
        for (int q = 0; q < kDW / 2; ++q) s += vp[(q * 4 + m) * 64 + cc];
      vec[m * 64 + cc] = s;
    }
    d_csync();
  }
  // the head's 64 channels live in warps 0-1: their sums use a 64-thread barrier
  if (t < 64) {
    const int ch = h * 64 + t;
    const float kkv = k * kk_w;
    const float nrm = sqrtf(d_sum64(kkv * kkv, c.red));
    const float aa = sigmoidf_(a0 + vec[64 + t]);
    const float kk = kkv / fmaxf(nrm, 1e-12f);
    const float kn = k * (1.0f + (aa - 1.0f) * ka);
    if (l == 0) a.b.v_first[ch] = v;
    else v = v + (vf - v) * sigmoidf_(v0 + vec[192 + t]);
    sr[t] = r;
    sd[t] = expf(-0.606531f * sigmoidf_(w0 + vec[t]));
    sk[t] = kn;
    sv[t] = v;
    skk[t] = kk;
    ska[t] = kk * aa;
  }
  d_csync();
  if (t < 256) {
    wkv7_head64(S, sr, sd, sk, sv, skk, ska, sy, Sg);  // the new state straight to global memory
    bar_sync(kDBar64 - 1, 256);                       // y of every channel visible to warps 0-1
    if (t < 64) {
      const int ch = h * 64 + t;
      const float yv = sy[t];
      const float2 mb = d_sum64x2(yv, sr[t] * sk[t] * rk, c.red + 2);
      const float mean = mb.x / 64.f;
      const float dv = yv - mean;
      const float var = d_sum64(dv * dv, c.red + 6) / 64.f;
      float o = dv * rsqrtf(var + 64e-5f) * lw + lb;
      o = o + mb.y * sv[t];
      a.b.att_y[ch] = o * vec[128 + t];
    }
  }
}

// Copy layer l's descriptor (weight views, vector pointers) into shared
// memory with 4-byte cp.async copies (the caller commits and waits): read
// from global memory it would cost a dependent L2 round trip at the start of
// every phase that uses it.
__device__ __forceinline__ void d_load_layer(const DArgs& a, LayerDev* dst, int l) {
  static_assert(sizeof(LayerDev) % 4 == 0, "layer descriptor in 4-byte words");
  constexpr int kWords = (int)(sizeof(LayerDev) / 4);
  const int t = threadIdx.x;
  if (t < kWords) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.layers + l) + t;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(reinterpret_cast<uint32_t*>(dst) + t)),
                 "l"(src)
                 : "memory");
  }
}

// X = LayerNorm0(emb[tok]).
__device__ __noinline__ void d_embed(const DArgs& a, DCons& c, int tok, float* X, float* TV, float* PV) {
  const int t = threadIdx.x, C = a.d.C;
  const PackedView& E = a.emb;
  if (a.emb_fast) {
    const int gpr = C >> E.lg;
    uint8_t* q = reinterpret_cast<uint8_t*>(TV);
    float2* sc = reinterpret_cast<float2*>(PV);
    #pragma unroll 1
    for (int o = t * 16; o < C; o += kDT * 16) cp_async16(q + o, E.payload + (size_t)tok * C + o);
    #pragma unroll 1
    for (int o = t * 16; o < gpr * 8; o += kDT * 16)
      cp_async16(reinterpret_cast<uint8_t*>(sc) + o, E.meta + (size_t)tok * gpr * 8 + o);
    cp_async_commit();
    cp_async_wait_all();
    d_csync();
    #pragma unroll 1
    for (int i = t; i < C; i += kDT) {
      const float2 s = sc[i >> E.lg];
      X[i] = sg8_dequant(q[i], s.x, s.y);
    }
  } else {
    #pragma unroll 1
    for (int i = t; i < C; i += kDT) X[i] = packed_at(E, tok, i);
  }
  d_csync();
  d_layer_norm(X, X, a.ln0_w, a.ln0_b, C, nullptr, c.red);
}

// This CTA's slice of the logits: first maximum -> amax partials.
__device__ __noinline__ void d_argmax_part(const DArgs& a, const DTable& T, float* s_bv, int* s_bi) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  #pragma unroll 1
  for (int i = T.zv0 + t; i < T.zv1; i += kDT) {
    const float v = __ldcg(a.b.logits + i);
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
  d_csync();
  if (t == 0) {
    float cb = -INFINITY;
    int ci = 0x7fffffff;
    for (int w = 0; w < kDW; ++w)
      if (s_bv[w] > cb || (s_bv[w] == cb && s_bi[w] < ci)) {
        cb = s_bv[w];
        ci = s_bi[w];
      }
    a.b.amax_v[blockIdx.x] = cb;
    a.b.amax_i[blockIdx.x] = ci;
  }
}

// First maximum over all CTAs' partials (every CTA computes the same token).
__device__ __noinline__ int d_argmax_all(const DArgs& a, int* s_tok) {
  const int t = threadIdx.x, lane = t & 31;
  if (t < 32) {
    float gb = -INFINITY;
    int gi = 0x7fffffff;
    for (int cta = lane; cta < (int)gridDim.x; cta += 32) {
      const float v = __ldcg(a.b.amax_v + cta);
      const int i = __ldcg(a.b.amax_i + cta);
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
    if (t == 0) *s_tok = gi == 0x7fffffff ? 0 : gi;
  }
  d_csync();
  return *s_tok;
}

// --------------------------------------------------------------- kernel
template <int LFK>
__global__ void __launch_bounds__(kDThreads, 1) decode_kernel(const __grid_constant__ DArgs ga) {
  extern __shared__ __align__(1024) uint8_t d_smraw[];
  uint8_t* sm = d_smraw + ((1024u - (smem_u32(d_smraw) & 1023u)) & 1023u);
  __shared__ DTable T;
  __shared__ uint64_t full[kDMaxSt], empty[kDMaxSt];
  __shared__ uint64_t pbar[4];  // preload mode: adp full / empty, item full / empty
  __shared__ float red[32];
  __shared__ int s_flag, s_tok;
  __shared__ volatile int s_abort;
  __shared__ float s_bv[kDW];
  __shared__ int s_bi[kDW];
  __shared__ float s_stat[4];  // mean / rstd of ln1 and ln2
  __shared__ DCons s_cons[kDW];
  __shared__ DLnMix s_q[kDW];
  __shared__ __align__(16) LayerDev s_ly[2];  // descriptors of the current and the next layer
  // the launch arguments in shared memory: the subroutines read them through
  // a reference, and those reads measured slower from the parameter space
  __shared__ __align__(16) DArgs s_args;
  static_assert(sizeof(DArgs) % 4 == 0 && sizeof(DArgs) <= 1024, "launch arguments in shared memory");

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int i = t; i < (int)(sizeof(DArgs) / 4); i += (int)blockDim.x)
    reinterpret_cast<uint32_t*>(&s_args)[i] = reinterpret_cast<const uint32_t*>(&ga)[i];
  __syncthreads();
  // the subroutines read the shared copy; the code below reads fields of the
  // parameter itself at fixed offsets (constant-bank operands)
  const DArgs& a = s_args;
  if (t == 0) {
    d_build_table(a, T);
    for (int i = 0; i < ga.nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kDW);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&pbar[i], 1);
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  if (warp == kDW) {
    if (lane == 0) d_producer(a, T, sm, full, empty, &s_abort, pbar);
    return;
  }

  const int C = ga.d.C, F = ga.d.F, H = ga.d.H, G = gridDim.x, bx = blockIdx.x;
  const bool fused = C <= 8 * kDT;  // one 8-column item per consumer thread: single-round preps
  float* X = reinterpret_cast<float*>(sm + ga.o_x);    // layer input (residual stream)
  float* XB = reinterpret_cast<float*>(sm + ga.o_xb);  // after attention
  float* TV = reinterpret_cast<float*>(sm + ga.o_t);   // normalised vector
  float* PV = reinterpret_cast<float*>(sm + ga.o_p);   // previous-token vector
  float* misc = reinterpret_cast<float*>(sm + ga.o_misc);
  uint8_t* dig = sm + ga.o_dig;
  DCons& c = s_cons[warp];
  if (lane == 0) {
    c.sm = sm;
    c.full = full;
    c.empty = empty;
    c.red = red;
    c.abort = &s_abort;
    c.flag = &s_flag;
    c.seq = c.pbuf = c.dead = c.tr = 0;
    c.pbar = pbar;
    c.nadp = c.nitm = 0;
    c.trow = bx == 0 ? 0 : (bx == G - 1 ? 1 : -1);
    c.target = 0;
  }
  __syncwarp();

  float* acc_rkv = ga.b.rkv;
  float* acc_ao = ga.b.ao;
  float* acc_hk = ga.b.h;
  float* acc_fo = ga.b.fo;
  float* logits = ga.b.logits;

  // accumulators start from zero in every launch (a failed launch may leave partial sums)
  d_zero(acc_rkv, T.z3c0, T.z3c1);
  d_zero(acc_hk, T.zf0, T.zf1);
  d_zero(acc_ao, T.zc0, T.zc1);
  d_zero(acc_fo, T.zc0, T.zc1);
  d_zero(logits, T.zv0, T.zv1);
  #pragma unroll 1
  for (int i = T.zr0 + t; i < T.zr1; i += kDT) ga.b.adp64[i] = 0ull;
  const bool ecm = ga.ecm != 0;  // FFN value rows in chunk order, output in fixed point
  unsigned long long* fo64 = ga.b.fo64;
  #pragma unroll 1
  for (int i = T.zc0 + t; i < T.zc1; i += kDT) fo64[i] = 0ull;
  int tok = ga.mode == 0 ? (ga.first_tok >= 0 ? ga.first_tok : __ldcg(ga.b.tok)) : __ldg(ga.forced);
  // streamed decode: the host's cancel word as CTA 0 read it during the
  // previous token's head (loaded a token ahead, so no step waits on the bus)
  int cancel_next = 0;
  d_load_layer(a, &s_ly[0], 0);
  cp_async_commit();
  cp_async_wait_all();  // published by the barrier below
  bool alive = d_gsync(a, c);
  int gl = 0;  // layers run by this launch: s_ly[gl & 1] holds layer l's descriptor
  for (int step = 0; step < ga.ntok && alive; ++step) {
    const bool head = ga.mode == 0 || step == ga.ntok - 1;
    if (ga.mode == 1) tok = __ldg(ga.forced + step);
    if (tok < 0 || tok >= ga.d.V) {
      if (t == 0) atomicOr(ga.b.err, kErrToken);
      tok = 0;
    }
    d_mark(a, c);  // token start
    cp_async_wait_all();  // layer 0's descriptor, published by the barriers of d_embed
    d_embed(a, c, tok, X, TV, PV);

    for (int l = 0; l < ga.d.L && alive; ++l, ++gl) {
      const LayerDev& Ly = s_ly[gl & 1];
      if (l > 0) {
        cp_async_wait_all();  // this layer's descriptor, published by the barrier
        if (!d_gsync(a, c)) {
          alive = false;
          break;
        }
      }
      d_mark(a, c);  // A start
      // ================= A: ln1, mixes, r/k/v rows, adapter first stages
      if (fused) {
        DLnMix q{};
        q.xs = l > 0 ? XB : X;
        q.add = l > 0 && !ecm ? acc_fo : nullptr;
        q.add64 = l > 0 && ecm ? fo64 : nullptr;
        q.xo = X;
        q.w = Ly.ln1_w;
        q.b = Ly.ln1_b;
        q.prev = ga.b.att_x + (size_t)l * C;
        q.pv = PV;
        q.mix[0] = Ly.x_r;
        q.mix[1] = Ly.x_k;
        q.mix[2] = Ly.x_v;
        q.nmix = 3;
        q.need = T.aneed;  // only the r/k/v digit sets this CTA's units read
        q.ln = TV;
        q.stat = s_stat;
        d_ln_mix<LFK>(a, c, d_warp_copy(s_q[warp], q), dig, ga.dig_set);
      } else {
        if (l > 0) {
#pragma unroll 1
          for (int i = t; i < C; i += kDT) X[i] = XB[i] + (ecm ? unfix(__ldcg(fo64 + i)) : __ldcg(acc_fo + i));
          d_csync();
        }
        d_layer_norm(TV, X, Ly.ln1_w, Ly.ln1_b, C, s_stat, red);
#pragma unroll 1
        for (int i = t; i < C; i += kDT) PV[i] = __ldcg(ga.b.att_x + (size_t)l * C + i);
        d_csync();
        if (T.aneed & 1u) d_build<LFK>(0, TV, PV, Ly.x_r, C, dig);
        if (T.aneed & 2u) d_build<LFK>(0, TV, PV, Ly.x_k, C, dig + ga.dig_set);
        if (T.aneed & 4u) d_build<LFK>(0, TV, PV, Ly.x_v, C, dig + 2 * ga.dig_set);
      }
      d_mark(a, c);  // A prep done
      d_units<LFK>(a, c, T.r[0], dig, ga.dig_set, C, C / 16, acc_rkv, 3 * C);
      d_mark(a, c);  // A units done
      d_items(a, c, T, l, Ly, TV, PV, misc);
      d_mark(a, c);  // A done
      // ================= B: one CTA per head
      const bool is_head = bx < H;
      float* S = reinterpret_cast<float*>(dig);  // digit sets are dead in B
      // the next layer's descriptor (the other buffer: the last reads of the
      // previous layer's ended with its phase D)
      d_load_layer(a, &s_ly[(gl + 1) & 1], l + 1 < ga.d.L ? l + 1 : 0);
      if (is_head) {
        const float* Sg = ga.b.wkv + ((size_t)l * H + bx) * 4096;
        #pragma unroll 1
        for (int u = t; u < 1024; u += kDT) cp_async16(S + u * 4, Sg + u * 4);
      }
      cp_async_commit();
      if (!d_gsync(a, c)) {
        alive = false;
        break;
      }
      d_mark(a, c);  // B barrier
      d_zero(acc_hk, T.zf0, T.zf1);
      if (l == 0) d_zero(logits, T.zv0, T.zv1);
      if (is_head) d_head_wkv(a, c, T, l, Ly, S, misc);
      d_mark(a, c);  // B done
      if (!d_gsync(a, c)) {
        alive = false;
        break;
      }
      d_mark(a, c);  // C barrier
      // ================= C: output projection; att_x[l] <- ln1 slice
      if (ecm) {
        #pragma unroll 1
        for (int i = T.zc0 + t; i < T.zc1; i += kDT) fo64[i] = 0ull;
      } else {
        d_zero(acc_fo, T.zc0, T.zc1);
      }
      #pragma unroll 1
      for (int i = T.zc0 + t; i < T.zc1; i += kDT)
        ga.b.att_x[(size_t)l * C + i] = TV[i];  // ln1 output of phase A, still in shared memory
      d_build<LFK>(2, nullptr, nullptr, ga.b.att_y, C, dig);
      d_mark(a, c);  // C prep done
      d_units<LFK>(a, c, T.r[1], dig, 0, C, 0, acc_ao, C);
      d_mark(a, c);  // C done
      if (!d_gsync(a, c)) {
        alive = false;
        break;
      }
      d_mark(a, c);  // D barrier
      // ================= D: x += att; ln2 + mix; ffn key rows
      d_zero(acc_rkv, T.z3c0, T.z3c1);
      #pragma unroll 1
      for (int i = T.zr0 + t; i < T.zr1; i += kDT) ga.b.adp64[i] = 0ull;
            if (fused) {
        DLnMix q{};
        q.xs = X;
        q.add = acc_ao;
        q.xo = XB;
        q.w = Ly.ln2_w;
        q.b = Ly.ln2_b;
        q.prev = ga.b.ffn_x + (size_t)l * C;
        q.mix[0] = Ly.ffn_x_k;
        q.nmix = 1;
        q.need = 1u;
        q.ln = TV;
        q.stat = s_stat + 2;
        d_ln_mix<LFK>(a, c, d_warp_copy(s_q[warp], q), dig, 0);
      } else {
#pragma unroll 1
        for (int i = t; i < C; i += kDT) {
          XB[i] = X[i] + __ldcg(acc_ao + i);
          PV[i] = __ldcg(ga.b.ffn_x + (size_t)l * C + i);
        }
        d_csync();
        d_layer_norm(TV, XB, Ly.ln2_w, Ly.ln2_b, C, s_stat + 2, red);
        d_build<LFK>(0, TV, PV, Ly.ffn_x_k, C, dig);
      }
      d_mark(a, c);  // D prep done
      d_units<LFK>(a, c, T.r[2], dig, 0, C, 0, acc_hk, F);
      d_mark(a, c);  // D done
      if (!d_gsync(a, c)) {
        alive = false;
        break;
      }
      d_mark(a, c);  // E barrier
      // ================= E: relu^2; ffn value rows; ffn_x[l] <- ln2 slice
      d_zero(acc_ao, T.zc0, T.zc1);
      #pragma unroll 1
      for (int i = T.zc0 + t; i < T.zc1; i += kDT)
        ga.b.ffn_x[(size_t)l * C + i] = TV[i];  // ln2 output of phase D, still in shared memory
      d_mark(a, c);  // E slices stored
      if (ecm) {
        // only the chunks of this CTA's units: [ech0, ech1] of kc columns each
        const int k0 = T.ech0 * ga.kc, kl = (T.ech1 - T.ech0 + 1) * ga.kc;
        d_build<LFK>(3, nullptr, nullptr, acc_hk + k0, kl, dig);
        d_mark(a, c);  // E prep done
        d_units<LFK>(a, c, T.r[3], dig, 0, kl, 0, nullptr, C, C / 16, T.ech0, fo64);
      } else {
        d_build<LFK>(3, nullptr, nullptr, acc_hk, F, dig);
        d_mark(a, c);  // E prep done
        d_units<LFK>(a, c, T.r[3], dig, 0, F, 0, acc_fo, C);
      }
      d_mark(a, c);  // E done
    }
    if (!alive) break;
    if (!head) continue;
    // ================= head: ln_out, logits, argmax (first maximum)
    if (!d_gsync(a, c)) {
      alive = false;
      break;
    }
    d_mark(a, c);  // head barrier
    // the host's cancel word crosses the bus once per token: the value read
    // during the previous token's head is acted on now (published to every CTA
    // before the last barrier of the token) and the next read is issued, to be
    // used one token later, so its latency never stalls a step
    int cancel_seen = 0;
    if (ga.ring_cancel && bx == 0 && t == 0) {
      cancel_seen = cancel_next;
      cancel_next = d_ld_relaxed_sys(ga.ring_cancel);
    }
    d_zero(acc_hk, T.zf0, T.zf1);
    if (fused) {
      DLnMix q{};
      q.xs = XB;
      q.add = ecm ? nullptr : acc_fo;
      q.add64 = ecm ? fo64 : nullptr;
      q.w = ga.lnout_w;
      q.b = ga.lnout_b;
      q.nmix = 1;
      q.need = 1u;
      q.ln = TV;
      d_ln_mix<LFK>(a, c, d_warp_copy(s_q[warp], q), dig, 0);
    } else {
#pragma unroll 1
      for (int i = t; i < C; i += kDT) PV[i] = XB[i] + (ecm ? unfix(__ldcg(fo64 + i)) : __ldcg(acc_fo + i));
      d_csync();
      d_layer_norm(TV, PV, ga.lnout_w, ga.lnout_b, C, nullptr, red);
      d_build<LFK>(1, TV, nullptr, nullptr, C, dig);
    }
    d_mark(a, c);  // head prep done
    d_units<LFK>(a, c, T.r[4], dig, 0, C, 0, logits, ga.d.V);
    d_mark(a, c);  // head done
    if (!d_gsync(a, c)) {
      alive = false;
      break;
    }
    if (ecm) {
      #pragma unroll 1
      for (int i = T.zc0 + t; i < T.zc1; i += kDT) fo64[i] = 0ull;
    } else {
      d_zero(acc_fo, T.zc0, T.zc1);
    }
    d_argmax_part(a, T, s_bv, s_bi);
    if (ga.ring_cancel && bx == 0 && t == 0) *ga.b.stop = cancel_seen;
    if (!d_gsync(a, c)) {
      alive = false;
      break;
    }
    tok = d_argmax_all(a, &s_tok);
    if (bx == 0 && t == 0) {
      ga.b.hist[step % ga.d.hist_cap] = tok;
      *ga.b.tok = tok;
      if (ga.ring_ids) {
        // one 32-bit store replaces the -1 the host left in the slot (the host
        // polls the slot itself, so no fence orders it with anything); the
        // count is exact once the launch has ended
        d_st_relaxed_sys(reinterpret_cast<unsigned*>(ga.ring_ids + step), (unsigned)tok);
        d_st_relaxed_sys(ga.ring_count, (unsigned)(step + 1));
      }
    }
    if (ga.ring_cancel && __ldcg(ga.b.stop)) {
      // cancelled by the host: every CTA stops after this token (the same
      // word, read after the same barrier); the producer sees the abort flag
      // in its slot waits, stops issuing and drains its copies in flight
      if (t == 0) s_abort = 1;
      break;
    }
  }
}

}  // namespace rwkvb
