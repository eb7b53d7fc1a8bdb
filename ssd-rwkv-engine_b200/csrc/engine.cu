// Fused RWKV-7 decode engine: one packed-model token step as a chain of phase
// kernels, launched with programmatic dependent launch (PDL) and captured in a
// CUDA graph.
//
// Per layer (mirrors forward_block_packed, packed_block_forward.py:76-166):
//   att_in  : ln1 + token-shift mixes (rwkv7_linear.py:165-171); r/k/v GEMVs;
//             first adapter projections (x @ W1, A1, G1, V1) as split-row
//             partial sums
//   wkv     : one CTA per head: second adapter projections for the head's
//             channels, kk-normalize, k update, v-first mix, decay, WKV7 state
//             update, GroupNorm, bonus, gate (rwkv7_linear.py:301-349)
//   att_out : output GEMV + residual; x_prev(att) <- ln1(x)
//   ffn_in  : ln2 + mix, key GEMV, relu^2 (rwkv7_linear.py:370-371, 409)
//   ffn_out : value GEMV + residual; x_prev(ffn) <- ln2(x)
// then head: ln_out + head GEMV + greedy argmax (first maximum).
//
// Data movement.  Weights never depend on the previous kernel, so every phase
// kernel starts its weight transfers (1-D TMA bulk copies into a shared-memory
// ring for the large SG8 projections, cp.async for the small adapter tiles)
// BEFORE `griddepcontrol.wait`; it then releases its dependent
// (`launch_dependents`) so the next phase can start its own transfers while
// this one computes.  Everything mutable (activations, recurrent state) is
// read and written only after the wait.
#include <atomic>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "stream.cuh"
#include "wkv7.cuh"

namespace rwkvb {

constexpr int kThreads = 256;
constexpr int kWkvThreads = 1024;
constexpr int kMaxPf = 8;
constexpr int kSlotBudget = 44 * 1024;
constexpr int kSlots = 4;
constexpr int kAdpRowsMax = 128;  // rows of a first-adapter matrix per CTA (upper bound)

struct Prefetch {
  const uint8_t* ptr[kMaxPf];
  uint64_t bytes[kMaxPf];
  uint64_t total;
  int n;
};

struct LayerDev {
  PackedView r, k, v, o, w1, w2, a1, a2, g1, g2, v1, v2, fk, fv;
  const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  const float *x_r, *x_w, *x_k, *x_v, *x_a, *x_g;
  const float *w0, *a0, *v0, *k_k, *k_a, *r_k, *lnx_w, *lnx_b, *ffn_x_k;
};

struct Bufs {
  float *att_x, *wkv, *ffn_x;  // recurrent state
  float *xa, *xb;              // residual stream (layer input / after attention)
  float *xln1, *xln2;          // normalised inputs kept for the state update
  float *rkv;                  // [3][C]
  float *adp;                  // [splits][Rtot] first-adapter partial sums
  float *att_y;                // [C]
  float *h;                    // [F]
  float *v_first;              // [C]
  float *logits;               // [V]
  float *ao, *fo;              // [C] attention / ffn output accumulators (persistent kernel)
  unsigned long long* adp64;   // [Rtot] first-adapter accumulators, 2^-32 fixed point (persistent kernel)
  unsigned long long* fo64;    // [C] ffn output accumulator, 2^-32 fixed point (persistent kernel, chunk-ordered E)
  float *amax_v;               // [grid] per-CTA argmax value
  int *amax_i;                 // [grid] per-CTA argmax index
  unsigned *ticket;            // last-CTA election for the argmax
  int *tok;                    // token consumed by the next step
  int *hist;                   // argmax history ring
  int *step;                   // steps since the last history reset
  int *err;                    // error flags (kErrToken | kErrTimeout)
  int *stop;                   // streamed decode: the host's cancel word as CTA 0 read it this token
};

struct Dims {
  int L, C, H, F, V;
  int rw, ra, rg, rv, rtot;  // adapter ranks, total
  int adp_splits, adp_rows;  // first-adapter row chunks (multi-kernel path)
  // persistent kernel: first-adapter items of adapter m (w, a, g, v) are
  // arow[m]-row chunks, numbered abase[m] .. abase[m + 1] - 1 (v last)
  int arow[4], abase[5];
  int hist_cap;
};

}  // namespace rwkvb
#include "decode.cuh"
namespace rwkvb {

// ------------------------------------------------------------ prefetch
__device__ __forceinline__ void issue_prefetch(const Prefetch& pf) {
  if (pf.n == 0 || threadIdx.x >= 32) return;
  const uint64_t b0 = pf.total * blockIdx.x / gridDim.x;
  const uint64_t b1 = pf.total * (blockIdx.x + 1) / gridDim.x;
  const unsigned lane = threadIdx.x;
  constexpr uint32_t kChunk = 32768;
  uint64_t base = 0;
  for (int r = 0; r < pf.n; ++r) {
    uint64_t lo = b0 > base ? b0 : base;
    uint64_t hi = b1 < base + pf.bytes[r] ? b1 : base + pf.bytes[r];
    if (lo < hi) {
      uintptr_t s = reinterpret_cast<uintptr_t>(pf.ptr[r]) + (lo - base);
      uintptr_t e = reinterpret_cast<uintptr_t>(pf.ptr[r]) + (hi - base);
      s = (s + 15) & ~(uintptr_t)15;
      e = e & ~(uintptr_t)15;
      for (uintptr_t p = s + (uintptr_t)lane * kChunk; p < e; p += 32u * kChunk) {
        uint32_t n = (uint32_t)((e - p) < kChunk ? (e - p) : kChunk);
        prefetch_l2_bulk(reinterpret_cast<const void*>(p), n);
      }
    }
    base += pf.bytes[r];
  }
}

// In-place LayerNorm of buf[0..C) (shared, already staged): two-pass mean /
// variance, eps 1e-5 (F.layer_norm, packed_block_forward.py:94-98).
__device__ __forceinline__ void layer_norm_inplace(float* buf, const float* w, const float* b, int C, float* red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) s += buf[i];
  const float mean = block_sum(s, red) / (float)C;
  float q = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const float d = buf[i] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(block_sum(q, red) / (float)C + 1e-5f);
  stage4(buf, C >> 2, [&](int i) {
    const float4 x = reinterpret_cast<const float4*>(buf)[i];
    const float4 ww = ldg4(w + 4 * i), bb = ldg4(b + 4 * i);
    return make_float4((x.x - mean) * rstd * ww.x + bb.x, (x.y - mean) * rstd * ww.y + bb.y,
                       (x.z - mean) * rstd * ww.z + bb.z, (x.w - mean) * rstd * ww.w + bb.w);
  });
}

// buf = LayerNorm(x) for a mutable global vector x (read through L2).
__device__ __forceinline__ void layer_norm_global(const float* x, const float* w, const float* b, int C, float* buf,
                                                  float* red) {
  stage4(buf, C >> 2, [&](int i) { return ldcg4(x + 4 * i); });
  layer_norm_inplace(buf, w, b, C, red);
}

// buf = buf + (prev - buf) * mix, in place (token shift, rwkv7_linear.py:165-171).
__device__ __forceinline__ void token_mix_inplace(float* buf, const float* prev, const float* mix, int C) {
  stage4(buf, C >> 2, [&](int i) {
    const float4 z = reinterpret_cast<const float4*>(buf)[i];
    const float4 p = ldcg4(prev + 4 * i), m = ldg4(mix + 4 * i);
    return make_float4(z.x + (p.x - z.x) * m.x, z.y + (p.y - z.y) * m.y, z.z + (p.z - z.z) * m.z,
                       z.w + (p.w - z.w) * m.w);
  });
}

__device__ __forceinline__ void store_vec(float* dst, const float* src, int C) {
  for (int i = threadIdx.x; i < (C >> 2); i += blockDim.x)
    reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
}

// Shared-memory carve-up for ring phases: [ring slots][bars][partials][vec][resid]
struct RingLayout {
  uint32_t slots_off, bars_off, part_off, vec_off, res_off, total;
};

__host__ inline RingLayout ring_layout(const RingPlan& P, int vec_floats, int res_floats) {
  RingLayout L;
  L.slots_off = 0;
  L.bars_off = (uint32_t)P.nst * P.slot_bytes;
  L.bars_off = (L.bars_off + 15) & ~15u;
  L.part_off = L.bars_off + 8 * kSlots;
  L.vec_off = L.part_off + (uint32_t)(2 * P.rs * P.nseg * 4);
  L.vec_off = (L.vec_off + 15) & ~15u;
  L.res_off = L.vec_off + (uint32_t)vec_floats * 4;
  L.res_off = (L.res_off + 15) & ~15u;
  L.total = L.res_off + (uint32_t)res_floats * 4 + 16;
  return L;
}

__device__ __forceinline__ RingSmem ring_smem(uint8_t* base, const RingLayout& L) {
  RingSmem S;
  S.slots = base + L.slots_off;
  S.bars = reinterpret_cast<uint64_t*>(base + L.bars_off);
  S.part = reinterpret_cast<float*>(base + L.part_off);
  return S;
}

template <class XIn, class Epi>
__device__ __forceinline__ bool ring_dispatch(int cpl, const PackedView& W, const RingPlan& P, const RingSmem& S,
                                              XIn xin, Epi epi, int* err) {
  switch (cpl) {
    case 1: return ring_run<1>(W, P, S, xin, epi, err);
    case 2: return ring_run<2>(W, P, S, xin, epi, err);
    case 3: return ring_run<3>(W, P, S, xin, epi, err);
    case 4: return ring_run<4>(W, P, S, xin, epi, err);
    default: return ring_run<5>(W, P, S, xin, epi, err);
  }
}

// ------------------------------------------------------------- embed
struct EmbedArgs {
  PackedView emb;
  const float *ln0_w, *ln0_b;
  Bufs b;
  Dims d;
  Prefetch pf;
  int fast;  // SG8 rows with whole groups, 16-byte aligned: stage the row with cp.async
};

__global__ void __launch_bounds__(kThreads) embed_kernel(EmbedArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) uint8_t smb[];
  pdl_launch_dependents();
  issue_prefetch(a.pf);
  pdl_wait();
  const int C = a.d.C;
  int tok = __ldcg(a.b.tok);
  if (tok < 0 || tok >= a.d.V) {
    if (threadIdx.x == 0) atomicOr(a.b.err, kErrToken);
    tok = 0;
  }
  float* row = reinterpret_cast<float*>(smb);
  if (a.fast) {
    uint8_t* q = smb + (size_t)C * 4;
    float2* sc = reinterpret_cast<float2*>(q + C);
    const int gpr = C >> a.emb.lg;
    cp_async_block(q, a.emb.payload + (size_t)tok * C, (uint32_t)C);
    cp_async_block(sc, a.emb.meta + (size_t)tok * gpr * 8, (uint32_t)gpr * 8u);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
      const float2 s = sc[i >> a.emb.lg];
      row[i] = sg8_dequant(q[i], s.x, s.y);
    }
  } else {
    for (int i = threadIdx.x; i < C; i += blockDim.x) row[i] = packed_at(a.emb, tok, i);
  }
  __syncthreads();
  layer_norm_inplace(row, a.ln0_w, a.ln0_b, C, red);
  store_vec(a.b.xa, row, C);
}

// ------------------------------------------------------------ att_in
struct AttInArgs {
  LayerDev l;
  Bufs b;
  Dims d;
  Prefetch pf;
  RingPlan plan;      // row range resolved per CTA
  RingLayout lay;
  int cpl;
  int ring;           // 1: ring path for r/k/v; 0: direct loads
  int gm;             // CTAs per matrix (r, k, v)
  int mode[3], lg[3]; // direct-path modes
  int layer;
};

__global__ void __launch_bounds__(kThreads, 2) att_in_kernel(AttInArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) uint8_t smb[];
  const int C = a.d.C;
  const float* prev = a.b.att_x + (size_t)a.layer * C;
  if ((int)blockIdx.x < 3 * a.gm) {
    const int m = blockIdx.x / a.gm, cb = blockIdx.x % a.gm;
    const PackedView& W = m == 0 ? a.l.r : (m == 1 ? a.l.k : a.l.v);
    const float* mix = m == 0 ? a.l.x_r : (m == 1 ? a.l.x_k : a.l.x_v);
    float* out = a.b.rkv + (size_t)m * C;
    RingPlan P = a.plan;
    P.row0 = cb * a.plan.row1;  // plan.row1 holds rows per CTA
    P.row1 = min(C, P.row0 + a.plan.row1);
    RingSmem S = ring_smem(smb, a.lay);
    float* xv = reinterpret_cast<float*>(smb + a.lay.vec_off);
    if (a.ring && P.row0 < P.row1) ring_start(W, P, S);
    pdl_launch_dependents();
    issue_prefetch(a.pf);
    pdl_wait();
    layer_norm_global(a.b.xa, a.l.ln1_w, a.l.ln1_b, C, xv, red);
    if (blockIdx.x == 0) store_vec(a.b.xln1, xv, C);
    __syncthreads();
    if (P.row0 >= P.row1) return;
    token_mix_inplace(xv, prev, mix, C);
    if (a.ring) {
      ring_dispatch(a.cpl, W, P, S, [&](int i) { return *reinterpret_cast<const float4*>(xv + i); },
                    [&](int row, float v) { out[row] = v; }, a.b.err);
    } else {
      float* sxc = xv + C;
      if (a.mode[m] == 1) {
        stage_input(C, xv, sxc, [&](int i) { return xv[i]; });
      }
      packed_rows(W, a.mode[m], a.lg[m], xv, sxc, P.row0, P.row1, [&](int row, float v) { out[row] = v; });
    }
    return;
  }
  // first adapter projections: work item = (matrix, chunk of adp_rows rows)
  const int item = blockIdx.x - 3 * a.gm;
  const bool active = item < (a.layer == 0 ? 3 : 4) * a.d.adp_splits;
  const int m = item / a.d.adp_splits, s = item % a.d.adp_splits;
  const PackedView& W = m == 0 ? a.l.w1 : (m == 1 ? a.l.a1 : (m == 2 ? a.l.g1 : a.l.v1));
  const float* mix = m == 0 ? a.l.x_w : (m == 1 ? a.l.x_a : (m == 2 ? a.l.x_g : a.l.x_v));
  const int off = m == 0 ? 0 : (m == 1 ? a.d.rw : (m == 2 ? a.d.rw + a.d.ra : a.d.rw + a.d.ra + a.d.rg));
  const int R = W.cols;
  const int i0 = s * a.d.adp_rows, i1 = min(C, i0 + a.d.adp_rows);
  float* xv = reinterpret_cast<float*>(smb);
  uint8_t* tq = smb + (size_t)C * 4;                                   // codes [rows][R]
  float2* tsc = reinterpret_cast<float2*>(tq + kAdpRowsMax * R + 16);  // scale pairs
  const bool tiled = W.kind == RWKVB_KIND_SG8 && W.lg >= 0 && (R % 16) == 0 &&
                     ((reinterpret_cast<uintptr_t>(W.payload) & 15u) == 0);
  uint32_t g0 = 0, ng = 0;
  if (active && tiled && i0 < i1) {
    // codes with cp.async (16B pieces), scale pairs with plain 8-byte loads
    cp_async_block(tq, W.payload + (size_t)i0 * R, (uint32_t)((i1 - i0) * R));
    cp_async_commit();
    g0 = (uint32_t)(((uint64_t)i0 * R) >> W.lg);
    ng = (uint32_t)((((uint64_t)i1 * R - 1) >> W.lg) - g0 + 1);
    for (uint32_t j = threadIdx.x; j < ng; j += blockDim.x)
      tsc[j] = __ldg(reinterpret_cast<const float2*>(W.meta) + g0 + j);
  }
  pdl_launch_dependents();
  pdl_wait();
  if (!active) return;
  layer_norm_global(a.b.xa, a.l.ln1_w, a.l.ln1_b, C, xv, red);
  token_mix_inplace(xv, prev, mix, C);
  if (tiled) cp_async_wait_all();
  __syncthreads();
  float* outp = a.b.adp + (size_t)s * a.d.rtot + off;
  for (int j = threadIdx.x; j < R; j += blockDim.x) {
    float acc = 0.f;
    if (tiled) {
      for (int i = i0; i < i1; ++i) {
        const uint32_t e = (uint32_t)i * (uint32_t)R + (uint32_t)j;
        const float2 sc = tsc[(e >> W.lg) - g0];
        acc = fmaf(xv[i], sg8_dequant(tq[(i - i0) * R + j], sc.x, sc.y), acc);
      }
    } else {
      for (int i = i0; i < i1; ++i) acc = fmaf(xv[i], packed_at(W, i, j), acc);
    }
    outp[j] = acc;
  }
}

// --------------------------------------------------------------- wkv
struct WkvArgs {
  LayerDev l;
  Bufs b;
  Dims d;
  Prefetch pf;
  int layer;
  int tiled;  // second-adapter tiles staged with cp.async (SG8, group >= 64)
};

__global__ void __launch_bounds__(kWkvThreads) wkv_kernel(WkvArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) uint8_t smb[];
  const int h = blockIdx.x, C = a.d.C, t = threadIdx.x;
  const int nm = a.layer == 0 ? 3 : 4;
  float* S = reinterpret_cast<float*>(smb);                          // [64][64] state
  float* mid = S + 4096;                                            // [rtot]
  float* vec = mid + ((a.d.rtot + 3) & ~3);                         // 4 x 64
  float* sr = vec + 256;
  float* sd = sr + 64;
  float* sk = sd + 64;
  float* sv = sk + 64;
  float* skk = sv + 64;
  float* ska = skk + 64;
  float* sy = ska + 64;
  float2* tsc = reinterpret_cast<float2*>(sy + 64);                 // [rtot] scale pair per row
  uint8_t* tq = reinterpret_cast<uint8_t*>(tsc + a.d.rtot);         // [rtot][64] codes
  // constant weights first: this head's 64 columns of W2/A2/G2/V2
  if (a.tiled) {
    int off = 0;
    for (int m = 0; m < nm; ++m) {
      const PackedView& W = m == 0 ? a.l.w2 : (m == 1 ? a.l.a2 : (m == 2 ? a.l.g2 : a.l.v2));
      for (int u = t; u < W.rows * 4; u += blockDim.x) {
        const int i = u >> 2, p = u & 3;
        cp_async16(tq + (size_t)(off + i) * 64 + p * 16, W.payload + (size_t)i * C + h * 64 + p * 16);
      }
      for (int i = t; i < W.rows; i += blockDim.x)
        tsc[off + i] = __ldg(reinterpret_cast<const float2*>(W.meta) + (((size_t)i * C + h * 64) >> W.lg));
      off += W.rows;
    }
    cp_async_commit();
  }
  pdl_launch_dependents();
  issue_prefetch(a.pf);
  pdl_wait();
  // this head's recurrent state
  float* Sg = a.b.wkv + ((size_t)a.layer * a.d.H + h) * 4096;
  for (int u = t; u < 1024; u += blockDim.x) cp_async16(S + u * 4, Sg + u * 4);
  cp_async_commit();
  // reduce the first-projection partial sums (fixed order, loads batched) and activate
  const int used = a.layer == 0 ? a.d.rw + a.d.ra + a.d.rg : a.d.rtot;
  for (int j = t; j < used; j += blockDim.x) {
    float acc = 0.f;
    for (int s0 = 0; s0 < a.d.adp_splits; s0 += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = s0 + u < a.d.adp_splits ? __ldcg(a.b.adp + (size_t)(s0 + u) * a.d.rtot + j) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += v[u];
    }
    if (j < a.d.rw) acc = tanhf(acc);
    else if (j >= a.d.rw + a.d.ra && j < a.d.rw + a.d.ra + a.d.rg) acc = sigmoidf_(acc);
    mid[j] = acc;
  }
  // per-channel activations of this head (threads 0..63), loaded while the copies land
  float r = 0.f, k = 0.f, v = 0.f, vf = 0.f;
  if (t < 64) {
    const int ch = h * 64 + t;
    r = __ldcg(a.b.rkv + ch);
    k = __ldcg(a.b.rkv + C + ch);
    v = __ldcg(a.b.rkv + 2 * C + ch);
    if (a.layer != 0) vf = __ldcg(a.b.v_first + ch);
  }
  cp_async_wait_all();
  __syncthreads();
  // second projections for the head's 64 channels: thread -> (matrix, channel, quarter)
  {
    const int q = t & 3, c = (t >> 2) & 63, m = t >> 8;
    const int off = m == 0 ? 0 : (m == 1 ? a.d.rw : (m == 2 ? a.d.rw + a.d.ra : a.d.rw + a.d.ra + a.d.rg));
    const int R = m == 0 ? a.d.rw : (m == 1 ? a.d.ra : (m == 2 ? a.d.rg : a.d.rv));
    float acc = 0.f;
    if (m < nm) {
      if (a.tiled) {
        for (int i = q; i < R; i += 4) {
          const float2 sc = tsc[off + i];
          acc = fmaf(mid[off + i], sg8_dequant(tq[(size_t)(off + i) * 64 + c], sc.x, sc.y), acc);
        }
      } else {
        const PackedView& W = m == 0 ? a.l.w2 : (m == 1 ? a.l.a2 : (m == 2 ? a.l.g2 : a.l.v2));
        for (int i = q; i < R; i += 4) acc = fmaf(mid[off + i], packed_at(W, i, h * 64 + c), acc);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (q == 0 && m < nm) vec[m * 64 + c] = acc;
  }
  __syncthreads();
  const float kkv = t < 64 ? k * a.l.k_k[h * 64 + t] : 0.f;
  const float nrm = sqrtf(block_sum(kkv * kkv, red));
  if (t < 64) {
    const int ch = h * 64 + t;
    const float aa = sigmoidf_(a.l.a0[ch] + vec[64 + t]);
    const float kk = kkv / fmaxf(nrm, 1e-12f);
    const float kn = k * (1.0f + (aa - 1.0f) * a.l.k_a[ch]);
    if (a.layer == 0) {
      a.b.v_first[ch] = v;
    } else {
      v = v + (vf - v) * sigmoidf_(a.l.v0[ch] + vec[192 + t]);
    }
    sr[t] = r;
    sd[t] = expf(-0.606531f * sigmoidf_(a.l.w0[ch] + vec[t]));
    sk[t] = kn;
    sv[t] = v;
    skk[t] = kk;
    ska[t] = kk * aa;
  }
  __syncthreads();
  if (t < 256) wkv7_head64(S, sr, sd, sk, sv, skk, ska, sy);
  __syncthreads();
  for (int u = t; u < 1024; u += blockDim.x)
    reinterpret_cast<float4*>(Sg)[u] = reinterpret_cast<const float4*>(S)[u];
  // GroupNorm over the head (eps 64e-5), bonus, gate
  const float yv = t < 64 ? sy[t] : 0.f;
  const float mean = block_sum(yv, red) / 64.f;
  const float dv = t < 64 ? yv - mean : 0.f;
  const float var = block_sum(dv * dv, red) / 64.f;
  const float bon = t < 64 ? sr[t] * sk[t] * a.l.r_k[h * 64 + t] : 0.f;
  const float bonus = block_sum(bon, red);
  if (t < 64) {
    const int ch = h * 64 + t;
    float o = dv * rsqrtf(var + 64e-5f) * a.l.lnx_w[ch] + a.l.lnx_b[ch];
    o = o + bonus * sv[t];
    a.b.att_y[ch] = o * vec[128 + t];
  }
}

// ------------------------------------------------------ GEMV phases
// kinds: 0 att_out, 1 ffn_in, 2 ffn_out, 3 head
struct PhaseArgs {
  PackedView w;
  RingPlan plan;
  RingLayout lay;
  int cpl, ring, mode, lg;
  int kind;
  int layer;
  const float *ln_w, *ln_b, *mixv;
  Prefetch pf;
  Bufs b;
  Dims d;
};

__global__ void __launch_bounds__(kThreads, 2) phase_kernel(PhaseArgs a) {
  __shared__ float red[32];
  __shared__ float bv[kThreads / 32];
  __shared__ int bi[kThreads / 32];
  extern __shared__ __align__(16) uint8_t smb[];
  const int K = a.w.cols, C = a.d.C;
  RingPlan P = a.plan;
  P.row0 = blockIdx.x * a.plan.row1;
  P.row1 = min(a.w.rows, P.row0 + a.plan.row1);
  RingSmem S = ring_smem(smb, a.lay);
  float* xv = reinterpret_cast<float*>(smb + a.lay.vec_off);
  float* rsd = reinterpret_cast<float*>(smb + a.lay.res_off);
  if (a.ring && P.row0 < P.row1) ring_start(a.w, P, S);
  pdl_launch_dependents();
  issue_prefetch(a.pf);
  pdl_wait();
  const Bufs& b = a.b;
  const int kind = a.kind;
  // input vector, staged once into shared memory
  const float* gsrc = kind == 0 ? b.att_y : b.h;
  if (kind == 0 || kind == 2) {
    if (!a.ring) stage4(xv, K >> 2, [&](int i) { return ldcg4(gsrc + 4 * i); });
  } else {
    layer_norm_global(kind == 1 ? b.xb : b.xa, a.ln_w, a.ln_b, K, xv, red);
    if (kind == 1) {
      if (blockIdx.x == 0) store_vec(b.xln2, xv, K);
      __syncthreads();
      token_mix_inplace(xv, b.ffn_x + (size_t)a.layer * C, a.mixv, K);
    }
  }
  const int nr = P.row1 - P.row0;
  if (nr <= 0) return;
  // residual rows and recurrent-state copies for this CTA's rows
  if (kind == 0 || kind == 2) {
    const float* res = kind == 0 ? b.xa : b.xb;
    const float* ln = kind == 0 ? b.xln1 : b.xln2;
    float* st = (kind == 0 ? b.att_x : b.ffn_x) + (size_t)a.layer * C;
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
      rsd[i] = __ldcg(res + P.row0 + i);
      st[P.row0 + i] = __ldcg(ln + P.row0 + i);
    }
    __syncthreads();
  }
  float best = -INFINITY;
  int besti = 0x7fffffff;
  const int r0 = P.row0;
  auto epi = [&](int row, float v) {
    if (kind == 0) b.xb[row] = rsd[row - r0] + v;
    else if (kind == 1) b.h[row] = v > 0.f ? v * v : 0.f;
    else if (kind == 2) b.xa[row] = rsd[row - r0] + v;
    else {
      b.logits[row] = v;
      if (v > best || (v == best && row < besti)) { best = v; besti = row; }
    }
  };
  if (a.ring) {
    if (kind == 0 || kind == 2)
      ring_dispatch(a.cpl, a.w, P, S, [&](int i) { return ldcg4(gsrc + i); }, epi, b.err);
    else
      ring_dispatch(a.cpl, a.w, P, S, [&](int i) { return *reinterpret_cast<const float4*>(xv + i); }, epi, b.err);
  } else {
    float* sxc = xv + K;
    if (a.mode == 1) stage_input(K, xv, sxc, [&](int i) { return xv[i]; });
    packed_rows(a.w, a.mode, a.lg, xv, sxc, P.row0, P.row1, epi);
  }
  if (kind != 3) return;
  // per-CTA argmax, then the last CTA to finish reduces and records the token
  float wb = best;
  int wi = besti;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, wb, o);
    const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
    if (ov > wb || (ov == wb && oi < wi)) { wb = ov; wi = oi; }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { bv[wid] = wb; bi[wid] = wi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float cb = -INFINITY;
    int ci = 0x7fffffff;
    for (int w = 0; w < kThreads / 32; ++w)
      if (bv[w] > cb || (bv[w] == cb && bi[w] < ci)) { cb = bv[w]; ci = bi[w]; }
    b.amax_v[blockIdx.x] = cb;
    b.amax_i[blockIdx.x] = ci;
    __threadfence();
    const unsigned prevt = atomicAdd(b.ticket, 1u);
    if (prevt == gridDim.x - 1) {
      __threadfence();
      float gb = -INFINITY;
      int gi = 0x7fffffff;
      for (unsigned c = 0; c < gridDim.x; ++c) {
        const float v = __ldcg(b.amax_v + c);
        const int i = __ldcg(b.amax_i + c);
        if (v > gb || (v == gb && i < gi)) { gb = v; gi = i; }
      }
      if (gi == 0x7fffffff) gi = 0;  // every logit NaN
      *b.tok = gi;
      const int st = *b.step;
      b.hist[st % a.d.hist_cap] = gi;
      *b.step = st + 1;
      *b.ticket = 0u;
    }
  }
}

__global__ void set_token_kernel(int* tok, int value, int* step, int reset_step) {
  *tok = value;
  if (reset_step) *step = 0;
}

}  // namespace rwkvb

using namespace rwkvb;

// =================================================================== engine
struct rwkvb_engine {
  int dev = 0;
  int sms = 148;
  uint32_t flags = 0;
  int pf_dist = 0;
  bool pdl = true;
  Dims d{};
  std::vector<LayerDev> layers;
  PackedView emb{}, head{};
  const float *ln0_w = nullptr, *ln0_b = nullptr, *lnout_w = nullptr, *lnout_b = nullptr;
  Bufs b{};
  void* arena = nullptr;
  int head_grid = 0;
  std::vector<Prefetch> phase_pf;  // weights of each phase, in step order
  cudaStream_t cap = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int launches = 0;
  // persistent path
  bool persistent = false;
  DArgs da{};
  int lfk = 2;
  size_t dsmem = 0;
  DLayerMaps* dmaps = nullptr;
  CUtensorMap* dhead = nullptr;
  LayerDev* dlayers = nullptr;
  int* dtokens = nullptr;  // forced-token staging [hist_cap]
  unsigned long long* dtrace = nullptr;  // phase timestamps (flag bit 3)
  int trace_cap = 0;
  // streamed decode: mapped pinned host ring (count at +0, cancel at +64, ids at +128)
  uint8_t* hring = nullptr;
  uint8_t* hring_dev = nullptr;  // the same memory as the device addresses it
  uint8_t* dstream = nullptr;    // streaming copy of the big matrices (persistent kernel)
  // staged layers (rwkvb_engine_create_staged): layer li is streamed when
  // stage_slot[li] >= 0; its image (stage_bytes) is copied from pinned host
  // memory into device slot stage_slot[li] on the copy stream before the
  // layer's kernels, after the slot's previous user in the step is done
  bool staged = false;
  std::vector<int> stage_slot;
  std::vector<const void*> stage_src;
  std::vector<void*> stage_dev;
  uint64_t stage_bytes = 0;
  cudaStream_t copy = nullptr;
  cudaEvent_t ev_fork = nullptr;
  std::vector<cudaEvent_t> ev_loaded, ev_done;  // per streamed layer, in step order
};

namespace {

LayerDev make_layer(const rwkvb_layer_desc& s) {
  LayerDev l;
  l.r = make_view(s.att_r); l.k = make_view(s.att_k); l.v = make_view(s.att_v); l.o = make_view(s.att_o);
  l.w1 = make_view(s.w1); l.w2 = make_view(s.w2); l.a1 = make_view(s.a1); l.a2 = make_view(s.a2);
  l.g1 = make_view(s.g1); l.g2 = make_view(s.g2);
  l.v1 = s.v1.data ? make_view(s.v1) : make_view(s.w1);
  l.v2 = s.v2.data ? make_view(s.v2) : make_view(s.w2);
  l.fk = make_view(s.ffn_key); l.fv = make_view(s.ffn_value);
  l.ln1_w = s.ln1_w; l.ln1_b = s.ln1_b; l.ln2_w = s.ln2_w; l.ln2_b = s.ln2_b;
  l.x_r = s.x_r; l.x_w = s.x_w; l.x_k = s.x_k; l.x_v = s.x_v; l.x_a = s.x_a; l.x_g = s.x_g;
  l.w0 = s.w0; l.a0 = s.a0; l.v0 = s.v0; l.k_k = s.k_k; l.k_a = s.k_a; l.r_k = s.r_k;
  l.lnx_w = s.lnx_w; l.lnx_b = s.lnx_b; l.ffn_x_k = s.ffn_x_k;
  return l;
}

bool desc_ok(const rwkvb_packed& p, int rows, int cols) {
  return p.data && p.rows == rows && p.cols == cols && p.group_size > 0 &&
         (p.kind == RWKVB_KIND_SG8 || (p.kind >= 3 && p.kind <= 7) || p.kind == RWKVB_KIND_LUT2_TENSOR);
}

void pf_add(Prefetch& pf, const rwkvb_packed& p) {
  if (pf.n < kMaxPf && p.data) {
    pf.ptr[pf.n] = p.data;
    pf.bytes[pf.n] = p.bytes;
    pf.total += p.bytes;
    ++pf.n;
  }
}

Prefetch pf_empty() {
  Prefetch p;
  memset(&p, 0, sizeof(p));
  return p;
}

void pf_cap(Prefetch& pf, uint64_t cap) {
  uint64_t tot = 0;
  for (int i = 0; i < pf.n; ++i) {
    if (tot + pf.bytes[i] > cap) {
      pf.bytes[i] = cap > tot ? cap - tot : 0;
      pf.n = i + 1;
      tot += pf.bytes[i];
      break;
    }
    tot += pf.bytes[i];
  }
  pf.total = tot;
}

template <class Arg>
cudaError_t launch(void (*k)(Arg), int grid, int block, size_t smem, cudaStream_t s, bool pdl, const Arg& arg) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, arg);
}

// Phase plan for a packed GEMV over `ctas` CTAs: ring when the layout allows.
// Shared memory: ring slots, the staged input vector (K floats, plus 16-wide
// chunk sums on the direct path) and the CTA's residual rows.
void plan_phase(const PackedView& w, int ctas, bool ln_input, RingPlan* plan, RingLayout* lay, int* cpl, int* ring,
                int* mode, int* lg, size_t* smem) {
  memset(plan, 0, sizeof(*plan));
  *mode = gemv_mode(w);
  *lg = ilog2u(w.group);
  const int K = w.cols;
  *ring = ring_plan(w, ctas, kSlotBudget, kSlots, cpl, plan) ? 1 : 0;
  if (!*ring) {
    *cpl = 0;
    plan->row1 = (w.rows + ctas - 1) / ctas;
    plan->nst = kSlots;
    plan->rs = 1;
    plan->nseg = 1;
    plan->slot_bytes = 0;
  }
  const int rpc = plan->row1;
  const int vecf = *ring ? (ln_input ? K : 0) : K + K / 16 + 8;
  *lay = ring_layout(*plan, vecf, (rpc + 3) & ~3);
  // two CTAs per SM: shrink the ring until both fit (227 KB per SM)
  while (*ring && plan->nst > 2 && lay->total > 110 * 1024) {
    plan->nst -= 1;
    *lay = ring_layout(*plan, vecf, (rpc + 3) & ~3);
  }
  *smem = lay->total;
}

int record_step(rwkvb_engine* e, cudaStream_t s) {
  const Dims& d = e->d;
  const int P = (int)e->phase_pf.size();
  int phase = 0;
  auto pf_for = [&](int p) {
    if (e->pf_dist <= 0) return pf_empty();
    return e->phase_pf[(p + e->pf_dist) % P];
  };
  cudaError_t err = cudaSuccess;
  auto chk = [&](cudaError_t x) { if (err == cudaSuccess && x != cudaSuccess) err = x; };
  e->launches = 0;
  // staged layers: the copy stream forks from the step's stream, so the
  // copies belong to the same step (and to its CUDA graph when captured)
  const int nslots = (int)e->stage_dev.size();
  int sj = 0;  // streamed layers met so far
  if (e->staged) {
    chk(cudaEventRecord(e->ev_fork, s));
    chk(cudaStreamWaitEvent(e->copy, e->ev_fork, 0));
  }
  auto stage_in = [&](int li) {  // before layer li's kernels
    if (!e->staged || e->stage_slot[li] < 0) return;
    const int slot = e->stage_slot[li];
    if (sj >= nslots) chk(cudaStreamWaitEvent(e->copy, e->ev_done[sj - nslots], 0));  // slot's previous user done
    chk(cudaMemcpyAsync(e->stage_dev[slot], e->stage_src[li], e->stage_bytes, cudaMemcpyHostToDevice, e->copy));
    chk(cudaEventRecord(e->ev_loaded[sj], e->copy));
    chk(cudaStreamWaitEvent(s, e->ev_loaded[sj], 0));
  };
  auto stage_out = [&](int li) {  // after layer li's kernels
    if (!e->staged || e->stage_slot[li] < 0) return;
    chk(cudaEventRecord(e->ev_done[sj], s));
    ++sj;
  };
  {
    EmbedArgs a;
    a.emb = e->emb; a.ln0_w = e->ln0_w; a.ln0_b = e->ln0_b; a.b = e->b; a.d = d; a.pf = pf_for(phase++);
    const PackedView& w = e->emb;
    const int gpr = w.lg >= 0 ? d.C >> w.lg : 1;
    a.fast = w.kind == RWKVB_KIND_SG8 && w.lg >= 4 && (d.C % (int)w.group) == 0 && gpr % 2 == 0 &&
             (reinterpret_cast<uintptr_t>(w.payload) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w.meta) & 15u) == 0;
    const size_t smem = (size_t)d.C * 5 + (size_t)gpr * 8 + 64;
    chk(launch(embed_kernel, 1, kThreads, smem, s, e->pdl, a));
    ++e->launches;
  }
  const int gm = (2 * e->sms) / 3 > 0 ? (2 * e->sms) / 3 : 1;
  for (int li = 0; li < d.L; ++li) {
    const LayerDev& l = e->layers[li];
    stage_in(li);
    {
      AttInArgs a;
      memset(&a, 0, sizeof(a));
      a.l = l; a.b = e->b; a.d = d; a.pf = pf_for(phase++); a.layer = li; a.gm = gm;
      size_t smem = 0;
      int mode = 0, lg = 0;
      plan_phase(l.r, gm, true, &a.plan, &a.lay, &a.cpl, &a.ring, &mode, &lg, &smem);
      const PackedView* mats[3] = {&l.r, &l.k, &l.v};
      for (int m = 0; m < 3; ++m) { a.mode[m] = gemv_mode(*mats[m]); a.lg[m] = ilog2u(mats[m]->group); }
      const int maxr = d.rw > d.ra ? (d.rw > d.rg ? d.rw : d.rg) : (d.ra > d.rg ? d.ra : d.rg);
      const int maxr2 = maxr > d.rv ? maxr : d.rv;
      const size_t adp_smem = (size_t)d.C * 4 + (size_t)kAdpRowsMax * maxr2 + 16 + 8 * ((size_t)kAdpRowsMax * maxr2 / 16 + 4);
      if (adp_smem > smem) smem = adp_smem;
      const int items = 4 * d.adp_splits;
      chk(launch(att_in_kernel, 3 * gm + items, kThreads, smem, s, e->pdl, a));
    }
    {
      WkvArgs a;
      a.l = l; a.b = e->b; a.d = d; a.pf = pf_for(phase++); a.layer = li;
      const PackedView* w2s[4] = {&l.w2, &l.a2, &l.g2, &l.v2};
      a.tiled = 1;
      for (int m = 0; m < 4; ++m) {
        const PackedView& w = *w2s[m];
        if (!(w.kind == RWKVB_KIND_SG8 && w.lg >= 6 && (d.C % (int)w.group) == 0 &&
              (reinterpret_cast<uintptr_t>(w.payload) & 15u) == 0))
          a.tiled = 0;
      }
      const size_t smem = (size_t)(4096 + ((d.rtot + 3) & ~3) + 256 + 7 * 64) * 4 + (size_t)d.rtot * 8 +
                          (size_t)d.rtot * 64 + 64;
      chk(launch(wkv_kernel, d.H, kWkvThreads, smem, s, e->pdl, a));
    }
    const PackedView* ws[3] = {&l.o, &l.fk, &l.fv};
    for (int k = 0; k < 3; ++k) {
      PhaseArgs a;
      memset(&a, 0, sizeof(a));
      a.w = *ws[k];
      a.kind = k;
      a.layer = li;
      a.ln_w = k == 1 ? l.ln2_w : nullptr;
      a.ln_b = k == 1 ? l.ln2_b : nullptr;
      a.mixv = k == 1 ? l.ffn_x_k : nullptr;
      a.pf = pf_for(phase++);
      a.b = e->b;
      a.d = d;
      size_t smem = 0;
      plan_phase(a.w, 2 * e->sms, k == 1, &a.plan, &a.lay, &a.cpl, &a.ring, &a.mode, &a.lg, &smem);
      const int grid = (a.w.rows + a.plan.row1 - 1) / a.plan.row1;
      chk(launch(phase_kernel, grid, kThreads, smem, s, e->pdl, a));
    }
    e->launches += 5;
    stage_out(li);
  }
  {
    PhaseArgs a;
    memset(&a, 0, sizeof(a));
    a.w = e->head; a.kind = 3; a.ln_w = e->lnout_w; a.ln_b = e->lnout_b;
    a.pf = pf_for(phase++); a.b = e->b; a.d = d;
    size_t smem = 0;
    plan_phase(a.w, e->head_grid, true, &a.plan, &a.lay, &a.cpl, &a.ring, &a.mode, &a.lg, &smem);
    const int grid = (a.w.rows + a.plan.row1 - 1) / a.plan.row1;
    chk(launch(phase_kernel, grid, kThreads, smem, s, e->pdl, a));
    ++e->launches;
  }
  return cuda_status(err != cudaSuccess ? err : cudaGetLastError());
}

int ensure_graph(rwkvb_engine* e) {
  if (e->exec || (e->flags & 1u)) return RWKVB_OK;
  cudaError_t err = cudaStreamBeginCapture(e->cap, cudaStreamCaptureModeThreadLocal);
  if (err != cudaSuccess) return cuda_status(err);
  int st = record_step(e, e->cap);
  cudaGraph_t g = nullptr;
  err = cudaStreamEndCapture(e->cap, &g);
  if (st != RWKVB_OK || err != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return st != RWKVB_OK ? st : cuda_status(err);
  }
  err = cudaGraphInstantiate(&e->exec, g, 0);
  if (err != cudaSuccess) {
    cudaGraphDestroy(g);
    e->exec = nullptr;
    return cuda_status(err);
  }
  e->graph = g;
  return RWKVB_OK;
}

int run_step(rwkvb_engine* e, cudaStream_t s) {
  if (e->flags & 1u) return record_step(e, s);
  return cuda_status(cudaGraphLaunch(e->exec, s));
}


// ---------------------------------------------------------- persistent plan
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Streaming copy of one SG8 matrix [rows][K] for the persistent kernel.  Unit u
// = (16-row tile u / nch, column chunk u % nch of kc = nb * 128 columns) is
// stored as the shared-memory image its ring slot receives from the two
// tensor-map copies it replaces: codes [nb blocks][16 rows][128 B] with the
// 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)), then the
// rows' (min, max) pairs of the chunk, [16][pr] float2.  Rows past the matrix
// are zero (min = max = 0: they contribute nothing).  One block per unit.
__global__ void stream_layout_kernel(uint8_t* dst, PackedView w, int nb, int pr, uint32_t unit_b, int units) {
  const int u = blockIdx.x;
  if (u >= units) return;
  const int K = w.cols, kc = nb * 128, nch = K / kc;
  const int tile = u / nch, ch = u - tile * nch;
  uint8_t* out = dst + (size_t)u * unit_b;
  for (int i = threadIdx.x; i < 16 * nb * 8; i += blockDim.x) {
    const int c = i & 7, r = (i >> 3) & 15, blk = i >> 7, row = tile * 16 + r;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < w.rows)
      v = *reinterpret_cast<const uint4*>(w.payload + (size_t)row * K + (size_t)ch * kc + blk * 128 + c * 16);
    *reinterpret_cast<uint4*>(out + blk * 2048 + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
  const int gpr = K >> w.lg;
  float2* pd = reinterpret_cast<float2*>(out + 16 * kc);
  for (int i = threadIdx.x; i < 16 * pr; i += blockDim.x) {
    const int r = i / pr, j = i - r * pr, row = tile * 16 + r;
    float2 v = make_float2(0.f, 0.f);
    if (row < w.rows) v = reinterpret_cast<const float2*>(w.meta)[(size_t)row * gpr + (size_t)ch * pr + j];
    pd[i] = v;
  }
}

// Phase-B adapter images of one adapter second stage W2 [R][C] (SG8, group
// 2^lg >= 64): for every head h (one block each) the block at
// dst + h * img_b + off holds the head's columns [64 h, 64 h + 64) transposed,
// [64][stride] codes (column c's R codes, zero up to stride), then per row r <
// rpad the two (min, max) pairs of the even-aligned group pair around the
// columns ([rpad][16 B], zero past R).  Transposed so that the column is the
// row of an integer-mma A operand and the rank the k dimension.
__global__ void adp_image_kernel(uint8_t* dst, PackedView w, uint32_t img_b, uint32_t off, int stride, int rpad) {
  const int h = blockIdx.x, R = w.rows, C = w.cols;
  uint8_t* out = dst + (size_t)h * img_b + off;
  for (int i = threadIdx.x; i < 64 * stride; i += blockDim.x) {
    const int c = i / stride, r = i - c * stride;
    out[i] = r < R ? w.payload[(size_t)r * C + h * 64 + c] : (uint8_t)0;
  }
  const int gpr = C >> w.lg, px = ((h * 64) >> w.lg) & ~1;
  uint4* pd = reinterpret_cast<uint4*>(out + (size_t)64 * stride);
  for (int r = threadIdx.x; r < rpad; r += blockDim.x)
    pd[r] = r < R ? *reinterpret_cast<const uint4*>(w.meta + ((size_t)r * gpr + px) * 8) : make_uint4(0u, 0u, 0u, 0u);
}

uint64_t stream_units(const PackedView& w, int kc) { return (uint64_t)((w.rows + 15) / 16) * (uint64_t)(w.cols / kc); }

// Build the streaming copy of every big matrix (bit 10 of the engine flags
// keeps the tensor-map loads from the reference layout instead).  On an
// allocation failure the tensor maps stay in use.
void plan_stream_copy(rwkvb_engine* e, std::vector<DLayerMaps>& hm, bool pre) {
  DArgs& a = e->da;
  a.pre = 0;
  if (e->flags & 0x400u) return;
  const uint32_t ub = a.code_b + a.pair_b;
  const int kc = a.kc;
  uint64_t total = stream_units(e->head, kc) * ub;
  for (const LayerDev& l : e->layers)
    total += (stream_units(l.r, kc) + stream_units(l.k, kc) + stream_units(l.v, kc) + stream_units(l.o, kc) +
              stream_units(l.fk, kc) + stream_units(l.fv, kc)) * ub;
  const uint64_t img_total = (uint64_t)e->d.H * (a.adp_b0 + (uint64_t)(e->d.L - 1) * a.adp_b1);
  if (pre) total += img_total;
  if (cudaMalloc((void**)&e->dstream, total) != cudaSuccess) {
    cudaGetLastError();
    e->dstream = nullptr;
    return;
  }
  uint8_t* cur = e->dstream;
  auto lay = [&](const PackedView& w) {
    const uint64_t n = stream_units(w, kc);
    stream_layout_kernel<<<(unsigned)n, 256>>>(cur, w, a.nb, a.pr, ub, (int)n);
    uint8_t* at = cur;
    cur += n * ub;
    return at;
  };
  for (size_t i = 0; i < e->layers.size(); ++i) {
    const LayerDev& l = e->layers[i];
    hm[i].su[0] = lay(l.r);  // r, k, v back to back: one region of 3C rows
    lay(l.k);
    lay(l.v);
    hm[i].su[1] = lay(l.o);
    hm[i].su[2] = lay(l.fk);
    hm[i].su[3] = lay(l.fv);
  }
  a.head_su = lay(e->head);
  if (pre) {
    for (size_t i = 0; i < e->layers.size(); ++i) {
      const LayerDev& l = e->layers[i];
      const uint32_t ib = i == 0 ? a.adp_b0 : a.adp_b1;
      const PackedView* w2[4] = {&l.w2, &l.a2, &l.g2, &l.v2};
      uint32_t off = 0;
      for (int m = 0; m < (i == 0 ? 3 : 4); ++m) {
        adp_image_kernel<<<e->d.H, 256>>>(cur, *w2[m], ib, off, a.aps[m], a.apr[m]);
        off += 64u * (uint32_t)a.aps[m] + 16u * (uint32_t)a.apr[m];
      }
      hm[i].ai = cur;
      cur += (size_t)e->d.H * ib;
    }
    a.pre = 1;
  }
}

int encode_big(const PackedView& w, const DArgs& a, CUtensorMap* q, CUtensorMap* p) {
  const uint64_t K = (uint64_t)w.cols, rows = (uint64_t)w.rows, gpr = K >> w.lg;
  const uint64_t qd[3] = {128, rows, K / 128}, qs[2] = {K, 128};
  const uint32_t qb[3] = {128, 16, (uint32_t)a.nb};
  int st = encode_u8_map(q, 3, w.payload, qd, qs, qb, true);
  const uint64_t pd[2] = {gpr * 8, rows}, ps[1] = {gpr * 8};
  const uint32_t pb[2] = {(uint32_t)a.pr * 8u, 16};
  if (st == RWKVB_OK) st = encode_u8_map(p, 2, w.meta, pd, ps, pb, false);
  return st;
}

int encode_adp2(const PackedView& w, int box_rows, CUtensorMap* q, CUtensorMap* p) {
  const uint64_t C = (uint64_t)w.cols, R = (uint64_t)w.rows, gpr = C >> w.lg;
  const uint64_t qd[2] = {C, R}, qs[1] = {C};
  const uint32_t qb[2] = {64, (uint32_t)box_rows};
  int st = encode_u8_map(q, 2, w.payload, qd, qs, qb, false);
  const uint64_t pd[2] = {gpr * 8, R}, ps[1] = {gpr * 8};
  const uint32_t pb[2] = {16, (uint32_t)box_rows};
  if (st == RWKVB_OK) st = encode_u8_map(p, 2, w.meta, pd, ps, pb, false);
  return st;
}

// Decide whether the persistent decode kernel can run this model, fill its
// arguments (everything except the per-launch token fields) and encode its
// tensor maps.
const void* decode_fn(int lfk);

bool plan_decode(rwkvb_engine* e) {
  const Dims& d = e->d;
  const LayerDev& l0 = e->layers[0];
  const int lg = l0.r.lg;
  if ((lg != 6 && lg != 7) || d.C % 128 != 0 || d.F % 128 != 0 || e->sms < d.H) return false;
  auto big_ok = [&](const PackedView& w) {
    return w.kind == RWKVB_KIND_SG8 && w.lg == lg && aligned16(w.payload) && aligned16(w.meta);
  };
  auto adp1_ok = [&](const PackedView& w) {
    return w.kind == RWKVB_KIND_SG8 && w.lg >= 2 && w.cols % 16 == 0 && aligned16(w.payload) && aligned16(w.meta);
  };
  auto adp2_ok = [&](const PackedView& w) {
    return w.kind == RWKVB_KIND_SG8 && w.lg >= 6 && d.C % (int)w.group == 0 && ((d.C >> w.lg) % 2) == 0 &&
           aligned16(w.payload) && aligned16(w.meta);
  };
  for (int i = 0; i < d.L; ++i) {
    const LayerDev& l = e->layers[i];
    if (!big_ok(l.r) || !big_ok(l.k) || !big_ok(l.v) || !big_ok(l.o) || !big_ok(l.fk) || !big_ok(l.fv)) return false;
    if (!adp1_ok(l.w1) || !adp1_ok(l.a1) || !adp1_ok(l.g1) || (i > 0 && !adp1_ok(l.v1))) return false;
    if (!adp2_ok(l.w2) || !adp2_ok(l.a2) || !adp2_ok(l.g2) || (i > 0 && !adp2_ok(l.v2))) return false;
  }
  if (!big_ok(e->head)) return false;
  int nb = 0;
  for (int c = kDW; c >= 1 && !nb; --c)
    if ((d.C / 128) % c == 0 && (d.F / 128) % c == 0 && (((c * 128) >> lg) % 2) == 0) nb = c;
  if (!nb) return false;
  DArgs& a = e->da;
  memset(&a, 0, sizeof(a));
  a.nb = nb;
  a.kc = nb * 128;
  a.pr = a.kc >> lg;
  a.lg = lg;
  a.fg = lg >= 7 ? 128 : 64;
  e->lfk = a.fg == 128 ? 2 : 1;
  a.code_b = 16u * (uint32_t)a.kc;
  a.pair_b = 16u * (uint32_t)a.pr * 8u;
  const int ranks[4] = {d.rw, d.ra, d.rg, d.rv};
  const LayerDev& lr = e->layers[d.L > 1 ? 1 : 0];
  const PackedView* w2s[4] = {&lr.w2, &lr.a2, &lr.g2, &lr.v2};
  int rmax = 0;
  for (int m = 0; m < 4; ++m) {
    a.abr[m] = ranks[m] < 256 ? (ranks[m] > 0 ? ranks[m] : 1) : 256;
    a.alg[m] = w2s[m]->lg;
    rmax = ranks[m] > rmax ? ranks[m] : rmax;
  }
  if (rmax > kDMisc - 256) return false;
  // First-adapter items: per adapter the largest row chunk (a power of two up
  // to 256 dividing C) whose codes and (min,max) pairs fit a GEMV unit's ring
  // slot, so the slot stays the unit's size; items are numbered adapter by
  // adapter (v last: layer 0 has none).  2.9B: 128/128/32/128 rows, 140 items,
  // at most one per CTA.
  int alg = 30;
  for (int i = 0; i < d.L; ++i) {
    const LayerDev& l = e->layers[i];
    const PackedView* w1s[4] = {&l.w1, &l.a1, &l.g1, &l.v1};
    for (int m = 0; m < (i > 0 ? 4 : 3); ++m) alg = w1s[m]->lg < alg ? w1s[m]->lg : alg;
  }
  // codes, (min, max) pairs, then the item rows' slice of the mix vector (fp32)
  auto item_bytes = [&](uint32_t rows, uint32_t rank) {
    const uint32_t nel = rows * rank;
    return (nel + 15u) / 16u * 16u + ((nel >> alg) + 4u) * 8u + 4u * rows;
  };
  const uint32_t unit_b = a.code_b + a.pair_b;
  e->d.abase[0] = 0;
  for (int m = 0; m < 4; ++m) {
    int r = 256;
    while (r > 16 && (d.C % r != 0 || item_bytes((uint32_t)r, (uint32_t)ranks[m]) > unit_b)) r /= 2;
    e->d.arow[m] = r;
    e->d.abase[m + 1] = e->d.abase[m] + (ranks[m] > 0 ? (d.C + r - 1) / r : 0);
  }
  // slot: one GEMV unit, one adapter first-stage item, one adapter second-stage piece
  uint32_t slot = unit_b;
  for (int m = 0; m < 4; ++m) {
    const uint32_t item = item_bytes((uint32_t)d.arow[m], (uint32_t)ranks[m]);
    slot = slot > item ? slot : item;
  }
  for (int m = 0; m < 4; ++m) slot = slot > (uint32_t)a.abr[m] * 80u ? slot : (uint32_t)a.abr[m] * 80u;
  a.slot = (slot + 1023u) / 1024u * 1024u;
  auto set_bytes = [&](int K) { return ((uint32_t)K * 3u + 2u * (uint32_t)(K / a.fg) * 4u + 15u) & ~15u; };
  a.dig_set = set_bytes(d.C);
  uint32_t dig = 3u * a.dig_set;
  // phase E's digits: the whole FFN width in row order; in chunk order only
  // the widest chunk span of one CTA's units
  a.ecm = (e->flags & 0x10000u) ? 0 : 1;  // bit 16: FFN value rows in row order, fp32 accumulation
  int kl = d.F;
  if (a.ecm) {
    const int tiles = d.C / 16, U = tiles * (d.F / a.kc);
    kl = 0;
    for (int b = 0; b < e->sms; ++b) {
      const int u0 = (int)((unsigned)U * (unsigned)b / (unsigned)e->sms);
      const int u1 = (int)((unsigned)U * (unsigned)(b + 1) / (unsigned)e->sms);
      const int span = u1 > u0 ? ((u1 - 1) / tiles - u0 / tiles + 1) * a.kc : 0;
      kl = span > kl ? span : kl;
    }
  }
  dig = dig > set_bytes(kl) ? dig : set_bytes(kl);
  const uint32_t wkv = (uint32_t)(4096 + ((d.rtot + 3) & ~3) + 256 + 7 * 64) * 4u;
  dig = dig > wkv ? dig : wkv;
  dig = (dig + 127u) & ~127u;
  const uint32_t vec = ((uint32_t)d.C * 4u + 127u) & ~127u;
  const uint32_t rest = dig + 4u * vec + kDPartBytes + (uint32_t)kDMisc * 4u;
  // per-block opt-in shared memory less the kernel's static shared memory and
  // the dynamic area's 1 KB alignment slack
  uint32_t budget = 227u * 1024u - 1024u - 5u * 1024u;
  {
    cudaFuncAttributes fa;
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess &&
        cudaFuncGetAttributes(&fa, decode_fn(e->lfk)) == cudaSuccess && (size_t)optin > fa.sharedSizeBytes + 1024u)
      budget = (uint32_t)((size_t)optin - fa.sharedSizeBytes - 1024u);
    cudaGetLastError();
  }
  // Ring depth: the consumers' own small loads (accumulators, vectors) queue
  // behind the weight tiles in flight on their SM, so a deeper ring than the
  // HBM latency needs lengthens every step of the per-layer dependency chain
  // (2.9B bs1: 448 tok/s with 3 slots, 434 with 6).  Flag bits 12..15 set
  // another depth (3..8).
  const int nst_cap = (int)((e->flags >> 12) & 0xFu);
  int nst = nst_cap ? (nst_cap < 3 ? 3 : (nst_cap < kDMaxSt ? nst_cap : kDMaxSt)) : kDRingDefault;
  while (nst > 3 && (uint32_t)nst * a.slot + rest > budget) --nst;
  if ((uint32_t)nst * a.slot + rest > budget) return false;
  a.nst = nst;
  uint32_t off = (uint32_t)nst * a.slot;
  a.o_dig = off;  off += dig;
  a.o_x = off;    off += vec;
  a.o_xb = off;   off += vec;
  a.o_t = off;    off += vec;
  a.o_p = off;    off += vec;
  a.o_part = off; off += kDPartBytes;
  a.o_misc = off; off += (uint32_t)kDMisc * 4u;
  // Preload mode: the phase-B adapter image of a head CTA (80 B per adapter
  // rank row) and the CTA's adapter first-stage item get dedicated shared
  // memory, loaded at the start of each layer, when both fit beside the ring
  // and no CTA has more than one item (bit 11 of the flags turns it off).
  // transposed images: rank padded to whole 32-code k-steps, column stride
  // = 32 mod 64 bytes (the eight columns of one fragment load on distinct banks)
  uint32_t blk[4];
  int rt = 0, nchunk = 0;
  for (int m = 0; m < 4; ++m) {
    a.apr[m] = (ranks[m] + 31) / 32 * 32;
    a.aps[m] = a.apr[m] + ((32 - a.apr[m] % 64) + 64) % 64;
    blk[m] = 64u * (uint32_t)a.aps[m] + 16u * (uint32_t)a.apr[m];
    rt += a.apr[m];
    nchunk += (a.apr[m] / 32 + kDPieceSteps - 1) / kDPieceSteps;
  }
  a.adp_b0 = blk[0] + blk[1] + blk[2];
  a.adp_b1 = d.L > 1 ? a.adp_b0 + blk[3] : a.adp_b0;
  const uint32_t adp_buf = ((a.adp_b1 > a.adp_b0 ? a.adp_b1 : a.adp_b0) + 127u) & ~127u;
  // phase B's tensor-core pieces keep x', its digits and the piece partials in misc
  const bool pieces_fit = nchunk <= kDMaxChunks && d_pieces_misc_floats(rt, nchunk) <= kDMisc;
  const bool want_pre = !(e->flags & 0x400u) && !(e->flags & 0x800u) && e->d.abase[4] <= e->sms &&
                        pieces_fit && off + adp_buf + a.slot <= budget;
  if (want_pre) {
    a.o_adp = off;  off += adp_buf;
    a.o_item = off; off += a.slot;
  }
  a.smem_total = off;
  // tensor maps
  std::vector<DLayerMaps> hm((size_t)d.L);
  memset(hm.data(), 0, sizeof(DLayerMaps) * hm.size());
  CUtensorMap hh[2];
  for (int i = 0; i < d.L; ++i) {
    const LayerDev& l = e->layers[i];
    const PackedView* big[6] = {&l.r, &l.k, &l.v, &l.o, &l.fk, &l.fv};
    for (int m = 0; m < 6; ++m)
      if (encode_big(*big[m], a, &hm[i].q[m], &hm[i].p[m]) != RWKVB_OK) return false;
    const PackedView* w2[4] = {&l.w2, &l.a2, &l.g2, &l.v2};
    for (int m = 0; m < (i > 0 ? 4 : 3); ++m)
      if (encode_adp2(*w2[m], a.abr[m], &hm[i].aq[m], &hm[i].ap[m]) != RWKVB_OK) return false;
  }
  if (encode_big(e->head, a, &hh[0], &hh[1]) != RWKVB_OK) return false;
  plan_stream_copy(e, hm, want_pre);
  if (!a.pre) a.smem_total = a.o_misc + (uint32_t)kDMisc * 4u;  // no dedicated buffers
  if (e->dstream && cudaDeviceSynchronize() != cudaSuccess) return false;
  if (cudaMalloc((void**)&e->dmaps, sizeof(DLayerMaps) * (size_t)d.L) != cudaSuccess ||
      cudaMalloc((void**)&e->dhead, sizeof(CUtensorMap) * 2) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cudaMemcpy(e->dmaps, hm.data(), sizeof(DLayerMaps) * (size_t)d.L, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(e->dhead, hh, sizeof(hh), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  a.layers = e->dlayers;
  a.lmaps = e->dmaps;
  a.head_maps = e->dhead;
  a.emb = e->emb;
  a.ln0_w = e->ln0_w; a.ln0_b = e->ln0_b; a.lnout_w = e->lnout_w; a.lnout_b = e->lnout_b;
  a.b = e->b;
  a.d = d;
  a.spin_limit = 1u << 22;
  a.l2_first = (e->flags & 0x200u) ? 0 : 1;  // bit 9: plain weight-stream loads (no L2 policy)
  const PackedView& E = e->emb;
  a.emb_fast = E.kind == RWKVB_KIND_SG8 && E.lg >= 4 && d.C % (int)E.group == 0 && ((d.C >> E.lg) % 2) == 0 &&
               aligned16(E.payload) && aligned16(E.meta);
  e->dsmem = (size_t)a.smem_total + 1024;
  return true;
}

const void* decode_fn(int lfk) {
  return lfk == 2 ? (const void*)decode_kernel<2> : (const void*)decode_kernel<1>;
}

int launch_persistent(rwkvb_engine* e, int ntok, int mode, int first_tok, const int* forced, cudaStream_t s,
                      bool streamed = false) {
  DArgs a = e->da;
  if (streamed) {
    a.ring_count = reinterpret_cast<unsigned*>(e->hring_dev);
    a.ring_cancel = reinterpret_cast<const int*>(e->hring_dev + 64);
    a.ring_ids = reinterpret_cast<int*>(e->hring_dev + 128);
  }
  a.ntok = ntok;
  a.mode = mode;
  a.first_tok = first_tok;
  a.forced = forced;
  a.gbar = e->b.ticket;  // the argmax ticket word doubles as the grid-barrier counter here
  a.trace = e->dtrace;
  a.trace_cap = e->trace_cap;
  if (e->dtrace) cudaMemsetAsync(e->dtrace + 2 * (size_t)e->trace_cap, 0, sizeof(unsigned long long) * 2 * (size_t)e->trace_cap, s);
  cudaError_t err = cudaMemsetAsync(a.gbar, 0, sizeof(unsigned), s);
  if (err != cudaSuccess) return cuda_status(err);
  void* args[] = {&a};
  err = cudaLaunchCooperativeKernel(decode_fn(e->lfk), dim3(e->sms), dim3(kDThreads), args, e->dsmem, s);
  return cuda_status(err);
}
}  // namespace

extern "C" int rwkvb_engine_create(const rwkvb_model_desc* m, uint32_t flags, rwkvb_engine** out) {
  if (!m || !out || !m->layers) return RWKVB_EARG;
  *out = nullptr;
  const int L = m->n_layer, C = m->n_embd, N = m->head_size, F = m->ffn, V = m->vocab;
  if (L <= 0 || C <= 0 || F <= 0 || V <= 0 || N != 64 || C % 64 != 0 || F % 16 != 0) return RWKVB_EUNSUPPORTED;
  if (!desc_ok(m->emb, V, C) || !desc_ok(m->head, V, C)) return RWKVB_EARG;
  if (!m->ln0_w || !m->ln0_b || !m->ln_out_w || !m->ln_out_b) return RWKVB_EARG;
  const rwkvb_layer_desc& l0 = m->layers[0];
  const int rw = l0.w1.cols, ra = l0.a1.cols, rg = l0.g1.cols;
  const int rv = L > 1 ? m->layers[1].v1.cols : (l0.v1.data ? l0.v1.cols : 0);
  for (int i = 0; i < L; ++i) {
    const rwkvb_layer_desc& s = m->layers[i];
    if (!desc_ok(s.att_r, C, C) || !desc_ok(s.att_k, C, C) || !desc_ok(s.att_v, C, C) || !desc_ok(s.att_o, C, C))
      return RWKVB_EARG;
    if (!desc_ok(s.w1, C, rw) || !desc_ok(s.w2, rw, C) || !desc_ok(s.a1, C, ra) || !desc_ok(s.a2, ra, C) ||
        !desc_ok(s.g1, C, rg) || !desc_ok(s.g2, rg, C))
      return RWKVB_EARG;
    if (i > 0 && (!desc_ok(s.v1, C, rv) || !desc_ok(s.v2, rv, C))) return RWKVB_EARG;
    if (!desc_ok(s.ffn_key, F, C) || !desc_ok(s.ffn_value, C, F)) return RWKVB_EARG;
    const float* vecs[] = {s.ln1_w, s.ln1_b, s.ln2_w, s.ln2_b, s.x_r, s.x_w, s.x_k, s.x_v, s.x_a, s.x_g,
                           s.w0, s.a0, s.k_k, s.k_a, s.r_k, s.lnx_w, s.lnx_b, s.ffn_x_k};
    for (const float* p : vecs)
      if (!p) return RWKVB_EARG;
    if (i > 0 && !s.v0) return RWKVB_EARG;
  }
  if (rw <= 0 || ra <= 0 || rg <= 0 || rw + ra + rg + rv > 2048) return RWKVB_EUNSUPPORTED;

  rwkvb_engine* e = new (std::nothrow) rwkvb_engine();
  if (!e) return RWKVB_EALLOC;
  cudaGetDevice(&e->dev);
  e->sms = device_sms();
  e->flags = flags;
  e->pf_dist = (flags & 0x100u) ? (int)((flags >> 4) & 0xF) : 0;  // bit 8: explicit L2 prefetch distance
  e->pdl = !(flags & 0x2u);                                        // bit 1: disable PDL
  Dims& d = e->d;
  d.L = L; d.C = C; d.H = C / 64; d.F = F; d.V = V;
  d.rw = rw; d.ra = ra; d.rg = rg; d.rv = rv; d.rtot = rw + ra + rg + rv;
  // first-adapter row chunk: as large as fits one ~22 KB ring slot (and a divisor of C)
  {
    const int rmax = rw > ra ? (rw > rg ? rw : rg) : (ra > rg ? ra : rg);
    const int rmax2 = rmax > rv ? rmax : rv;
    d.adp_rows = 128;
    while (d.adp_rows > 16 && (d.adp_rows * rmax2 > 21 * 1024 || C % d.adp_rows != 0)) d.adp_rows /= 2;
  }
  d.adp_splits = (C + d.adp_rows - 1) / d.adp_rows;
  d.hist_cap = 1 << 16;
  for (int i = 0; i < L; ++i) e->layers.push_back(make_layer(m->layers[i]));
  e->emb = make_view(m->emb);
  e->head = make_view(m->head);
  e->ln0_w = m->ln0_w; e->ln0_b = m->ln0_b; e->lnout_w = m->ln_out_w; e->lnout_b = m->ln_out_b;
  e->head_grid = 2 * e->sms;

  const size_t H = d.H;
  size_t fl[] = {(size_t)L * C, (size_t)L * H * 4096, (size_t)L * C, (size_t)C, (size_t)C, (size_t)C, (size_t)C,
                 (size_t)3 * C, (size_t)d.adp_splits * d.rtot, (size_t)C, (size_t)F, (size_t)C, (size_t)V,
                 (size_t)e->head_grid * 2 + 8, (size_t)C, (size_t)C, (size_t)d.rtot * 2, (size_t)C * 2};
  size_t total = 0, offs[20];
  for (int i = 0; i < 18; ++i) {
    offs[i] = total;
    total += ((fl[i] * 4 + 255) / 256) * 256;
  }
  const size_t ints_off = total;
  total += ((size_t)(e->head_grid * 2 + 8) * 4 + 255) / 256 * 256;
  const size_t misc_off = total;
  total += 256;
  const size_t hist_off = total;
  total += (size_t)d.hist_cap * 4;
  if (cudaMalloc(&e->arena, total) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return RWKVB_EALLOC;
  }
  cudaMemset(e->arena, 0, total);
  char* base = (char*)e->arena;
  float** fb[] = {&e->b.att_x, &e->b.wkv, &e->b.ffn_x, &e->b.xa, &e->b.xb, &e->b.xln1, &e->b.xln2,
                  &e->b.rkv, &e->b.adp, &e->b.att_y, &e->b.h, &e->b.v_first, &e->b.logits, &e->b.amax_v};
  for (int i = 0; i < 14; ++i) *fb[i] = (float*)(base + offs[i]);
  e->b.ao = (float*)(base + offs[14]);
  e->b.fo = (float*)(base + offs[15]);
  e->b.adp64 = (unsigned long long*)(base + offs[16]);
  e->b.fo64 = (unsigned long long*)(base + offs[17]);
  e->b.amax_i = (int*)(base + ints_off);
  e->b.ticket = (unsigned*)(base + misc_off);
  e->b.tok = (int*)(base + misc_off + 16);
  e->b.step = (int*)(base + misc_off + 32);
  e->b.err = (int*)(base + misc_off + 48);
  e->b.stop = (int*)(base + misc_off + 64);
  e->b.hist = (int*)(base + hist_off);

  // weights touched by each phase, in step order (embed, 5 per layer, head)
  e->phase_pf.push_back(pf_empty());
  for (int i = 0; i < L; ++i) {
    const rwkvb_layer_desc& s = m->layers[i];
    Prefetch p = pf_empty();
    pf_add(p, s.att_r); pf_add(p, s.att_k); pf_add(p, s.att_v);
    pf_add(p, s.w1); pf_add(p, s.a1); pf_add(p, s.g1);
    if (i > 0) pf_add(p, s.v1);
    e->phase_pf.push_back(p);
    p = pf_empty();
    pf_add(p, s.w2); pf_add(p, s.a2); pf_add(p, s.g2);
    if (i > 0) pf_add(p, s.v2);
    e->phase_pf.push_back(p);
    p = pf_empty(); pf_add(p, s.att_o); e->phase_pf.push_back(p);
    p = pf_empty(); pf_add(p, s.ffn_key); e->phase_pf.push_back(p);
    p = pf_empty(); pf_add(p, s.ffn_value); e->phase_pf.push_back(p);
  }
  {
    Prefetch p = pf_empty();
    pf_add(p, m->head);
    pf_cap(p, 48ull << 20);
    e->phase_pf.push_back(p);
  }

  int st = RWKVB_OK;
  // persistent decode path (one cooperative launch for the whole loop)
  if (cudaMalloc((void**)&e->dlayers, sizeof(LayerDev) * (size_t)L) != cudaSuccess ||
      cudaMalloc((void**)&e->dtokens, sizeof(int) * (size_t)d.hist_cap) != cudaSuccess) {
    cudaGetLastError();
    st = RWKVB_EALLOC;
  }
  if (st == RWKVB_OK)
    st = cuda_status(cudaMemcpy(e->dlayers, e->layers.data(), sizeof(LayerDev) * (size_t)L, cudaMemcpyHostToDevice));
  if (st == RWKVB_OK && (flags & 0x8u)) {
    e->trace_cap = 1 << 16;
    if (cudaMalloc((void**)&e->dtrace, sizeof(unsigned long long) * 4 * (size_t)e->trace_cap) != cudaSuccess) {
      cudaGetLastError();
      st = RWKVB_EALLOC;
    }
  }
  if (st == RWKVB_OK && !(flags & 0x4u) && plan_decode(e)) {
    const void* fn = decode_fn(e->lfk);
    int per_sm = 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)e->dsmem) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDThreads, e->dsmem) == cudaSuccess &&
        per_sm >= 1) {
      e->persistent = true;
    }
    cudaGetLastError();
  }
  const void* kernels[] = {(const void*)phase_kernel, (const void*)att_in_kernel, (const void*)wkv_kernel,
                           (const void*)embed_kernel};
  for (const void* k : kernels)
    if (st == RWKVB_OK) st = allow_big_smem(k);
  if (st == RWKVB_OK) st = cuda_status(cudaStreamCreateWithFlags(&e->cap, cudaStreamNonBlocking));
  if (st == RWKVB_OK) st = cuda_status(cudaDeviceSynchronize());
  if (st != RWKVB_OK) {
    rwkvb_engine_destroy(e);
    return st;
  }
  *out = e;
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_create_staged(const rwkvb_model_desc* m, const rwkvb_stage_desc* st, uint32_t flags,
                                          rwkvb_engine** out) {
  if (!m || !st || !out || st->n_slots <= 0 || !st->slot_of_layer || !st->host_src || !st->slot_dev ||
      st->layer_bytes == 0)
    return RWKVB_EARG;
  *out = nullptr;
  int streamed = 0;
  for (int i = 0; i < m->n_layer; ++i) {
    const int sl = st->slot_of_layer[i];
    if (sl >= st->n_slots || sl < -1) return RWKVB_EARG;
    if (sl >= 0) {
      if (!st->host_src[i] || !st->slot_dev[sl]) return RWKVB_EARG;
      ++streamed;
    }
  }
  rwkvb_engine* e = nullptr;
  // staged layers run as the multi-kernel step (bit 2: no persistent kernel)
  const int rc = rwkvb_engine_create(m, flags | 0x4u, &e);
  if (rc != RWKVB_OK) return rc;
  e->staged = streamed > 0;
  e->stage_bytes = st->layer_bytes;
  e->stage_slot.assign(st->slot_of_layer, st->slot_of_layer + m->n_layer);
  e->stage_src.assign(st->host_src, st->host_src + m->n_layer);
  e->stage_dev.assign(st->slot_dev, st->slot_dev + st->n_slots);
  cudaError_t err = cudaSuccess;
  if (e->staged) {
    err = cudaStreamCreateWithFlags(&e->copy, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming);
    for (int j = 0; j < streamed && err == cudaSuccess; ++j) {
      cudaEvent_t a = nullptr, b = nullptr;
      err = cudaEventCreateWithFlags(&a, cudaEventDisableTiming);
      if (err == cudaSuccess) err = cudaEventCreateWithFlags(&b, cudaEventDisableTiming);
      if (a) e->ev_loaded.push_back(a);
      if (b) e->ev_done.push_back(b);
    }
  }
  if (err != cudaSuccess) {
    rwkvb_engine_destroy(e);
    return cuda_status(err);
  }
  *out = e;
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_destroy(rwkvb_engine* e) {
  if (!e) return RWKVB_EARG;
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->graph) cudaGraphDestroy(e->graph);
  if (e->cap) cudaStreamDestroy(e->cap);
  if (e->arena) cudaFree(e->arena);
  if (e->dlayers) cudaFree(e->dlayers);
  if (e->dmaps) cudaFree(e->dmaps);
  if (e->dhead) cudaFree(e->dhead);
  if (e->dtokens) cudaFree(e->dtokens);
  if (e->dtrace) cudaFree(e->dtrace);
  if (e->hring) cudaFreeHost(e->hring);
  if (e->dstream) cudaFree(e->dstream);
  for (cudaEvent_t ev : e->ev_loaded) cudaEventDestroy(ev);
  for (cudaEvent_t ev : e->ev_done) cudaEventDestroy(ev);
  if (e->ev_fork) cudaEventDestroy(e->ev_fork);
  if (e->copy) cudaStreamDestroy(e->copy);
  delete e;
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_buffers(rwkvb_engine* e, float** att_x, float** wkv, float** ffn_x, float** logits) {
  if (!e) return RWKVB_EARG;
  if (att_x) *att_x = e->b.att_x;
  if (wkv) *wkv = e->b.wkv;
  if (ffn_x) *ffn_x = e->b.ffn_x;
  if (logits) *logits = e->b.logits;
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_reset(rwkvb_engine* e, void* stream) {
  if (!e) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  const Dims& d = e->d;
  cudaError_t err = cudaMemsetAsync(e->b.att_x, 0, sizeof(float) * (size_t)d.L * d.C, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->b.wkv, 0, sizeof(float) * (size_t)d.L * d.H * 4096, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->b.ffn_x, 0, sizeof(float) * (size_t)d.L * d.C, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->b.err, 0, sizeof(int), s);
  return cuda_status(err);
}

static int check_err_flag(rwkvb_engine* e, cudaStream_t s) {
  int h = 0;
  cudaError_t err = cudaMemcpyAsync(&h, e->b.err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_status(err);
  if (h) {
    cudaMemsetAsync(e->b.err, 0, sizeof(int), s);
    cudaStreamSynchronize(s);
    return (h & kErrTimeout) ? RWKVB_ETIMEOUT : RWKVB_EARG;
  }
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_forward(rwkvb_engine* e, const int32_t* tokens, int32_t n, void* stream) {
  if (!e || (!tokens && n > 0) || n < 0) return RWKVB_EARG;
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->d.V) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  if (e->persistent) {
    int st = RWKVB_OK;
    for (int done = 0; done < n && st == RWKVB_OK;) {
      const int chunk = (n - done) < e->d.hist_cap ? (n - done) : e->d.hist_cap;
      st = cuda_status(cudaMemcpyAsync(e->dtokens, tokens + done, sizeof(int32_t) * chunk, cudaMemcpyHostToDevice, s));
      if (st == RWKVB_OK) st = launch_persistent(e, chunk, 1, 0, e->dtokens, s);
      done += chunk;
    }
    return st;
  }
  int st = ensure_graph(e);
  for (int i = 0; i < n && st == RWKVB_OK; ++i) {
    set_token_kernel<<<1, 1, 0, s>>>(e->b.tok, tokens[i], e->b.step, 0);
    st = cuda_status(cudaGetLastError());
    if (st == RWKVB_OK) st = run_step(e, s);
  }
  return st;
}

extern "C" int rwkvb_engine_decode_greedy_async(rwkvb_engine* e, int32_t first, int32_t n, int32_t* out_dev,
                                                void* stream) {
  if (!e || n < 0 || (n > 0 && !out_dev) || first < 0 || first >= e->d.V) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  if (e->persistent) {
    int st = RWKVB_OK;
    for (int done = 0; done < n && st == RWKVB_OK;) {
      const int chunk = (n - done) < e->d.hist_cap ? (n - done) : e->d.hist_cap;
      st = launch_persistent(e, chunk, 0, done == 0 ? first : -1, nullptr, s);
      if (st == RWKVB_OK)
        st = cuda_status(cudaMemcpyAsync(out_dev + done, e->b.hist, sizeof(int32_t) * chunk,
                                         cudaMemcpyDeviceToDevice, s));
      done += chunk;
    }
    return st;
  }
  int st = ensure_graph(e);
  if (st != RWKVB_OK) return st;
  set_token_kernel<<<1, 1, 0, s>>>(e->b.tok, first, e->b.step, 1);
  st = cuda_status(cudaGetLastError());
  int done = 0;
  while (st == RWKVB_OK && done < n) {
    const int chunk = (n - done) < e->d.hist_cap ? (n - done) : e->d.hist_cap;
    for (int i = 0; i < chunk && st == RWKVB_OK; ++i) st = run_step(e, s);
    if (st == RWKVB_OK)
      st = cuda_status(cudaMemcpyAsync(out_dev + done, e->b.hist, sizeof(int32_t) * chunk,
                                       cudaMemcpyDeviceToDevice, s));
    if (st == RWKVB_OK && done + chunk < n) st = cuda_status(cudaMemsetAsync(e->b.step, 0, sizeof(int), s));
    done += chunk;
  }
  return st;
}

extern "C" int rwkvb_engine_decode_greedy(rwkvb_engine* e, int32_t first, int32_t n, int32_t* out_host,
                                          void* stream) {
  if (!e || n < 0 || (n > 0 && !out_host)) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  int32_t* dev = nullptr;
  if (n > 0 && cudaMallocAsync((void**)&dev, sizeof(int32_t) * (size_t)n, s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  int st = rwkvb_engine_decode_greedy_async(e, first, n, dev, s);
  if (st == RWKVB_OK && n > 0)
    st = cuda_status(cudaMemcpyAsync(out_host, dev, sizeof(int32_t) * (size_t)n, cudaMemcpyDeviceToHost, s));
  if (dev) cudaFreeAsync(dev, s);
  const int st2 = cuda_status(cudaStreamSynchronize(s));
  if (st == RWKVB_OK) st = st2;
  if (st == RWKVB_OK) st = check_err_flag(e, s);
  return st;
}

static int ensure_host_ring(rwkvb_engine* e) {
  if (e->hring) return RWKVB_OK;
  const size_t bytes = 128 + sizeof(int32_t) * (size_t)e->d.hist_cap;
  void* h = nullptr;
  if (cudaHostAlloc(&h, bytes, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  memset(h, 0, bytes);
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
    cudaGetLastError();
    cudaFreeHost(h);
    return RWKVB_ECUDA;
  }
  e->hring = (uint8_t*)h;
  e->hring_dev = (uint8_t*)d;
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_host_ring(rwkvb_engine* e, int32_t** ids, volatile uint32_t** count,
                                      volatile int32_t** cancel, int32_t* cap) {
  if (!e) return RWKVB_EARG;
  if (!e->persistent) return RWKVB_EUNSUPPORTED;
  const int st = ensure_host_ring(e);
  if (st != RWKVB_OK) return st;
  if (ids) *ids = reinterpret_cast<int32_t*>(e->hring + 128);
  if (count) *count = reinterpret_cast<volatile uint32_t*>(e->hring);
  if (cancel) *cancel = reinterpret_cast<volatile int32_t*>(e->hring + 64);
  if (cap) *cap = e->d.hist_cap;
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_decode_stream(rwkvb_engine* e, int32_t first, int32_t n, int32_t* out_dev,
                                          void* stream) {
  if (!e || n < 0 || first < 0 || first >= e->d.V) return RWKVB_EARG;
  if (!e->persistent) return RWKVB_EUNSUPPORTED;
  if (n > e->d.hist_cap) return RWKVB_EARG;
  int st = ensure_host_ring(e);
  if (st != RWKVB_OK) return st;
  // the previous streamed decode of this engine has finished (documented
  // precondition), so nothing on the device writes the ring now
  *reinterpret_cast<volatile uint32_t*>(e->hring) = 0u;
  *reinterpret_cast<volatile int32_t*>(e->hring + 64) = 0;
  volatile int32_t* ids = reinterpret_cast<volatile int32_t*>(e->hring + 128);
  for (int i = 0; i < n; ++i) ids[i] = -1;  // a step's id replaces -1 when the step ends
  std::atomic_thread_fence(std::memory_order_seq_cst);
  if (n == 0) return RWKVB_OK;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_persistent(e, n, 0, first, nullptr, s, true);
  if (st == RWKVB_OK && out_dev)
    st = cuda_status(cudaMemcpyAsync(out_dev, e->b.hist, sizeof(int32_t) * (size_t)n, cudaMemcpyDeviceToDevice, s));
  return st;
}

extern "C" int rwkvb_engine_check(rwkvb_engine* e, void* stream) {
  if (!e) return RWKVB_EARG;
  return check_err_flag(e, (cudaStream_t)stream);
}

extern "C" int rwkvb_engine_launches_per_step(rwkvb_engine* e, int32_t* out) {
  if (!e || !out) return RWKVB_EARG;
  *out = e->persistent ? 0 : 2 + 5 * e->d.L;  // persistent: one launch per decode call, not per step
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_trace(rwkvb_engine* e, uint64_t* out, int32_t cap, int32_t* n_out) {
  if (!e || !out || cap <= 0 || !n_out) return RWKVB_EARG;
  if (!e->dtrace) return RWKVB_EUNSUPPORTED;
  const int n = cap < 4 * e->trace_cap ? cap : 4 * e->trace_cap;
  const int st = cuda_status(cudaMemcpy(out, e->dtrace, sizeof(uint64_t) * (size_t)n, cudaMemcpyDeviceToHost));
  *n_out = n;
  return st;
}
