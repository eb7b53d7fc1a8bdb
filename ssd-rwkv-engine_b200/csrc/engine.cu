// Fused RWKV-7 decode engine: one packed-model token step as a chain of
// phase kernels captured in a CUDA graph.
//
// Per layer (mirrors forward_block_packed, packed_block_forward.py:76-166):
//   att_in  : ln1 + token-shift mixes (rwkv7_linear.py:165-171), r/k/v GEMVs
//             and the first adapter projections (x @ W1, A1, G1, V1) as
//             split-row partial sums
//   wkv     : one CTA per head: adapter second projections for the head's
//             channels, kk-normalize, k update, v-first mix, decay, WKV7
//             state update, GroupNorm, bonus, gate (rwkv7_linear.py:301-349)
//   att_out : output GEMV + residual; x_prev(att) <- ln1(x)
//   ffn_in  : ln2 + mix, key GEMV, relu^2 (rwkv7_linear.py:370-371, 409)
//   ffn_out : value GEMV + residual; x_prev(ffn) <- ln2(x)
// then head: ln_out + head GEMV + greedy argmax (first maximum).
//
// Weights are streamed once per token.  Every phase kernel first issues bulk
// L2 prefetches of the weights of the phase `prefetch_distance` steps ahead
// (split across its CTAs), so HBM keeps streaming while the dependent chain
// of small kernels advances.
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "wkv7.cuh"

namespace rwkvb {

constexpr int kThreads = 256;
constexpr int kMaxPf = 8;

struct Prefetch {
  const uint8_t* ptr[kMaxPf];
  uint64_t bytes[kMaxPf];
  uint64_t total;
  int n;
};

struct LayerDev {
  PackedView r, k, v, o, w1, w2, a1, a2, g1, g2, v1, v2, fk, fv;
  int mode_r, mode_k, mode_v, mode_o, mode_fk, mode_fv;
  int lg_r, lg_k, lg_v, lg_o, lg_fk, lg_fv;
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
  float *amax_v;               // [grid] per-CTA argmax value
  int *amax_i;                 // [grid] per-CTA argmax index
  unsigned *ticket;            // last-CTA election for the argmax
  int *tok;                    // token consumed by the next step
  int *hist;                   // argmax history ring
  int *step;                   // steps since the last history reset
  int *err;                    // error flags (bit0: token out of range)
};

struct Dims {
  int L, C, H, F, V;
  int rw, ra, rg, rv, rtot;  // adapter ranks, total
  int adp_splits, adp_rows;  // first-adapter row split
  int hist_cap;
};

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

// LayerNorm of a global vector into shared memory (two-pass mean / variance).
__device__ __forceinline__ void layer_norm_to_smem(const float* x, const float* w, const float* b, int C,
                                                   float* out, float* red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    float v = x[i];
    out[i] = v;
    s += v;
  }
  const float mean = block_sum(s, red) / (float)C;
  float q = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    float d = out[i] - mean;
    q += d * d;
  }
  const float var = block_sum(q, red) / (float)C;
  const float rstd = rsqrtf(var + 1e-5f);
  for (int i = threadIdx.x; i < C; i += blockDim.x) out[i] = (out[i] - mean) * rstd * w[i] + b[i];
  __syncthreads();
}

// ------------------------------------------------------------- embed
struct EmbedArgs {
  PackedView emb;
  const float *ln0_w, *ln0_b;
  Bufs b;
  Dims d;
  Prefetch pf;
};

__global__ void __launch_bounds__(kThreads) embed_kernel(EmbedArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) float sm[];
  issue_prefetch(a.pf);
  const int C = a.d.C;
  int tok = *a.b.tok;
  if (tok < 0 || tok >= a.d.V) {
    if (threadIdx.x == 0) atomicOr(a.b.err, 1);
    tok = 0;
  }
  float* row = sm;
  for (int i = threadIdx.x; i < C; i += blockDim.x) row[i] = packed_at(a.emb, tok, i);
  __syncthreads();
  layer_norm_to_smem(row, a.ln0_w, a.ln0_b, C, row, red);
  for (int i = threadIdx.x; i < C; i += blockDim.x) a.b.xa[i] = row[i];
}

// ------------------------------------------------------------ att_in
struct AttInArgs {
  LayerDev l;
  Bufs b;
  Dims d;
  Prefetch pf;
  int rkv_ctas, rkv_rpc;  // CTAs [0, rkv_ctas) do r/k/v rows; the rest adapters
  int layer;
};

__global__ void __launch_bounds__(kThreads, 2) att_in_kernel(AttInArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) float sm[];
  issue_prefetch(a.pf);
  const int C = a.d.C;
  float* ln = sm;                       // ln1(x)          [C]
  float* sx = sm + C;                   // mixed input     [C]
  float* sxc = sx + C;                  // chunk sums      [C/16]
  layer_norm_to_smem(a.b.xa, a.l.ln1_w, a.l.ln1_b, C, ln, red);
  const float* prev = a.b.att_x + (size_t)a.layer * C;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < C; i += blockDim.x) a.b.xln1[i] = ln[i];

  if ((int)blockIdx.x < a.rkv_ctas) {
    const int g0 = blockIdx.x * a.rkv_rpc;
    const int g1 = min(3 * C, g0 + a.rkv_rpc);
    for (int m = g0 / C; m <= (g1 - 1) / C && g0 < g1; ++m) {
      const int r0 = max(g0, m * C) - m * C, r1 = min(g1, (m + 1) * C) - m * C;
      const float* mix = m == 0 ? a.l.x_r : (m == 1 ? a.l.x_k : a.l.x_v);
      const PackedView& W = m == 0 ? a.l.r : (m == 1 ? a.l.k : a.l.v);
      const int mode = m == 0 ? a.l.mode_r : (m == 1 ? a.l.mode_k : a.l.mode_v);
      const int lg = m == 0 ? a.l.lg_r : (m == 1 ? a.l.lg_k : a.l.lg_v);
      if (mode == 1) {
        stage_input(C, sx, sxc, [&](int i) { return ln[i] + (prev[i] - ln[i]) * mix[i]; });
      } else {
        for (int i = threadIdx.x; i < C; i += blockDim.x) sx[i] = ln[i] + (prev[i] - ln[i]) * mix[i];
        __syncthreads();
      }
      float* out = a.b.rkv + (size_t)m * C;
      packed_rows(W, mode, lg, sx, sxc, r0, r1, [&](int row, float v) { out[row] = v; });
      __syncthreads();
    }
  } else {
    // first adapter projections: work item = (matrix, row chunk)
    const int item = blockIdx.x - a.rkv_ctas;
    const int nm = a.layer == 0 ? 3 : 4;
    const int m = item / a.d.adp_splits, s = item % a.d.adp_splits;
    if (m >= nm) return;
    const float* mix = m == 0 ? a.l.x_w : (m == 1 ? a.l.x_a : (m == 2 ? a.l.x_g : a.l.x_v));
    const PackedView& W = m == 0 ? a.l.w1 : (m == 1 ? a.l.a1 : (m == 2 ? a.l.g1 : a.l.v1));
    const int off = m == 0 ? 0 : (m == 1 ? a.d.rw : (m == 2 ? a.d.rw + a.d.ra : a.d.rw + a.d.ra + a.d.rg));
    const int i0 = s * a.d.adp_rows, i1 = min(C, i0 + a.d.adp_rows);
    for (int i = threadIdx.x; i < C; i += blockDim.x) sx[i] = ln[i] + (prev[i] - ln[i]) * mix[i];
    __syncthreads();
    transposed_partial(W, sx, i0, i1, 0, W.cols, a.b.adp + (size_t)s * a.d.rtot + off);
  }
}

// --------------------------------------------------------------- wkv
struct WkvArgs {
  LayerDev l;
  Bufs b;
  Dims d;
  Prefetch pf;
  int layer;
};

__global__ void __launch_bounds__(1024) wkv_kernel(WkvArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) float sm[];
  issue_prefetch(a.pf);
  const int h = blockIdx.x, C = a.d.C;
  const int nm = a.layer == 0 ? 3 : 4;
  float* mid = sm;                          // [rtot] first-projection results
  float* vec = sm + ((a.d.rtot + 3) & ~3);  // 4 x 64: w, a, g, v_gate of this head
  float* sr = vec + 256;
  float* sd = sr + 64;
  float* sk = sd + 64;
  float* sv = sk + 64;
  float* skk = sv + 64;
  float* ska = skk + 64;
  float* sy = ska + 64;
  // reduce the first-projection partial sums (fixed order) and activate
  const int used = a.layer == 0 ? a.d.rw + a.d.ra + a.d.rg : a.d.rtot;
  for (int j = threadIdx.x; j < used; j += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < a.d.adp_splits; ++s) acc += a.b.adp[(size_t)s * a.d.rtot + j];
    if (j < a.d.rw) acc = tanhf(acc);
    else if (j >= a.d.rw + a.d.ra && j < a.d.rw + a.d.ra + a.d.rg) acc = sigmoidf_(acc);
    mid[j] = acc;
  }
  __syncthreads();
  // second projections for this head's 64 channels:
  // thread -> (matrix m, channel c, quarter q of the rank), reduced over q
  {
    const int t = threadIdx.x;
    const int q = t & 3, c = (t >> 2) & 63, m = t >> 8;
    float acc = 0.f;
    if (m < nm) {
      const PackedView& W = m == 0 ? a.l.w2 : (m == 1 ? a.l.a2 : (m == 2 ? a.l.g2 : a.l.v2));
      const int off = m == 0 ? 0 : (m == 1 ? a.d.rw : (m == 2 ? a.d.rw + a.d.ra : a.d.rw + a.d.ra + a.d.rg));
      const int ch = h * 64 + c;
      for (int i = q; i < W.rows; i += 4) acc = fmaf(mid[off + i], packed_at(W, i, ch), acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (q == 0 && m < nm) vec[m * 64 + c] = acc;
  }
  __syncthreads();
  // per-channel preparation (threads 0..63)
  const int t = threadIdx.x;
  float kkv = 0.f;
  if (t < 64) {
    const int ch = h * 64 + t;
    const float k = a.b.rkv[C + ch];
    kkv = k * a.l.k_k[ch];
  }
  // ||kk|| over the head: threads 0..63 hold the values, others hold 0
  const float nrm = sqrtf(block_sum(kkv * kkv, red));
  if (t < 64) {
    const int ch = h * 64 + t;
    const float r = a.b.rkv[ch];
    const float k = a.b.rkv[C + ch];
    float v = a.b.rkv[2 * C + ch];
    const float aa = sigmoidf_(a.l.a0[ch] + vec[64 + t]);
    const float kk = kkv / fmaxf(nrm, 1e-12f);
    const float kn = k * (1.0f + (aa - 1.0f) * a.l.k_a[ch]);
    if (a.layer == 0) {
      a.b.v_first[ch] = v;
    } else {
      const float vf = a.b.v_first[ch];
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
  if (t < 256) wkv7_head64(a.b.wkv + ((size_t)a.layer * a.d.H + h) * 4096, sr, sd, sk, sv, skk, ska, sy);
  __syncthreads();
  // GroupNorm over the head (eps 64e-5), bonus, gate
  float yv = t < 64 ? sy[t] : 0.f;
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

// ------------------------------------------------------ generic GEMV phase
// One packed GEMV over `rows` rows with the input staged from `src` (optionally
// layer-normed and token-shift mixed) and a residual / activation epilogue.
struct GemvPhaseArgs {
  PackedView w;
  int mode, lg, rpc;
  // input = ln ? mix(LN(src)) : src ; mix(z) = z + (prev - z) * mixv
  const float* src;
  const float *ln_w, *ln_b, *prev, *mixv;
  float* ln_out;      // CTA 0 stores LN(src) here (may be null)
  // epilogue: out[row] = resid ? resid[row] + v : (relu2 ? relu(v)^2 : v)
  float* out;
  const float* resid;
  int relu2;
  // state copy: state_dst[row] = state_src[row] for this CTA's rows
  float* state_dst;
  const float* state_src;
  Prefetch pf;
  // argmax (head)
  int argmax;
  Bufs b;
  Dims d;
};

__global__ void __launch_bounds__(kThreads, 2) gemv_phase_kernel(GemvPhaseArgs a) {
  __shared__ float red[32];
  __shared__ float bv[kThreads / 32];
  __shared__ int bi[kThreads / 32];
  extern __shared__ __align__(16) float sm[];
  issue_prefetch(a.pf);
  const int K = a.w.cols;
  float* ln = sm;
  float* sx = sm + K;
  float* sxc = sx + K;
  const float* in = a.src;
  if (a.ln_w) {
    layer_norm_to_smem(a.src, a.ln_w, a.ln_b, K, ln, red);
    if (blockIdx.x == 0 && a.ln_out)
      for (int i = threadIdx.x; i < K; i += blockDim.x) a.ln_out[i] = ln[i];
    in = ln;
  }
  const float* prev = a.prev;
  const float* mixv = a.mixv;
  auto f = [&](int i) { float z = in[i]; return mixv ? z + (prev[i] - z) * mixv[i] : z; };
  if (a.mode == 1) {
    stage_input(K, sx, sxc, f);
  } else {
    for (int i = threadIdx.x; i < K; i += blockDim.x) sx[i] = f(i);
    __syncthreads();
  }
  const int r0 = blockIdx.x * a.rpc, r1 = min(a.w.rows, r0 + a.rpc);
  if (a.state_dst)
    for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) a.state_dst[i] = a.state_src[i];
  float best = -INFINITY;
  int besti = 0x7fffffff;
  float* out = a.out;
  const float* resid = a.resid;
  const int relu2 = a.relu2, am = a.argmax;
  packed_rows(a.w, a.mode, a.lg, sx, sxc, r0, r1, [&](int row, float v) {
    if (resid) v = resid[row] + v;
    else if (relu2) v = v > 0.f ? v * v : 0.f;
    out[row] = v;
    if (am && (v > best || (v == best && row < besti))) { best = v; besti = row; }
  });
  if (!am) return;
  // per-CTA argmax (lane 0 of each warp holds its rows' best), then the last CTA reduces
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { bv[wid] = best; bi[wid] = besti; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float cb = -INFINITY;
    int ci = 0x7fffffff;
    for (int w = 0; w < kThreads / 32; ++w)
      if (bv[w] > cb || (bv[w] == cb && bi[w] < ci)) { cb = bv[w]; ci = bi[w]; }
    a.b.amax_v[blockIdx.x] = cb;
    a.b.amax_i[blockIdx.x] = ci;
    __threadfence();
    unsigned prevt = atomicAdd(a.b.ticket, 1u);
    if (prevt == gridDim.x - 1) {
      __threadfence();
      float gb = -INFINITY;
      int gi = 0x7fffffff;
      for (unsigned c = 0; c < gridDim.x; ++c) {
        float v = __ldcg(a.b.amax_v + c);
        int i = __ldcg(a.b.amax_i + c);
        if (v > gb || (v == gb && i < gi)) { gb = v; gi = i; }
      }
      if (gi == 0x7fffffff) gi = 0;  // all logits NaN: torch would return a NaN index; keep 0
      *a.b.tok = gi;
      int st = *a.b.step;
      a.b.hist[st % a.d.hist_cap] = gi;
      *a.b.step = st + 1;
      *a.b.ticket = 0u;
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
  int pf_dist = 1;
  Dims d{};
  std::vector<LayerDev> layers;
  PackedView emb{}, head{};
  int head_mode = 0, head_lg = 0;
  const float *ln0_w = nullptr, *ln0_b = nullptr, *lnout_w = nullptr, *lnout_b = nullptr;
  Bufs b{};
  void* arena = nullptr;
  size_t arena_bytes = 0;
  int head_grid = 0;
  // phase schedule
  std::vector<Prefetch> phase_pf;  // weights of each phase, in step order
  cudaStream_t cap = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int launches = 0;
};

namespace {

LayerDev make_layer(const rwkvb_layer_desc& s) {
  LayerDev l;
  l.r = make_view(s.att_r); l.k = make_view(s.att_k); l.v = make_view(s.att_v); l.o = make_view(s.att_o);
  l.w1 = make_view(s.w1); l.w2 = make_view(s.w2); l.a1 = make_view(s.a1); l.a2 = make_view(s.a2);
  l.g1 = make_view(s.g1); l.g2 = make_view(s.g2); l.v1 = make_view(s.v1); l.v2 = make_view(s.v2);
  l.fk = make_view(s.ffn_key); l.fv = make_view(s.ffn_value);
  l.mode_r = gemv_mode(l.r); l.mode_k = gemv_mode(l.k); l.mode_v = gemv_mode(l.v);
  l.mode_o = gemv_mode(l.o); l.mode_fk = gemv_mode(l.fk); l.mode_fv = gemv_mode(l.fv);
  l.lg_r = ilog2u(l.r.group); l.lg_k = ilog2u(l.k.group); l.lg_v = ilog2u(l.v.group);
  l.lg_o = ilog2u(l.o.group); l.lg_fk = ilog2u(l.fk.group); l.lg_fv = ilog2u(l.fv.group);
  l.ln1_w = s.ln1_w; l.ln1_b = s.ln1_b; l.ln2_w = s.ln2_w; l.ln2_b = s.ln2_b;
  l.x_r = s.x_r; l.x_w = s.x_w; l.x_k = s.x_k; l.x_v = s.x_v; l.x_a = s.x_a; l.x_g = s.x_g;
  l.w0 = s.w0; l.a0 = s.a0; l.v0 = s.v0; l.k_k = s.k_k; l.k_a = s.k_a; l.r_k = s.r_k;
  l.lnx_w = s.lnx_w; l.lnx_b = s.lnx_b; l.ffn_x_k = s.ffn_x_k;
  return l;
}

bool desc_ok(const rwkvb_packed& p, int rows, int cols) {
  return p.data && p.rows == rows && p.cols == cols && p.group_size > 0 &&
         (p.kind == RWKVB_KIND_SG8 || (p.kind >= 3 && p.kind <= 7));
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

// Cap one phase's prefetch (the vocabulary head is larger than L2).
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

int record_step(rwkvb_engine* e, cudaStream_t s) {
  const Dims& d = e->d;
  const int P = (int)e->phase_pf.size();
  int phase = 0;
  auto pf_for = [&](int p) {
    if (e->pf_dist <= 0) return pf_empty();
    return e->phase_pf[(p + e->pf_dist) % P];
  };
  e->launches = 0;
  {
    EmbedArgs a;
    a.emb = e->emb; a.ln0_w = e->ln0_w; a.ln0_b = e->ln0_b; a.b = e->b; a.d = d; a.pf = pf_for(phase++);
    embed_kernel<<<1, kThreads, d.C * sizeof(float), s>>>(a);
    ++e->launches;
  }
  const int rows3 = 3 * d.C;
  const int rkv_ctas_target = 2 * e->sms;
  const int rkv_rpc = (rows3 + rkv_ctas_target - 1) / rkv_ctas_target;
  const int rkv_ctas = (rows3 + rkv_rpc - 1) / rkv_rpc;
  const size_t att_in_smem = (size_t)(2 * d.C + d.C / 16 + 4) * sizeof(float);
  const size_t wkv_smem = (size_t)(((d.rtot + 3) & ~3) + 256 + 7 * 64) * sizeof(float);
  for (int li = 0; li < d.L; ++li) {
    const LayerDev& l = e->layers[li];
    {
      AttInArgs a;
      a.l = l; a.b = e->b; a.d = d; a.pf = pf_for(phase++);
      a.rkv_ctas = rkv_ctas; a.rkv_rpc = rkv_rpc; a.layer = li;
      const int nm = li == 0 ? 3 : 4;
      att_in_kernel<<<rkv_ctas + nm * d.adp_splits, kThreads, att_in_smem, s>>>(a);
    }
    {
      WkvArgs a;
      a.l = l; a.b = e->b; a.d = d; a.pf = pf_for(phase++); a.layer = li;
      wkv_kernel<<<d.H, 1024, wkv_smem, s>>>(a);
    }
    auto gemv_phase = [&](const PackedView& w, int mode, int lg, const float* src, const float* lnw,
                          const float* lnb, const float* prev, const float* mixv, float* ln_out, float* out,
                          const float* resid, int relu2, float* sdst, const float* ssrc, int argmax, int grid_target) {
      GemvPhaseArgs a;
      memset(&a, 0, sizeof(a));
      a.w = w; a.mode = mode; a.lg = lg;
      a.rpc = (w.rows + grid_target - 1) / grid_target;
      a.src = src; a.ln_w = lnw; a.ln_b = lnb; a.prev = prev; a.mixv = mixv; a.ln_out = ln_out;
      a.out = out; a.resid = resid; a.relu2 = relu2; a.state_dst = sdst; a.state_src = ssrc;
      a.pf = pf_for(phase++); a.argmax = argmax; a.b = e->b; a.d = d;
      const int grid = (w.rows + a.rpc - 1) / a.rpc;
      const size_t smem = (size_t)(2 * w.cols + w.cols / 16 + 4) * sizeof(float);
      gemv_phase_kernel<<<grid, kThreads, smem, s>>>(a);
      return grid;
    };
    const int gt = 2 * e->sms;
    // att_out: x_b = x_a + Wo @ att_y ; att_x[l] <- ln1(x_a)
    gemv_phase(l.o, l.mode_o, l.lg_o, e->b.att_y, nullptr, nullptr, nullptr, nullptr, nullptr, e->b.xb, e->b.xa, 0,
               e->b.att_x + (size_t)li * d.C, e->b.xln1, 0, gt);
    // ffn_in: h = relu(Wk @ mix(ln2(x_b), ffn_x[l]))^2 ; xln2 <- ln2(x_b)
    gemv_phase(l.fk, l.mode_fk, l.lg_fk, e->b.xb, l.ln2_w, l.ln2_b, e->b.ffn_x + (size_t)li * d.C, l.ffn_x_k,
               e->b.xln2, e->b.h, nullptr, 1, nullptr, nullptr, 0, gt);
    // ffn_out: x_a = x_b + Wv @ h ; ffn_x[l] <- ln2(x_b)
    gemv_phase(l.fv, l.mode_fv, l.lg_fv, e->b.h, nullptr, nullptr, nullptr, nullptr, nullptr, e->b.xa, e->b.xb, 0,
               e->b.ffn_x + (size_t)li * d.C, e->b.xln2, 0, gt);
    e->launches += 5;
  }
  {
    GemvPhaseArgs a;
    memset(&a, 0, sizeof(a));
    a.w = e->head; a.mode = e->head_mode; a.lg = e->head_lg;
    a.rpc = (e->head.rows + e->head_grid - 1) / e->head_grid;
    a.src = e->b.xa; a.ln_w = e->lnout_w; a.ln_b = e->lnout_b;
    a.out = e->b.logits; a.pf = pf_for(phase++); a.argmax = 1; a.b = e->b; a.d = d;
    const int grid = (e->head.rows + a.rpc - 1) / a.rpc;
    const size_t smem = (size_t)(2 * e->head.cols + e->head.cols / 16 + 4) * sizeof(float);
    gemv_phase_kernel<<<grid, kThreads, smem, s>>>(a);
    ++e->launches;
  }
  return cuda_status(cudaGetLastError());
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

}  // namespace

extern "C" int rwkvb_engine_create(const rwkvb_model_desc* m, uint32_t flags, rwkvb_engine** out) {
  if (!m || !out || !m->layers) return RWKVB_EARG;
  *out = nullptr;
  const int L = m->n_layer, C = m->n_embd, N = m->head_size, F = m->ffn, V = m->vocab;
  if (L <= 0 || C <= 0 || F <= 0 || V <= 0 || N != 64 || C % 64 != 0 || C % 16 != 0 || F % 16 != 0)
    return RWKVB_EUNSUPPORTED;
  if (!desc_ok(m->emb, V, C) || !desc_ok(m->head, V, C)) return RWKVB_EARG;
  if (!m->ln0_w || !m->ln0_b || !m->ln_out_w || !m->ln_out_b) return RWKVB_EARG;
  const rwkvb_layer_desc& l0 = m->layers[0];
  const int rw = l0.w1.cols, ra = l0.a1.cols, rg = l0.g1.cols, rv = l0.v1.cols;
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
  if (rw + ra + rg + rv > 4096 || rw <= 0 || ra <= 0 || rg <= 0) return RWKVB_EUNSUPPORTED;

  rwkvb_engine* e = new (std::nothrow) rwkvb_engine();
  if (!e) return RWKVB_EALLOC;
  cudaGetDevice(&e->dev);
  e->sms = device_sms();
  e->flags = flags;
  e->pf_dist = (int)((flags >> 4) & 0xF);  // bits 4..7: prefetch distance (0 = off)
  if (!(flags & 0x100u)) e->pf_dist = 1;    // bit 8 set: use the explicit distance
  Dims& d = e->d;
  d.L = L; d.C = C; d.H = C / 64; d.F = F; d.V = V;
  d.rw = rw; d.ra = ra; d.rg = rg; d.rv = rv; d.rtot = rw + ra + rg + rv;
  d.adp_rows = C >= 2048 ? 64 : 128;
  d.adp_splits = (C + d.adp_rows - 1) / d.adp_rows;
  d.hist_cap = 1 << 16;
  for (int i = 0; i < L; ++i) e->layers.push_back(make_layer(m->layers[i]));
  e->emb = make_view(m->emb);
  e->head = make_view(m->head);
  e->head_mode = gemv_mode(e->head);
  e->head_lg = ilog2u(e->head.group);
  e->ln0_w = m->ln0_w; e->ln0_b = m->ln0_b; e->lnout_w = m->ln_out_w; e->lnout_b = m->ln_out_b;
  e->head_grid = 2 * e->sms;

  // one arena for every engine-owned buffer
  const size_t H = d.H;
  size_t fl[] = {(size_t)L * C, (size_t)L * H * 4096, (size_t)L * C, (size_t)C, (size_t)C, (size_t)C, (size_t)C,
                 (size_t)3 * C, (size_t)d.adp_splits * d.rtot, (size_t)C, (size_t)F, (size_t)C, (size_t)V,
                 (size_t)e->head_grid + 8};
  size_t total = 0;
  size_t offs[16];
  for (int i = 0; i < 14; ++i) {
    offs[i] = total;
    total += ((fl[i] * 4 + 255) / 256) * 256;
  }
  const size_t ints_off = total;
  total += ((size_t)(e->head_grid + 8) * 4 + 255) / 256 * 256;  // amax_i
  const size_t misc_off = total;
  total += 256;                                                  // ticket, tok, step, err
  const size_t hist_off = total;
  total += (size_t)d.hist_cap * 4;
  if (cudaMalloc(&e->arena, total) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return RWKVB_EALLOC;
  }
  e->arena_bytes = total;
  cudaMemset(e->arena, 0, total);
  char* base = (char*)e->arena;
  float** fb[] = {&e->b.att_x, &e->b.wkv, &e->b.ffn_x, &e->b.xa, &e->b.xb, &e->b.xln1, &e->b.xln2,
                  &e->b.rkv, &e->b.adp, &e->b.att_y, &e->b.h, &e->b.v_first, &e->b.logits, &e->b.amax_v};
  for (int i = 0; i < 14; ++i) *fb[i] = (float*)(base + offs[i]);
  e->b.amax_i = (int*)(base + ints_off);
  e->b.ticket = (unsigned*)(base + misc_off);
  e->b.tok = (int*)(base + misc_off + 16);
  e->b.step = (int*)(base + misc_off + 32);
  e->b.err = (int*)(base + misc_off + 48);
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
  const size_t big = (size_t)(2 * (F > C ? F : C) + (F > C ? F : C) / 16 + 4) * sizeof(float);
  if (big > kMaxSmem) st = RWKVB_EUNSUPPORTED;
  if (st == RWKVB_OK && big > 48 * 1024) st = allow_big_smem((const void*)gemv_phase_kernel);
  if (st == RWKVB_OK) st = allow_big_smem((const void*)att_in_kernel);
  if (st == RWKVB_OK) st = allow_big_smem((const void*)wkv_kernel);
  if (st == RWKVB_OK) st = allow_big_smem((const void*)embed_kernel);
  if (st == RWKVB_OK) st = cuda_status(cudaStreamCreateWithFlags(&e->cap, cudaStreamNonBlocking));
  if (st == RWKVB_OK) st = cuda_status(cudaDeviceSynchronize());
  if (st != RWKVB_OK) {
    rwkvb_engine_destroy(e);
    return st;
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
    return RWKVB_EARG;
  }
  return RWKVB_OK;
}

extern "C" int rwkvb_engine_forward(rwkvb_engine* e, const int32_t* tokens, int32_t n, void* stream) {
  if (!e || (!tokens && n > 0) || n < 0) return RWKVB_EARG;
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->d.V) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
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
    if (st == RWKVB_OK && done + chunk < n) {
      // restart the history ring; the next step still consumes the last argmax
      st = cuda_status(cudaMemsetAsync(e->b.step, 0, sizeof(int), s));
    }
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
  int st2 = cuda_status(cudaStreamSynchronize(s));
  if (st == RWKVB_OK) st = st2;
  if (st == RWKVB_OK) st = check_err_flag(e, s);
  return st;
}

extern "C" int rwkvb_engine_launches_per_step(rwkvb_engine* e, int32_t* out) {
  if (!e || !out) return RWKVB_EARG;
  *out = 2 + 5 * e->d.L;
  return RWKVB_OK;
}
