// Persistent decode kernel: the whole greedy decode loop (every layer of every
// token) in one cooperative launch, one CTA of 512 threads per SM.
//
// Each CTA owns a fixed slice of every projection's rows.  Its weight rows are
// streamed in execution order through a shared-memory ring by 1-D TMA bulk
// copies; the ring runs ahead across phase boundaries, so HBM keeps streaming
// while the CTAs meet at the grid barriers that the RWKV-7 data flow needs
// (5 per layer: r/k/v+adapters -> WKV -> output proj -> FFN key -> FFN value).
// Every wait (ring slot, grid barrier) is bounded; a timeout sets the engine's
// error word, drains this CTA's in-flight copies and ends the kernel.
//
// Included by engine.cu after LayerDev / Bufs / Dims.
#pragma once

namespace rwkvb {

constexpr int kPThreads = 512;
constexpr int kPWarps = kPThreads / 32;

// Geometry of one projection width K (all ring matrices share the group size).
struct PGeom {
  int K, gpr, nseg, kseg, cpl, rs;
  uint32_t row_bytes;
};

struct PArgs {
  const LayerDev* layers;  // device array [L]
  PackedView emb, head;
  const float *ln0_w, *ln0_b, *lnout_w, *lnout_b;
  Bufs b;
  Dims d;
  PGeom gc, gf;       // K = n_embd, K = ffn
  int lg;             // log2(group) of the ring matrices
  int nst;            // ring slots
  uint32_t slot_bytes;
  int ntok, mode;     // mode 0: greedy (step 0 consumes first_tok); 1: forced tokens
  int first_tok;
  const int* forced;  // mode 1 token list
  unsigned* gbar;     // grid barrier counter, zero at launch
  uint32_t spin_limit;
  int emb_fast;
  unsigned long long* trace;  // optional phase timestamps: [2][trace_cap] (CTA 0, last CTA)
  int trace_cap;
  // shared-memory offsets (bytes)
  uint32_t o_bars, o_part, o_x, o_ln, o_wkv, o_xb, o_ln2, o_misc, smem_total;
};

// ---------------------------------------------------------------- cursor
// Stage sequence of one CTA: per token, per layer phases A (r/k/v rows of the
// concatenated [3C] rows, then first-adapter items), C (att_out rows),
// D (ffn key rows), E (ffn value rows); then the head rows.  The per-CTA row
// ranges and stage counts are computed once into shared memory (PTable); only
// thread 0 walks the issue cursor, and each issued stage's descriptor is kept
// beside its ring slot for the consumers.
struct Cursor {
  int tok, layer, phase, j;  // phase 0 A, 1 C, 2 D, 3 E, 4 head
};

struct Stage {
  const uint8_t* q;
  const uint8_t* s;
  uint32_t qb, sb;
  int kind;   // 0 GEMV rows, 1 first-adapter item
  int mat;    // GEMV: 0 r,1 k,2 v,3 o,4 fk,5 fv,6 head ; adapter: 0 w1,1 a1,2 g1,3 v1
  int row0, nrows;  // GEMV rows / adapter row range
  int item;         // adapter split index
};

constexpr int kMaxItems = 8;
constexpr int kMaxLayers = 64;

// Per-layer source pointers used by the issue cursor, kept in shared memory so
// that refilling a slot never waits on a global load.
struct LayerSrc {
  const uint8_t* pay[6];   // r, k, v, o, fk, fv code payloads
  const uint8_t* meta[6];  // their scale pairs
  const uint8_t* apay[4];  // first adapters w1, a1, g1, v1
  const uint8_t* ameta[4];
  int acols[4], alg[4];
};

struct PTable {
  int npiece;                  // phase A r/k/v pieces (<= 3)
  int pm[3], pr0[3], pr1[3], pn[3];
  int nrkv;                    // phase A r/k/v stages
  int nitem[2];                // adapter items: [0] layer 0 (3 matrices), [1] other layers
  int item[kMaxItems];         // global item ids (matrix * splits + split), ascending
  int r0[4], r1[4], n[4];      // phases C, D, E, head
};

__device__ __forceinline__ void split_rows(int n, int parts, int i, int* a, int* b) {
  const int base = n / parts, rem = n % parts;
  *a = i * base + min(i, rem);
  *b = *a + base + (i < rem ? 1 : 0);
}

__device__ __forceinline__ int nstages(int rows, int rs) { return rows > 0 ? (rows + rs - 1) / rs : 0; }

// Fill the table (thread 0).
__device__ __forceinline__ void build_table(const PArgs& a, PTable& T) {
  const int G = gridDim.x, bx = blockIdx.x, C = a.d.C;
  int r0, r1;
  split_rows(3 * C, G, bx, &r0, &r1);
  T.npiece = 0;
  T.nrkv = 0;
  for (int m = 0; m < 3; ++m) {
    const int lo = max(r0, m * C), hi = min(r1, (m + 1) * C);
    if (hi > lo) {
      const int k = T.npiece++;
      T.pm[k] = m;
      T.pr0[k] = lo - m * C;
      T.pr1[k] = hi - m * C;
      T.pn[k] = nstages(hi - lo, a.gc.rs);
      T.nrkv += T.pn[k];
    }
  }
  const int items3 = 3 * a.d.adp_splits, items4 = 4 * a.d.adp_splits;
  T.nitem[0] = T.nitem[1] = 0;
  for (int it = bx; it < items4 && T.nitem[1] < kMaxItems; it += G) {
    T.item[T.nitem[1]++] = it;
    if (it < items3) T.nitem[0] = T.nitem[1];
  }
  const int rows[4] = {C, a.d.F, C, a.d.V};
  const int rs[4] = {a.gc.rs, a.gc.rs, a.gf.rs, a.gc.rs};
  for (int p = 0; p < 4; ++p) {
    split_rows(rows[p], G, bx, &T.r0[p], &T.r1[p]);
    T.n[p] = nstages(T.r1[p] - T.r0[p], rs[p]);
  }
}

__device__ __forceinline__ int phase_count(const PTable& T, int l, int ph) {
  return ph == 0 ? T.nrkv + T.nitem[l == 0 ? 0 : 1] : T.n[ph - 1];
}

__device__ __forceinline__ const PackedView& gemv_mat(const PArgs& a, int l, int mat) {
  const LayerDev& L = a.layers[l];
  switch (mat) {
    case 0: return L.r;
    case 1: return L.k;
    case 2: return L.v;
    case 3: return L.o;
    case 4: return L.fk;
    case 5: return L.fv;
    default: return a.head;
  }
}

__device__ __forceinline__ const PackedView& adp_mat(const PArgs& a, int l, int m) {
  const LayerDev& L = a.layers[l];
  return m == 0 ? L.w1 : (m == 1 ? L.a1 : (m == 2 ? L.g1 : L.v1));
}

// Move to the first stage at or after `c`; false when the launch is done.
__device__ __forceinline__ bool cursor_norm(const PArgs& a, const PTable& T, Cursor& c) {
  while (c.tok < a.ntok) {
    if (c.j < phase_count(T, c.layer, c.phase)) return true;
    c.j = 0;
    if (c.phase == 4) {
      c.phase = 0;
      c.layer = 0;
      ++c.tok;
    } else if (c.phase == 3) {
      if (c.layer + 1 < a.d.L) {
        ++c.layer;
        c.phase = 0;
      } else {
        c.phase = 4;
      }
    } else {
      ++c.phase;
    }
  }
  return false;
}

__device__ __forceinline__ Stage stage_of(const PArgs& a, const PTable& T, const LayerSrc* LS, const Cursor& c) {
  Stage s;
  s.kind = 0;
  s.item = 0;
  int r0 = 0, r1 = 0, mat = 0, j = c.j;
  const PGeom* g = &a.gc;
  if (c.phase == 0) {
    if (j < T.nrkv) {
      int k = 0;
      while (j >= T.pn[k]) j -= T.pn[k++];
      mat = T.pm[k];
      r0 = T.pr0[k] + j * a.gc.rs;
      r1 = min(T.pr1[k], r0 + a.gc.rs);
    } else {
      const int item = T.item[j - T.nrkv];
      const int m = item / a.d.adp_splits, sp = item - m * a.d.adp_splits;
      const LayerSrc& ls = LS[c.layer];
      const int R = ls.acols[m], lgm = ls.alg[m];
      const int i0 = sp * a.d.adp_rows, i1 = min(a.d.C, i0 + a.d.adp_rows);
      const uint32_t g0 = (uint32_t)(((uint64_t)i0 * R) >> lgm);
      const uint32_t g1 = (uint32_t)((((uint64_t)i1 * R - 1) >> lgm) + 1);
      const uint32_t g0a = g0 & ~1u, g1a = (g1 + 1) & ~1u;  // 16-byte aligned pair range
      s.kind = 1;
      s.mat = m;
      s.item = sp;
      s.row0 = i0;
      s.nrows = i1 - i0;
      s.q = ls.apay[m] + (size_t)i0 * R;
      s.qb = (uint32_t)((i1 - i0) * R);
      s.s = ls.ameta[m] + (size_t)g0a * 8;
      s.sb = (g1a - g0a) * 8u;
      return s;
    }
  } else {
    const int p = c.phase - 1;
    const int rs = p == 2 ? a.gf.rs : a.gc.rs;
    if (p == 2) g = &a.gf;
    mat = p == 0 ? 3 : (p == 1 ? 4 : (p == 2 ? 5 : 6));
    r0 = T.r0[p] + j * rs;
    r1 = min(T.r1[p], r0 + rs);
  }
  const uint8_t* pay = mat == 6 ? a.head.payload : LS[c.layer].pay[mat];
  const uint8_t* meta = mat == 6 ? a.head.meta : LS[c.layer].meta[mat];
  s.mat = mat;
  s.row0 = r0;
  s.nrows = r1 - r0;
  s.q = pay + (size_t)r0 * g->K;
  s.qb = (uint32_t)(s.nrows * g->K);
  s.s = meta + (size_t)r0 * g->gpr * 8;
  s.sb = (uint32_t)s.nrows * (uint32_t)g->gpr * 8u;
  return s;
}

__device__ __forceinline__ void issue_stage(const PArgs& a, uint8_t* smb, uint64_t* bars, int slot, const Stage& s) {
  uint8_t* dst = smb + (size_t)slot * a.slot_bytes;
  mbar_expect_tx(&bars[slot], s.qb + s.sb);
  bulk_g2s(dst, s.q, s.qb, &bars[slot]);
  // scales / pairs after the codes, 16-byte aligned
  bulk_g2s(dst + ((s.qb + 15u) & ~15u), s.s, s.sb, &bars[slot]);
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long v;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(v));
  return v;
}

// --------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// All CTAs meet; returns false (CTA-uniform) if the bounded wait gave up.
__device__ __forceinline__ bool grid_sync(const PArgs& a, unsigned& target, int* flag) {
  __syncthreads();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.gbar, 1u);
    bool ok = false;
    for (uint32_t i = 0; i < a.spin_limit; ++i) {
      if (ld_acquire(a.gbar) >= target) { ok = true; break; }
      __nanosleep(64);
    }
    *flag = ok ? 0 : 1;
    if (!ok) atomicOr(a.b.err, kErrTimeout);
  }
  __syncthreads();
  return *flag == 0;
}

// ------------------------------------------------------------- GEMV stage
// Rows [row0, row0+nr) of the slot times the input held in registers (x of
// this warp's K segment).  Writes per-(row, segment) partials.
template <int CPL>
__device__ __forceinline__ void gemv_stage(const uint8_t* slot, const PGeom& g, int lg, int nr, const float (&xr)[CPL][16],
                                           const float (&xs)[CPL], float* part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = warp % g.nseg, wsub = warp / g.nseg, wper = kPWarps / g.nseg;
  const int nchunk = g.kseg >> 4, gshift = lg - 4;
  // scale pairs follow this stage's codes (nr rows), 16-byte aligned
  const float2* ss = reinterpret_cast<const float2*>(slot + (((uint32_t)nr * g.K + 15u) & ~15u));
  for (int ri = wsub; ri < nr; ri += wper) {
    const uint8_t* q = slot + (size_t)ri * g.K + seg * g.kseg;
    const float2* sc = ss + ri * g.gpr + ((seg * g.kseg) >> lg);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane + 32 * j;
      if (c < nchunk) {
        const uint4 qq = *reinterpret_cast<const uint4*>(q + c * 16);
        const float2 s = sc[c >> gshift];
        float2 d = make_float2(0.f, 0.f);
        d = dot4_u8(qq.x, make_float4(xr[j][0], xr[j][1], xr[j][2], xr[j][3]), d);
        d = dot4_u8(qq.y, make_float4(xr[j][4], xr[j][5], xr[j][6], xr[j][7]), d);
        d = dot4_u8(qq.z, make_float4(xr[j][8], xr[j][9], xr[j][10], xr[j][11]), d);
        d = dot4_u8(qq.w, make_float4(xr[j][12], xr[j][13], xr[j][14], xr[j][15]), d);
        acc = fmaf((s.y - s.x) * kInv255, d.x + d.y, fmaf(s.x, xs[j], acc));
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) part[ri * g.nseg + seg] = acc;
  }
}

// Load this warp's input segment (x = xin4(i), 4 at a time) into registers.
template <int CPL, class XIn>
__device__ __forceinline__ void load_x(const PGeom& g, XIn xin4, float (&xr)[CPL][16], float (&xs)[CPL]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = warp % g.nseg, nchunk = g.kseg >> 4;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = lane + 32 * j;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 v = c < nchunk ? xin4(seg * g.kseg + c * 16 + 4 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
      xr[j][4 * u] = v.x;
      xr[j][4 * u + 1] = v.y;
      xr[j][4 * u + 2] = v.z;
      xr[j][4 * u + 3] = v.w;
    }
  }
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) sum += xr[j][e];
    xs[j] = sum;
  }
}

// ----------------------------------------------------------- the kernel
template <int CPL>
__global__ void __launch_bounds__(kPThreads, 1) persistent_kernel(PArgs a) {
  extern __shared__ __align__(128) uint8_t smb[];
  __shared__ float red[32];
  __shared__ int flag;
  __shared__ int s_tok;
  __shared__ float s_bv[kPWarps];
  __shared__ int s_bi[kPWarps];
  __shared__ PTable T;
  __shared__ Stage sdesc[8];  // descriptor of the stage held by each ring slot
  __shared__ LayerSrc LS[kMaxLayers];

  const int C = a.d.C, F = a.d.F, G = gridDim.x, bx = blockIdx.x, t = threadIdx.x;
  const int lane = t & 31, wid = t >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smb + a.o_bars);
  float* part = reinterpret_cast<float*>(smb + a.o_part);
  float* X = reinterpret_cast<float*>(smb + a.o_x);     // residual stream (layer input) [C]
  float* LN = reinterpret_cast<float*>(smb + a.o_ln);   // ln1(X) [C]
  float* XB = reinterpret_cast<float*>(smb + a.o_xb);   // after attention [C] (aliases wkv area)
  float* LN2 = reinterpret_cast<float*>(smb + a.o_ln2); // ln2(XB) [C]
  uint8_t* wk = smb + a.o_wkv;                           // WKV head scratch
  float* misc = reinterpret_cast<float*>(smb + a.o_misc);
  unsigned target = 0;
  bool alive = true;
  int tr = 0;  // trace slot
  const int trow = bx == 0 ? 0 : (bx == G - 1 ? 1 : -1);
  auto mark = [&]() {
    if (a.trace && trow >= 0 && t == 0 && tr < a.trace_cap) a.trace[(size_t)trow * a.trace_cap + tr] = global_ns();
    ++tr;
  };

  // ---- per-layer source table, then the ring prologue
  for (int l = t; l < a.d.L; l += kPThreads) {
    const LayerDev& L = a.layers[l];
    const PackedView* gm[6] = {&L.r, &L.k, &L.v, &L.o, &L.fk, &L.fv};
    for (int m = 0; m < 6; ++m) { LS[l].pay[m] = gm[m]->payload; LS[l].meta[m] = gm[m]->meta; }
    const PackedView* am[4] = {&L.w1, &L.a1, &L.g1, &L.v1};
    for (int m = 0; m < 4; ++m) {
      LS[l].apay[m] = am[m]->payload;
      LS[l].ameta[m] = am[m]->meta;
      LS[l].acols[m] = am[m]->cols;
      LS[l].alg[m] = am[m]->lg;
    }
  }
  __syncthreads();
  Cursor ic{0, 0, 0, 0};
  if (t == 0) {
    build_table(a, T);
    for (int i = 0; i < a.nst; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    for (int i = 0; i < a.nst; ++i) {
      if (!cursor_norm(a, T, ic)) break;
      sdesc[i] = stage_of(a, T, LS, ic);
      issue_stage(a, smb, bars, i, sdesc[i]);
      ++ic.j;
    }
  }
  __syncthreads();
  int seq = 0;  // stages consumed by this CTA

  float xr[CPL][16];
  float xs[CPL];
  int xr_tag = -1;  // which input the registers hold

  // Wait for the next stage, run compute(stage, slot, partials) while the slot
  // is live, refill the slot, then run epi(stage, partials).
  auto consume = [&](auto compute, auto epi) -> bool {
    const int slot = seq % a.nst;
    // every thread polls the slot's barrier (bounded); the CTA agrees on the outcome
    const bool got = mbar_wait_bounded(&bars[slot], (uint32_t)((seq / a.nst) & 1), a.spin_limit);
    if (!__syncthreads_and(got)) {
      if (t == 0) atomicOr(a.b.err, kErrTimeout);
      return false;
    }
    const Stage st = sdesc[slot];
    float* pt = part + (seq & 1) * 512;
    compute(st, smb + (size_t)slot * a.slot_bytes, pt);
    __syncthreads();
    if (t == 0 && cursor_norm(a, T, ic)) {
      sdesc[slot] = stage_of(a, T, LS, ic);
      issue_stage(a, smb, bars, slot, sdesc[slot]);
      ++ic.j;
    }
    epi(st, pt);
    ++seq;
    return true;
  };

  // LayerNorm in place over smem v[0..C) with weight/bias (eps 1e-5)
  auto layer_norm = [&](float* v, const float* w, const float* bb) {
    float s = 0.f;
    for (int i = t; i < C; i += kPThreads) s += v[i];
    const float mean = block_sum(s, red) / (float)C;
    float q = 0.f;
    for (int i = t; i < C; i += kPThreads) { const float d = v[i] - mean; q += d * d; }
    const float rstd = rsqrtf(block_sum(q, red) / (float)C + 1e-5f);
    for (int i = t; i < C; i += kPThreads) v[i] = (v[i] - mean) * rstd * __ldg(w + i) + __ldg(bb + i);
    __syncthreads();
  };

  auto load_vec = [&](float* dst, const float* src, int n) {
    for (int i = t; i < (n >> 2); i += kPThreads)
      reinterpret_cast<float4*>(dst)[i] = ldcg4(src + 4 * i);
    __syncthreads();
  };

  int tok = a.mode == 0 ? (a.first_tok >= 0 ? a.first_tok : __ldcg(a.b.tok)) : __ldg(a.forced);
  for (int step = 0; step < a.ntok && alive; ++step) {
    if (a.mode == 1) tok = __ldg(a.forced + step);
    if (tok < 0 || tok >= a.d.V) {
      if (t == 0) atomicOr(a.b.err, kErrToken);
      tok = 0;
    }
    mark();  // token start
    // ---- embedding + ln0 (every CTA, locally)
    {
      const PackedView& E = a.emb;
      if (a.emb_fast) {
        const int gpr = C >> E.lg;
        uint8_t* q = reinterpret_cast<uint8_t*>(LN);
        float2* sc = reinterpret_cast<float2*>(q + C);
        cp_async_block(q, E.payload + (size_t)tok * C, (uint32_t)C);
        cp_async_block(sc, E.meta + (size_t)tok * gpr * 8, (uint32_t)gpr * 8u);
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
        for (int i = t; i < C; i += kPThreads) {
          const float2 s = sc[i >> E.lg];
          X[i] = sg8_dequant(q[i], s.x, s.y);
        }
      } else {
        for (int i = t; i < C; i += kPThreads) X[i] = packed_at(E, tok, i);
      }
      __syncthreads();
      layer_norm(X, a.ln0_w, a.ln0_b);
    }

    for (int l = 0; l < a.d.L && alive; ++l) {
      const LayerDev& Ly = a.layers[l];
      const float* prev_att = a.b.att_x + (size_t)l * C;
      if (l > 0) {
        if (!grid_sync(a, target, &flag)) { alive = false; break; }
        load_vec(X, a.b.xa, C);
      }
      mark();  // A start (x ready)
      // ======== phase A: ln1, mixes, r/k/v rows, first adapters
      for (int i = t; i < C; i += kPThreads) LN[i] = X[i];
      __syncthreads();
      layer_norm(LN, Ly.ln1_w, Ly.ln1_b);
      xr_tag = -1;
      const int nA = phase_count(T, l, 0);
      for (int k = 0; k < nA && alive; ++k) {
        alive = consume(
            [&](const Stage& st, const uint8_t* slot, float* pt) {
              if (st.kind == 0) {
                const float* mix = st.mat == 0 ? Ly.x_r : (st.mat == 1 ? Ly.x_k : Ly.x_v);
                if (xr_tag != st.mat) {
                  load_x<CPL>(a.gc, [&](int i) {
                    const float4 z = *reinterpret_cast<const float4*>(LN + i);
                    const float4 p = ldcg4(prev_att + i), m = ldg4(mix + i);
                    return make_float4(z.x + (p.x - z.x) * m.x, z.y + (p.y - z.y) * m.y, z.z + (p.z - z.z) * m.z,
                                       z.w + (p.w - z.w) * m.w);
                  }, xr, xs);
                  xr_tag = st.mat;
                }
                gemv_stage<CPL>(slot, a.gc, a.lg, st.nrows, xr, xs, pt);
              } else {
                // first adapter item: rows [row0, row0+nrows) of W [C, R] (x @ W)
                const float* mix = st.mat == 0 ? Ly.x_w : (st.mat == 1 ? Ly.x_a : (st.mat == 2 ? Ly.x_g : Ly.x_v));
                const int R = LS[l].acols[st.mat], nr = st.nrows, wlg = LS[l].alg[st.mat];
                float* xm = misc;  // [nr] mixed input
                for (int i = t; i < nr; i += kPThreads) {
                  const int gi = st.row0 + i;
                  xm[i] = LN[gi] + (__ldcg(prev_att + gi) - LN[gi]) * __ldg(mix + gi);
                }
                __syncthreads();
                const uint8_t* cq = slot;
                const float2* cs = reinterpret_cast<const float2*>(slot + ((st.qb + 15u) & ~15u));
                const uint32_t g0 = ((uint32_t)(((uint64_t)st.row0 * R) >> wlg)) & ~1u;
                const int nrg = kPThreads / R;  // row groups
                if (t < nrg * R) {
                  const int j = t % R, rg = t / R;
                  float acc = 0.f;
                  for (int i = rg; i < nr; i += nrg) {
                    const uint32_t e = (uint32_t)(st.row0 + i) * (uint32_t)R + (uint32_t)j;
                    const float2 sc = cs[(e >> wlg) - g0];
                    acc = fmaf(xm[i], sg8_dequant(cq[i * R + j], sc.x, sc.y), acc);
                  }
                  misc[256 + rg * R + j] = acc;
                }
              }
            },
            [&](const Stage& st, float* pt) {
              if (st.kind == 0) {
                if (t < st.nrows) {
                  float v = 0.f;
                  for (int s = 0; s < a.gc.nseg; ++s) v += pt[t * a.gc.nseg + s];
                  a.b.rkv[(size_t)st.mat * C + st.row0 + t] = v;
                }
              } else {
                const int R = LS[l].acols[st.mat];
                const int nrg = kPThreads / R;
                const int off = st.mat == 0 ? 0 : (st.mat == 1 ? a.d.rw : (st.mat == 2 ? a.d.rw + a.d.ra : a.d.rw + a.d.ra + a.d.rg));
                for (int j = t; j < R; j += kPThreads) {
                  float v = 0.f;
                  for (int rg = 0; rg < nrg; ++rg) v += misc[256 + rg * R + j];
                  a.b.adp[(size_t)st.item * a.d.rtot + off + j] = v;
                }
                __syncthreads();  // misc is reused by the next adapter item
              }
            });
      }
      if (!alive) break;
      mark();  // phase A done
      // ======== phase B: one head per CTA (head h = bx)
      const int H = a.d.H;
      const bool has_head = bx < H;
      const int nm = l == 0 ? 3 : 4;
      float* S = reinterpret_cast<float*>(wk);            // [64][64]
      float* mid = S + 4096;                              // [rtot]
      float* vec = mid + ((a.d.rtot + 3) & ~3);           // 4 x 64
      float* sr = vec + 256;
      float* sd = sr + 64;
      float* sk = sd + 64;
      float* sv = sk + 64;
      float* skk = sv + 64;
      float* ska = skk + 64;
      float* sy = ska + 64;
      float2* tsc = reinterpret_cast<float2*>(sy + 64);   // [rtot]
      uint8_t* tq = reinterpret_cast<uint8_t*>(tsc + a.d.rtot);  // [rtot][64]
      float* Sg = a.b.wkv + ((size_t)l * H + bx) * 4096;
      if (has_head) {
        // constant second-adapter tiles and this CTA's own head state: before the barrier
        int off = 0;
        for (int m = 0; m < nm; ++m) {
          const PackedView& W = m == 0 ? Ly.w2 : (m == 1 ? Ly.a2 : (m == 2 ? Ly.g2 : Ly.v2));
          for (int u = t; u < W.rows * 4; u += kPThreads) {
            const int i = u >> 2, p = u & 3;
            cp_async16(tq + (size_t)(off + i) * 64 + p * 16, W.payload + (size_t)i * C + bx * 64 + p * 16);
          }
          for (int i = t; i < W.rows; i += kPThreads)
            tsc[off + i] = __ldg(reinterpret_cast<const float2*>(W.meta) + (((size_t)i * C + bx * 64) >> W.lg));
          off += W.rows;
        }
        for (int u = t; u < 1024; u += kPThreads) cp_async16(S + u * 4, Sg + u * 4);
        cp_async_commit();
      }
      if (!grid_sync(a, target, &flag)) { alive = false; break; }
      mark();  // B barrier
      if (has_head) {
        const int h = bx;
        const int used = l == 0 ? a.d.rw + a.d.ra + a.d.rg : a.d.rtot;
        for (int j = t; j < used; j += kPThreads) {
          float acc = 0.f;
          for (int s0 = 0; s0 < a.d.adp_splits; s0 += 24) {
            float v[24];
#pragma unroll
            for (int u = 0; u < 24; ++u)
              v[u] = s0 + u < a.d.adp_splits ? __ldcg(a.b.adp + (size_t)(s0 + u) * a.d.rtot + j) : 0.f;
#pragma unroll
            for (int u = 0; u < 24; ++u) acc += v[u];
          }
          if (j < a.d.rw) acc = tanhf(acc);
          else if (j >= a.d.rw + a.d.ra && j < a.d.rw + a.d.ra + a.d.rg) acc = sigmoidf_(acc);
          mid[j] = acc;
        }
        float r = 0.f, k = 0.f, v = 0.f, vf = 0.f;
        if (t < 64) {
          const int ch = h * 64 + t;
          r = __ldcg(a.b.rkv + ch);
          k = __ldcg(a.b.rkv + C + ch);
          v = __ldcg(a.b.rkv + 2 * C + ch);
          if (l != 0) vf = __ldcg(a.b.v_first + ch);
        }
        cp_async_wait_all();
        __syncthreads();
        {
          // thread -> (matrix m, channel c, half q of the rank)
          const int q = t & 1, c = (t >> 1) & 63, m = t >> 7;
          const int off = m == 0 ? 0 : (m == 1 ? a.d.rw : (m == 2 ? a.d.rw + a.d.ra : a.d.rw + a.d.ra + a.d.rg));
          const int R = m == 0 ? a.d.rw : (m == 1 ? a.d.ra : (m == 2 ? a.d.rg : a.d.rv));
          float acc = 0.f;
          if (m < nm) {
            for (int i = q; i < R; i += 2) {
              const float2 sc = tsc[off + i];
              acc = fmaf(mid[off + i], sg8_dequant(tq[(size_t)(off + i) * 64 + c], sc.x, sc.y), acc);
            }
          }
          acc += __shfl_xor_sync(0xffffffffu, acc, 1);
          if (q == 0 && m < nm) vec[m * 64 + c] = acc;
        }
        __syncthreads();
        const float kkv = t < 64 ? k * Ly.k_k[h * 64 + t] : 0.f;
        const float nrm = sqrtf(block_sum(kkv * kkv, red));
        if (t < 64) {
          const int ch = h * 64 + t;
          const float aa = sigmoidf_(Ly.a0[ch] + vec[64 + t]);
          const float kk = kkv / fmaxf(nrm, 1e-12f);
          const float kn = k * (1.0f + (aa - 1.0f) * Ly.k_a[ch]);
          if (l == 0) a.b.v_first[ch] = v;
          else v = v + (vf - v) * sigmoidf_(Ly.v0[ch] + vec[192 + t]);
          sr[t] = r;
          sd[t] = expf(-0.606531f * sigmoidf_(Ly.w0[ch] + vec[t]));
          sk[t] = kn;
          sv[t] = v;
          skk[t] = kk;
          ska[t] = kk * aa;
        }
        __syncthreads();
        if (t < 256) wkv7_head64(S, sr, sd, sk, sv, skk, ska, sy);
        __syncthreads();
        for (int u = t; u < 1024; u += kPThreads)
          reinterpret_cast<float4*>(Sg)[u] = reinterpret_cast<const float4*>(S)[u];
        const float yv = t < 64 ? sy[t] : 0.f;
        const float mean = block_sum(yv, red) / 64.f;
        const float dv = t < 64 ? yv - mean : 0.f;
        const float var = block_sum(dv * dv, red) / 64.f;
        const float bon = t < 64 ? sr[t] * sk[t] * Ly.r_k[h * 64 + t] : 0.f;
        const float bonus = block_sum(bon, red);
        if (t < 64) {
          const int ch = h * 64 + t;
          float o = dv * rsqrtf(var + 64e-5f) * Ly.lnx_w[ch] + Ly.lnx_b[ch];
          o = o + bonus * sv[t];
          a.b.att_y[ch] = o * vec[128 + t];
        }
      }
      mark();  // B compute done
      if (!grid_sync(a, target, &flag)) { alive = false; break; }
      mark();  // C barrier
      // ======== phase C: output projection + residual; x_prev(att) <- ln1
      xr_tag = -1;
      const int nC = phase_count(T, l, 1);
      for (int k = 0; k < nC && alive; ++k) {
        alive = consume(
            [&](const Stage& st, const uint8_t* slot, float* pt) {
              if (xr_tag != 3) {
                load_x<CPL>(a.gc, [&](int i) { return ldcg4(a.b.att_y + i); }, xr, xs);
                xr_tag = 3;
              }
              gemv_stage<CPL>(slot, a.gc, a.lg, st.nrows, xr, xs, pt);
            },
            [&](const Stage& st, float* pt) {
              if (t < st.nrows) {
                float v = 0.f;
                for (int s = 0; s < a.gc.nseg; ++s) v += pt[t * a.gc.nseg + s];
                const int row = st.row0 + t;
                a.b.xb[row] = X[row] + v;
                a.b.att_x[(size_t)l * C + row] = LN[row];
              }
            });
      }
      if (!alive) break;
      mark();  // C done
      if (!grid_sync(a, target, &flag)) { alive = false; break; }
      mark();  // D barrier
      // ======== phase D: ln2 + mix, FFN key rows, relu^2
      load_vec(XB, a.b.xb, C);
      for (int i = t; i < C; i += kPThreads) LN2[i] = XB[i];
      __syncthreads();
      layer_norm(LN2, Ly.ln2_w, Ly.ln2_b);
      const float* prev_ffn = a.b.ffn_x + (size_t)l * C;
      xr_tag = -1;
      const int nD = phase_count(T, l, 2);
      for (int k = 0; k < nD && alive; ++k) {
        alive = consume(
            [&](const Stage& st, const uint8_t* slot, float* pt) {
              if (xr_tag != 4) {
                load_x<CPL>(a.gc, [&](int i) {
                  const float4 z = *reinterpret_cast<const float4*>(LN2 + i);
                  const float4 p = ldcg4(prev_ffn + i), m = ldg4(Ly.ffn_x_k + i);
                  return make_float4(z.x + (p.x - z.x) * m.x, z.y + (p.y - z.y) * m.y, z.z + (p.z - z.z) * m.z,
                                     z.w + (p.w - z.w) * m.w);
                }, xr, xs);
                xr_tag = 4;
              }
              gemv_stage<CPL>(slot, a.gc, a.lg, st.nrows, xr, xs, pt);
            },
            [&](const Stage& st, float* pt) {
              if (t < st.nrows) {
                float v = 0.f;
                for (int s = 0; s < a.gc.nseg; ++s) v += pt[t * a.gc.nseg + s];
                a.b.h[st.row0 + t] = v > 0.f ? v * v : 0.f;
              }
            });
      }
      if (!alive) break;
      mark();  // D done
      if (!grid_sync(a, target, &flag)) { alive = false; break; }
      mark();  // E barrier
      // ======== phase E: FFN value rows + residual; x_prev(ffn) <- ln2
      xr_tag = -1;
      const int nE = phase_count(T, l, 3);
      for (int k = 0; k < nE && alive; ++k) {
        alive = consume(
            [&](const Stage& st, const uint8_t* slot, float* pt) {
              if (xr_tag != 5) {
                load_x<CPL>(a.gf, [&](int i) { return ldcg4(a.b.h + i); }, xr, xs);
                xr_tag = 5;
              }
              gemv_stage<CPL>(slot, a.gf, a.lg, st.nrows, xr, xs, pt);
            },
            [&](const Stage& st, float* pt) {
              if (t < st.nrows) {
                float v = 0.f;
                for (int s = 0; s < a.gf.nseg; ++s) v += pt[t * a.gf.nseg + s];
                const int row = st.row0 + t;
                a.b.xa[row] = XB[row] + v;
                a.b.ffn_x[(size_t)l * C + row] = LN2[row];
              }
            });
      }
      mark();  // E done
    }
    if (!alive) break;
    // ======== head: ln_out, logits, argmax
    if (!grid_sync(a, target, &flag)) { alive = false; break; }
    mark();  // head barrier
    load_vec(X, a.b.xa, C);
    layer_norm(X, a.lnout_w, a.lnout_b);
    xr_tag = -1;
    float best = -INFINITY;
    int besti = 0x7fffffff;
    const int nH = phase_count(T, 0, 4);
    for (int k = 0; k < nH && alive; ++k) {
      alive = consume(
          [&](const Stage& st, const uint8_t* slot, float* pt) {
            if (xr_tag != 6) {
              load_x<CPL>(a.gc, [&](int i) { return *reinterpret_cast<const float4*>(X + i); }, xr, xs);
              xr_tag = 6;
            }
            gemv_stage<CPL>(slot, a.gc, a.lg, st.nrows, xr, xs, pt);
          },
          [&](const Stage& st, float* pt) {
            if (t < st.nrows) {
              float v = 0.f;
              for (int s = 0; s < a.gc.nseg; ++s) v += pt[t * a.gc.nseg + s];
              const int row = st.row0 + t;
              a.b.logits[row] = v;
              if (v > best || (v == best && row < besti)) { best = v; besti = row; }
            }
          });
    }
    if (!alive) break;
    mark();  // head done
    // per-CTA argmax -> global partials -> every CTA reduces (first maximum)
    {
      float wb = best;
      int wi = besti;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, wb, o);
        const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
        if (ov > wb || (ov == wb && oi < wi)) { wb = ov; wi = oi; }
      }
      if (lane == 0) { s_bv[wid] = wb; s_bi[wid] = wi; }
      __syncthreads();
      if (t == 0) {
        float cb = -INFINITY;
        int ci = 0x7fffffff;
        for (int w = 0; w < kPWarps; ++w)
          if (s_bv[w] > cb || (s_bv[w] == cb && s_bi[w] < ci)) { cb = s_bv[w]; ci = s_bi[w]; }
        a.b.amax_v[bx] = cb;
        a.b.amax_i[bx] = ci;
      }
    }
    if (!grid_sync(a, target, &flag)) { alive = false; break; }
    if (t < 32) {
      float gb = -INFINITY;
      int gi = 0x7fffffff;
      for (int c = lane; c < G; c += 32) {
        const float v = __ldcg(a.b.amax_v + c);
        const int i = __ldcg(a.b.amax_i + c);
        if (v > gb || (v == gb && i < gi)) { gb = v; gi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, gb, o);
        const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
        if (ov > gb || (ov == gb && oi < gi)) { gb = ov; gi = oi; }
      }
      if (t == 0) s_tok = gi == 0x7fffffff ? 0 : gi;
    }
    __syncthreads();
    tok = s_tok;
    if (bx == 0 && t == 0) {
      a.b.hist[step % a.d.hist_cap] = tok;
      *a.b.tok = tok;
    }
  }
  if (!alive) {
    // drain this CTA's in-flight copies (bounded) before exiting
    if (t == 0) {
      for (int u = seq; u < seq + a.nst; ++u) mbar_wait_bounded(&bars[u % a.nst], (uint32_t)((u / a.nst) & 1), 1u << 16);
    }
    __syncthreads();
  }
}

}  // namespace rwkvb
