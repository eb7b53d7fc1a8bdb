// Batched decode: the tcgen05 SG8 GEMM (bgemm.cuh) behind the op-level entry
// rwkvb_gemm_sg8_f32, and the host plan shared with the batched engine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "bgemm.cuh"
#include "common.cuh"
#include "l2mma.cuh"
#include "internal.h"
#include "wkv7.cuh"

namespace rwkvb {

namespace {
// Dynamic shared memory of one CTA: the 227 KB opt-in limit less the kernel's
// static shared memory (barriers) and a margin.
constexpr size_t kBgSmemBudget = 227 * 1024 - 2048;

int bg_allow_smem(size_t bytes) {
  static std::mutex mu;
  static size_t granted[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return RWKVB_ECUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (granted[dev] < bytes) {
    const cudaError_t e = cudaFuncSetAttribute(bgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return cuda_status(e);
    granted[dev] = bytes;
  }
  return RWKVB_OK;
}
}  // namespace

// Padded sessions and digit rows (MMA N) for nb sessions.
int bg_padded_sessions(int nb) { return (nb + 15) & ~15; }
int bg_digit_rows(int nb) {
  const int bp = bg_padded_sessions(nb);
  return (3 * bp + 1 + 15) & ~15;
}

// A matrix usable by the batched GEMM: SG8, rows and cols multiples of 128,
// group 64 or 128, code payload 16-byte aligned (TMA).
bool bg_matrix_ok(const rwkvb_packed& w) {
  if (w.kind != RWKVB_KIND_SG8 || !w.data) return false;
  if (w.rows <= 0 || w.cols <= 0 || w.rows % 128 || w.cols % 128) return false;
  if (w.group_size != 64 && w.group_size != 128) return false;
  const PackedView v = make_view(w);
  if (reinterpret_cast<uintptr_t>(v.payload) % 16 || reinterpret_cast<uintptr_t>(v.meta) % 8) return false;
  const uint64_t need = 8 + (uint64_t)w.rows * w.cols / w.group_size * 8 + (uint64_t)w.rows * w.cols;
  return w.bytes >= need;
}

// Digit-matrix description for bg_setup.
struct BgDigits {
  uint8_t* rows;  // [nrows][k]
  float2* cs;     // [k / group][bp]
  int k;
};

struct BgJob {
  const rwkvb_packed* w;
  int digits;  // index into the BgDigits array
  float* out;  // partial sums [pieces][nb][rows]
};

// Fill a launch description for `njobs` matrices over `ndig` digit matrices.
// Returns the grid size in *grid and the maximum number of pieces of a tile
// (the first dimension of every job's partial buffer) in *pieces.
int bg_setup(BgArgs* a, const BgJob* jobs, int njobs, const BgDigits* dg, int ndig, int nb, int sms, int* grid,
             int* pieces, size_t* smem, int* err_word) {
  if (njobs <= 0 || njobs > kBgMaxMats || ndig <= 0 || ndig > kBgMaxMats || nb <= 0 || nb > kBgMaxSessions)
    return RWKVB_EARG;
  std::memset(a, 0, sizeof(*a));
  a->nb = nb;
  a->bp = bg_padded_sessions(nb);
  a->nrows = bg_digit_rows(nb);
  for (int d = 0; d < ndig; ++d) {
    const uint64_t dims[2] = {(uint64_t)dg[d].k, (uint64_t)a->nrows};
    const uint64_t strides[1] = {(uint64_t)dg[d].k};
    const uint32_t box[2] = {128, (uint32_t)a->nrows};
    const int st = encode_u8_map(&a->bmap[d], 2, dg[d].rows, dims, strides, box, true);
    if (st != RWKVB_OK) return st;
    a->cs[d] = reinterpret_cast<const float*>(dg[d].cs);
  }
  int total = 0;
  for (int j = 0; j < njobs; ++j) {
    const rwkvb_packed& w = *jobs[j].w;
    if (!bg_matrix_ok(w) || jobs[j].digits < 0 || jobs[j].digits >= ndig || dg[jobs[j].digits].k != w.cols)
      return RWKVB_EARG;
    const PackedView v = make_view(w);
    BgMat& M = a->mat[j];
    M.pairs = reinterpret_cast<const float2*>(v.meta);
    M.out = jobs[j].out;
    M.rows = w.rows;
    M.k = w.cols;
    M.lg = w.group_size == 64 ? 6 : 7;
    M.digits = jobs[j].digits;
    M.tiles = w.rows / 128;
    M.stage0 = total;
    total += M.tiles * (w.cols / 128);
    const uint64_t dims[2] = {(uint64_t)w.cols, (uint64_t)w.rows};
    const uint64_t strides[1] = {(uint64_t)w.cols};
    const uint32_t box[2] = {128, 128};
    const int st = encode_u8_map(&a->amap[j], 2, v.payload, dims, strides, box, true);
    if (st != RWKVB_OK) return st;
  }
  a->nmat = njobs;
  a->total = total;
  const int n = std::min(sms, total);
  if ((long long)total * n >= (1ll << 31)) return RWKVB_EUNSUPPORTED;  // the kernel splits stages in 32-bit arithmetic
  const size_t stage_bytes = (size_t)kBgTileBytes + (size_t)a->nrows * 128;
  a->stages = (int)std::min<size_t>(kBgMaxStages, (kBgSmemBudget - 1024) / stage_bytes);
  if (a->stages < 2) return RWKVB_EUNSUPPORTED;
  a->idesc = idesc_u8u8_s32(128, a->nrows);
  a->err = err_word;
  int pmax = 1;
  for (int j = 0; j < njobs; ++j) {
    const BgMat& M = a->mat[j];
    const int G = M.k / 128;
    for (int t = 0; t < M.tiles; ++t) {
      const long long f = M.stage0 + (long long)t * G;
      pmax = std::max(pmax, bg_cta_of(f + G - 1, total, n) - bg_cta_of(f, total, n) + 1);
    }
  }
  *grid = n;
  *pieces = pmax;
  *smem = (size_t)a->stages * stage_bytes + 1024;
  return RWKVB_OK;
}

// Pieces per tile of a single-matrix launch (tiles x G stages over min(sms, total) CTAs).
int bg_pieces_single(int tiles, int G, int sms) {
  const int total = tiles * G, n = std::min(sms, total);
  int pmax = 1;
  for (int t = 0; t < tiles; ++t) {
    const long long f = (long long)t * G;
    pmax = std::max(pmax, bg_cta_of(f + G - 1, total, n) - bg_cta_of(f, total, n) + 1);
  }
  return pmax;
}

// Launch `k`, with programmatic stream serialization when `pdl` is set: the
// kernel may start while the previous kernel of the stream finishes; every
// kernel here begins with griddepcontrol.wait (a no-op without the attribute)
// before it touches data the previous kernel writes or reads.
template <typename... K, typename... A>
int bt_go(bool pdl, void (*k)(K...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...));
}

int bg_launch(const BgArgs& a, int grid, size_t smem, cudaStream_t s, bool pdl = false) {
  int st = bg_allow_smem(smem);
  if (st != RWKVB_OK) return st;
  return bt_go(pdl, bgemm_kernel, dim3(grid), dim3(kBgThreads), smem, s, a);
}

// Constant rows of a digit matrix: zero everything, then the ones row (3 bp).
int bg_digits_init(uint8_t* rows, int k, int nb, cudaStream_t s) {
  const int bp = bg_padded_sessions(nb), nrows = bg_digit_rows(nb);
  cudaError_t e = cudaMemsetAsync(rows, 0, (size_t)nrows * k, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(rows + (size_t)3 * bp * k, 1, (size_t)k, s);
  return cuda_status(e);
}

int bg_digits(uint8_t* rows, float2* cs, const float* x, int ldx, int k, int nb, int group, cudaStream_t s,
              bool pdl = false) {
  const int lfk = group == 64 ? 6 : 7;
  const int warps = nb * (k >> lfk);
  return bt_go(pdl, bg_digits_kernel, dim3((warps + 7) / 8), dim3(256), 0, s, rows, cs, x, ldx, k, nb,
               bg_padded_sessions(nb), lfk);
}

}  // namespace rwkvb

using namespace rwkvb;

namespace rwkvb {
namespace {
// Launch description and workspace of one (weight, batch) pair on one device,
// built on first use and kept: tensor maps, digit rows (constant rows written
// once), per-session constants, partial sums and an error word.
struct BgOpEntry {
  const uint8_t* wdata;
  int rows, cols, nb, dev;
  BgArgs a;
  int grid, pieces;
  size_t smem;
  uint8_t* dig;
  float2* cs;
  float* part;
  int* err;
  uint64_t last_use;
};

constexpr size_t kBgOpCacheMax = 32;
std::mutex g_bgop_mu;
std::vector<BgOpEntry*> g_bgop;
uint64_t g_bgop_clock = 0;

void bgop_free(BgOpEntry* e) {
  if (e->dig) cudaFree(e->dig);
  delete e;
}

int bgop_get(const rwkvb_packed& w, int nb, cudaStream_t s, BgOpEntry** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RWKVB_ECUDA;
  std::lock_guard<std::mutex> lock(g_bgop_mu);
  for (BgOpEntry* e : g_bgop)
    if (e->wdata == w.data && e->rows == w.rows && e->cols == w.cols && e->nb == nb && e->dev == dev) {
      e->last_use = ++g_bgop_clock;
      *out = e;
      return RWKVB_OK;
    }
  BgOpEntry* e = new (std::nothrow) BgOpEntry();
  if (!e) return RWKVB_EALLOC;
  e->wdata = w.data, e->rows = w.rows, e->cols = w.cols, e->nb = nb, e->dev = dev;
  const int K = w.cols, N = w.rows, bp = bg_padded_sessions(nb), nrows = bg_digit_rows(nb);
  const size_t dig_bytes = (size_t)nrows * K;
  const size_t cs_off = (dig_bytes + 255) & ~size_t(255);
  const size_t cs_bytes = sizeof(float2) * (size_t)(K / w.group_size) * bp;
  const size_t err_off = (cs_off + cs_bytes + 255) & ~size_t(255);
  const size_t part_off = err_off + 256;
  // partial sums sized by the pieces per tile of the launch plan
  const int sms = device_sms();
  const int pieces = bg_pieces_single(N / 128, K / 128, sms);
  const size_t part_bytes = sizeof(float) * (size_t)pieces * nb * N;
  if (cudaMalloc((void**)&e->dig, part_off + part_bytes) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return RWKVB_EALLOC;
  }
  e->cs = reinterpret_cast<float2*>(e->dig + cs_off);
  e->err = reinterpret_cast<int*>(e->dig + err_off);
  e->part = reinterpret_cast<float*>(e->dig + part_off);
  BgDigits dg{e->dig, e->cs, K};
  BgJob job{&w, 0, e->part};
  int st = bg_setup(&e->a, &job, 1, &dg, 1, nb, sms, &e->grid, &e->pieces, &e->smem, e->err);
  if (st == RWKVB_OK && e->pieces != pieces) st = RWKVB_EUNSUPPORTED;
  if (st == RWKVB_OK) st = bg_digits_init(e->dig, K, nb, s);
  if (st == RWKVB_OK) st = cuda_status(cudaMemsetAsync(e->err, 0, sizeof(int), s));
  if (st != RWKVB_OK) {
    bgop_free(e);
    return st;
  }
  if (g_bgop.size() >= kBgOpCacheMax) {  // evict the least recently used entry
    size_t victim = 0;
    for (size_t i = 1; i < g_bgop.size(); ++i)
      if (g_bgop[i]->last_use < g_bgop[victim]->last_use) victim = i;
    cudaStreamSynchronize(s);
    bgop_free(g_bgop[victim]);
    g_bgop.erase(g_bgop.begin() + (long)victim);
  }
  e->last_use = ++g_bgop_clock;
  g_bgop.push_back(e);
  *out = e;
  return RWKVB_OK;
}
}  // namespace
}  // namespace rwkvb

extern "C" int rwkvb_gemm_sg8_f32(float* y, const rwkvb_packed* w, const float* x, int32_t batch, int32_t* err_word,
                                  void* stream) {
  if (!y || !w || !x || batch <= 0 || batch > kBgMaxSessions) return RWKVB_EARG;
  if (!bg_matrix_ok(*w)) return w->kind == RWKVB_KIND_SG8 ? RWKVB_EUNSUPPORTED : RWKVB_EARG;
  if (reinterpret_cast<uintptr_t>(x) % 16) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  BgOpEntry* e = nullptr;
  int st = bgop_get(*w, batch, s, &e);
  if (st != RWKVB_OK) return st;
  const int K = w->cols, N = w->rows;
  BgArgs a = e->a;
  if (err_word) a.err = err_word;
  st = bg_digits(e->dig, e->cs, x, K, K, batch, (int)w->group_size, s);
  if (st == RWKVB_OK) st = bg_launch(a, e->grid, e->smem, s);
  if (st == RWKVB_OK) {
    bg_reduce_kernel<<<(batch * N + 255) / 256, 256, 0, s>>>(y, e->part, batch, N, 0, K / 128, a.total, e->grid);
    st = cuda_status(cudaGetLastError());
  }
  return st;
}

// ==========================================================================
// Batched decode engine: nb <= 64 independent sessions of one packed RWKV-7
// model advance one token per step together.  Every big projection is a
// tcgen05 batched GEMM (bgemm.cuh); LayerNorms, token shift, digit rows, the
// LoRA-style adapters, WKV7 and the argmax are small kernels around them.  One
// step is captured as a CUDA graph and replayed.
// Per layer (packed_block_forward.py:76-166, rwkv7_linear.py:125-435):
//   in      x (+ folded FFN value pieces); ln1; six token-shift mixes; digit
//           rows of the r/k/v inputs; fp32 w/a/g/v adapter inputs
//   rkv     GEMM r, k, v
//   adp1    first adapter stages x @ W1 (split over input rows) -> partials
//   adpr    reduce the partials, tanh (w) / sigmoid (g)
//   adp2    second adapter stages (mid @ W2)
//   wkv     per (head, session): kk-normalize, decay, WKV7, GroupNorm, bonus, gate
//   ydig    digit rows of the gated output
//   o       GEMM output projection
//   ffn     x + attention; ln2; mix; digit rows
//   key     GEMM ffn key
//   hdig    relu^2 and digit rows of the FFN hidden vector
//   value   GEMM ffn value (folded into the next layer's input)
// then ln_out, the head GEMM and a first-maximum argmax per session.
// ==========================================================================
namespace rwkvb {

constexpr int kBtThreads = 256;
constexpr int kBtAdpCols = 32;  // first-stage adapter columns per CTA
constexpr int kBtAdpKc = 128;   // first-stage input rows per CTA

struct BtPieces {
  int stage0, G, total, ncta;
  const int* np;  // device: pieces of each 128-row tile (precomputed at plan time)
};

// Pieces of output row n's tile: one cached load (the CTA split of a tile's
// stages is fixed by the launch plan, so it is tabulated once per engine
// instead of two 64-bit divisions per element).
__device__ __forceinline__ int bt_npieces(const BtPieces& p, int n) { return __ldg(p.np + (n >> 7)); }

// Sum of the pieces of element (b, n) of a GEMM output [pieces][nb][rows], in
// piece order; the loads are independent and issued together.
__device__ __forceinline__ float bt_fold(const float* part, const BtPieces& p, int nb, int rows, int b, int n) {
  const int np = bt_npieces(p, n);
  const float* q = part + (size_t)b * rows + n;
  const size_t st = (size_t)nb * rows;
  float v[12];
#pragma unroll
  for (int u = 0; u < 12; ++u) v[u] = u < np ? q[u * st] : 0.f;
  float s = v[0];
#pragma unroll
  for (int u = 1; u < 12; ++u)
    if (u < np) s += v[u];
  for (int u = 12; u < np; ++u) s += q[u * st];
  return s;
}

// bt_fold for the four elements n..n+3 (n % 4 == 0: one 128-row tile, so one
// piece count): 16-byte loads, all issued together.
__device__ __forceinline__ float4 bt_fold4(const float* part, const BtPieces& p, int nb, int rows, int b, int n) {
  const int np = bt_npieces(p, n);
  const float* q = part + (size_t)b * rows + n;
  const size_t st = (size_t)nb * rows;
  float4 v[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) v[u] = u < np ? ldcg4(q + u * st) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 s = v[0];
#pragma unroll
  for (int u = 1; u < 8; ++u)
    if (u < np) s = make_float4(s.x + v[u].x, s.y + v[u].y, s.z + v[u].z, s.w + v[u].w);
  for (int u = 8; u < np; ++u) {
    const float4 w = ldcg4(q + u * st);
    s = make_float4(s.x + w.x, s.y + w.y, s.z + w.z, s.w + w.w);
  }
  return s;
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 f4_lerp(float4 z, float4 p, float4 m) {  // z + (p - z) * m
  return make_float4(z.x + (p.x - z.x) * m.x, z.y + (p.y - z.y) * m.y, z.z + (p.z - z.z) * m.z, z.w + (p.w - z.w) * m.w);
}

// LayerNorm of a row held as one float4 per thread (threads t < C / 4): two
// block sums (mean, then centred squares), eps 1e-5.
__device__ __forceinline__ float4 bt_ln4(float4 x, bool act, float4 w, float4 bb, int C, float* red) {
  const float mean = block_sum(act ? x.x + x.y + x.z + x.w : 0.f, red) / (float)C;
  const float4 d = make_float4(x.x - mean, x.y - mean, x.z - mean, x.w - mean);
  const float rstd = rsqrtf(block_sum(act ? d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w : 0.f, red) / (float)C + 1e-5f);
  return make_float4(d.x * rstd * w.x + bb.x, d.y * rstd * w.y + bb.y, d.z * rstd * w.z + bb.z, d.w * rstd * w.w + bb.w);
}

// Digit rows of the block's shared-memory vector src[0..K) for session b.
__device__ __forceinline__ void bt_digits_block(const float* src, int K, int lfk, uint8_t* dig, float2* cs, int b,
                                                int bp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int per = 1 << (lfk - 5);
  for (int g = warp; g < (K >> lfk); g += nw) {
    const float* p = src + ((size_t)g << lfk) + lane * per;
    float v[4] = {p[0], p[1], per == 4 ? p[2] : 0.f, per == 4 ? p[3] : 0.f};
    bg_emit_group(v, per, dig, cs, (size_t)K, ((size_t)g << lfk) + lane * per, b, bp, g);
  }
}

// Two-pass LayerNorm of buf[0..C) in place (eps 1e-5, F.layer_norm).
__device__ __forceinline__ void bt_layer_norm(float* buf, const float* w, const float* bias, int C, float* red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) s += buf[i];
  const float mean = block_sum(s, red) / (float)C;
  float q = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const float d = buf[i] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(block_sum(q, red) / (float)C + 1e-5f);
  for (int i = threadIdx.x; i < C; i += blockDim.x) buf[i] = (buf[i] - mean) * rstd * w[i] + bias[i];
  __syncthreads();
}

// --------------------------------------------------------------- embed
struct BtEmbedArgs {
  PackedView emb;
  const float *ln0_w, *ln0_b;
  const int* tok;  // [nb]
  float* x;        // [nb][C]
  int* step;       // incremented once per step (by block 0)
  int* err;
  int C, V;
  unsigned long long* epoch;  // tensor-parallel exchange epoch (incremented once per step), or null
};

__global__ void __launch_bounds__(kBtThreads) bt_embed_kernel(BtEmbedArgs a) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  __shared__ float red[32];
  extern __shared__ __align__(16) float bt_sm[];
  const int b = blockIdx.x, C = a.C;
  int tok = a.tok[b];
  if (tok < 0 || tok >= a.V) {
    if (threadIdx.x == 0) atomicOr(a.err, kErrToken);
    tok = 0;
  }
  if (b == 0 && threadIdx.x == 0) {
    *a.step += 1;
    if (a.epoch) *a.epoch += 1;
  }
  for (int i = threadIdx.x; i < C; i += blockDim.x) bt_sm[i] = packed_at(a.emb, tok, i);
  __syncthreads();
  bt_layer_norm(bt_sm, a.ln0_w, a.ln0_b, C, red);
  for (int i = threadIdx.x; i < C; i += blockDim.x) a.x[(size_t)b * C + i] = bt_sm[i];
}

// ------------------------------------------------------- layer / head input
struct BtInArgs {
  float* x;              // [nb][C] residual stream (written when folding)
  const float* xm;       // [nb][C] stream after the previous attention (fold source)
  const float* part;     // previous FFN value pieces, or null (x already complete)
  BtPieces pp;
  const float *ln_w, *ln_b;
  float* state;          // att_x[l] [nb][C], or null for the head input
  const float* mix[6];   // x_r, x_w, x_k, x_v, x_a, x_g
  uint8_t* dig[3];       // r, k, v digit rows (head: dig[0] = ln_out rows)
  float2* cs[3];
  float* xa4;            // [4][nb][C]: w, a, g, v adapter inputs
  int C, nb, bp, lfk;
  const float* add;      // tensor parallel: all-reduced value projection [nb][C] (x = xm + add), or null
};

constexpr int kBtRowThreads = 1024;  // per-session row kernels (one CTA per session)

// One float4 of the row per thread (C / 4 <= kBtRowThreads): the LayerNorm
// weights are fetched before the dependency wait, every load of the input is
// issued in one round, and the mixes are fetched while the LayerNorm sums run.
__global__ void __launch_bounds__(kBtRowThreads) bt_in_kernel(BtInArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) float bt_sm[];
  const int b = blockIdx.x, C = a.C, t = threadIdx.x, i = 4 * t;
  const bool act = i < C;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w4 = z4, b4 = z4, m4[6];
#pragma unroll
  for (int j = 0; j < 6; ++j) m4[j] = z4;
  if (act) {
    w4 = ldg4(a.ln_w + i);
    b4 = ldg4(a.ln_b + i);
  }
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  float* xl = bt_sm;       // ln output
  float* mixed = xl + C;   // r, k, v inputs [3][C]
  float4 x4 = z4, p4 = z4;
  if (act) {
    const size_t o = (size_t)b * C + i;
    if (a.state) p4 = ldcg4(a.state + o);
    if (a.part) {
      x4 = f4_add(ldcg4(a.xm + o), bt_fold4(a.part, a.pp, a.nb, C, b, i));
      *reinterpret_cast<float4*>(a.x + o) = x4;
    } else if (a.add) {
      x4 = f4_add(ldcg4(a.xm + o), ldcg4(a.add + o));
      *reinterpret_cast<float4*>(a.x + o) = x4;
    } else {
      x4 = ldcg4(a.x + o);
    }
    if (a.state)  // the mixes (weights) land while the LayerNorm sums run
#pragma unroll
      for (int j = 0; j < 6; ++j) m4[j] = ldg4(a.mix[j] + i);
  }
  const float4 y4 = bt_ln4(x4, act, w4, b4, C, red);
  if (!a.state) {  // head input: ln_out only
    if (act) *reinterpret_cast<float4*>(xl + i) = y4;
    __syncthreads();
    bt_digits_block(xl, C, a.lfk, a.dig[0], a.cs[0], b, a.bp);
    return;
  }
  if (act) {
    const size_t o = (size_t)b * C + i;
    *reinterpret_cast<float4*>(a.state + o) = y4;
    *reinterpret_cast<float4*>(mixed + i) = f4_lerp(y4, p4, m4[0]);          // r
    *reinterpret_cast<float4*>(mixed + C + i) = f4_lerp(y4, p4, m4[2]);      // k
    const float4 vv = f4_lerp(y4, p4, m4[3]);
    *reinterpret_cast<float4*>(mixed + 2 * C + i) = vv;                     // v
    float* xw = a.xa4 + o;
    const size_t ps = (size_t)a.nb * C;
    *reinterpret_cast<float4*>(xw) = f4_lerp(y4, p4, m4[1]);                // w
    *reinterpret_cast<float4*>(xw + ps) = f4_lerp(y4, p4, m4[4]);           // a
    *reinterpret_cast<float4*>(xw + 2 * ps) = f4_lerp(y4, p4, m4[5]);       // g
    *reinterpret_cast<float4*>(xw + 3 * ps) = vv;                           // v
  }
  __syncthreads();
  // digit rows of r, k, v: one warp per (input, group)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int G = C >> a.lfk, per = 1 << (a.lfk - 5);
  for (int w = warp; w < 3 * G; w += nw) {
    const int j = w / G, g = w - j * G;
    const float* src = mixed + (size_t)j * C + ((size_t)g << a.lfk) + lane * per;
    float v[4] = {src[0], src[1], per == 4 ? src[2] : 0.f, per == 4 ? src[3] : 0.f};
    bg_emit_group(v, per, a.dig[j], a.cs[j], (size_t)C, ((size_t)g << a.lfk) + lane * per, b, a.bp, g);
  }
}

// ------------------------------------------------ adapter first stages
// out[s][b][off_m + c] = sum_{i in rows of split s} x_m[b][i] W1_m[i][c]
struct BtAdp1Args {
  PackedView w[4];  // w1, a1, g1, v1: [C][R_m] (x @ W convention)
  int R[4], off[4];
  int blk0[5];      // first column block of each adapter; blk0[nm] = blocks
  int nm;
  int fast[4];      // SG8, R % 32 == 0, 16-byte aligned codes, group >= 32: vector tile loads
  const float* xa4; // [4][nb][C]
  float* out;       // [splits][nb][rtot]
  int C, nb, rtot;
};

constexpr int kBtXsStride = 68;  // padded session stride of the staged inputs (bank spread, float4 aligned)

__global__ void __launch_bounds__(kBtThreads) bt_adp1_kernel(BtAdp1Args a) {
  extern __shared__ __align__(16) float bt_sm[];
  float* xs = bt_sm;                          // [kc][68]: inputs of 64 sessions
  float* ws = xs + kBtAdpKc * kBtXsStride;    // [kc][32]: dequantised weights
  const int t = threadIdx.x;
  int m = 0;
  while (m + 1 < a.nm && (int)blockIdx.x >= a.blk0[m + 1]) ++m;
  const PackedView& W = a.w[m];
  const int R = a.R[m];
  const int c0 = ((int)blockIdx.x - a.blk0[m]) * kBtAdpCols;
  const int k0 = blockIdx.y * kBtAdpKc;
  const float* xsrc = a.xa4 + (size_t)m * a.nb * a.C;
  // the weights do not depend on the previous kernel: dequantised before its wait
  if (a.fast[m]) {
    // one thread per (row, 16 codes): the row's 32 codes are contiguous
    for (int idx = t; idx < kBtAdpKc * 2; idx += blockDim.x) {
      const int kk = idx >> 1, hlf = idx & 1;
      const uint64_t e0 = (uint64_t)(k0 + kk) * R + c0 + 16 * hlf;
      const uint4 q = *reinterpret_cast<const uint4*>(W.payload + e0);
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
      const float2* pr = reinterpret_cast<const float2*>(W.meta);
      const uint64_t g0 = e0 >> W.lg, g1 = (e0 + 15) >> W.lg;
      const float2 p0 = __ldg(pr + g0), p1 = __ldg(pr + g1);
      const uint64_t split = (g1 << W.lg) - e0;  // first element of group g1 (<= 16 when g1 != g0)
      float* dst = ws + kk * kBtAdpCols + 16 * hlf;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const float2 pp = (g1 != g0 && (uint64_t)u >= split) ? p1 : p0;
        dst[u] = sg8_dequant((qw[u >> 2] >> (8 * (u & 3))) & 0xffu, pp.x, pp.y);
      }
    }
  } else {
    for (int idx = t; idx < kBtAdpKc * kBtAdpCols; idx += blockDim.x) {
      const int kk = idx / kBtAdpCols, j = idx - kk * kBtAdpCols;
      ws[idx] = c0 + j < R ? packed_at(W, k0 + kk, c0 + j) : 0.f;
    }
  }
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  // inputs x[b][k0 .. k0 + 127] of the 64 session slots: 8 float4 loads per
  // thread, all in flight before the first store; lanes take consecutive
  // sessions, so the transposed stores xs[k][b] hit distinct banks
  {
    constexpr int kPer = kBtAdpKc * 64 / 4 / kBtThreads;
    static_assert(kPer * 4 * kBtThreads == kBtAdpKc * 64, "x slice split");
    float4 v[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int idx = t + r * kBtThreads, b = idx & 63, k4 = idx >> 6;
      v[r] = b < a.nb ? *reinterpret_cast<const float4*>(xsrc + (size_t)b * a.C + k0 + 4 * k4)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int idx = t + r * kBtThreads, b = idx & 63, k4 = idx >> 6;
      xs[(4 * k4 + 0) * kBtXsStride + b] = v[r].x;
      xs[(4 * k4 + 1) * kBtXsStride + b] = v[r].y;
      xs[(4 * k4 + 2) * kBtXsStride + b] = v[r].z;
      xs[(4 * k4 + 3) * kBtXsStride + b] = v[r].w;
    }
  }
  __syncthreads();
  // threads: (k slice, column pair jq, session quad bq); 2^lp quads cover the
  // sessions (16 at 64), and the 16 >> lp slices split the CTA's 128 inputs, so
  // few sessions still keep every thread's FMAs useful
  const int nq = (a.nb + 3) >> 2;
  const int lp = nq > 8 ? 4 : nq > 4 ? 3 : nq > 2 ? 2 : nq > 1 ? 1 : 0;
  const int U = 16 << lp;  // threads per slice
  const int u = t & (U - 1), bq = u & ((1 << lp) - 1), jq = u >> lp;
  const int kn = kBtAdpKc >> (4 - lp), kb = (t >> (4 + lp)) * kn;
  float acc[4][2] = {};
#pragma unroll 4
  for (int kk = kb; kk < kb + kn; ++kk) {
    const float4 xv = *reinterpret_cast<const float4*>(xs + kk * kBtXsStride + 4 * bq);
    const float2 wv = *reinterpret_cast<const float2*>(ws + kk * kBtAdpCols + 2 * jq);
    acc[0][0] = fmaf(xv.x, wv.x, acc[0][0]);
    acc[0][1] = fmaf(xv.x, wv.y, acc[0][1]);
    acc[1][0] = fmaf(xv.y, wv.x, acc[1][0]);
    acc[1][1] = fmaf(xv.y, wv.y, acc[1][1]);
    acc[2][0] = fmaf(xv.z, wv.x, acc[2][0]);
    acc[2][1] = fmaf(xv.z, wv.y, acc[2][1]);
    acc[3][0] = fmaf(xv.w, wv.x, acc[3][0]);
    acc[3][1] = fmaf(xv.w, wv.y, acc[3][1]);
  }
  if (lp == 4) {  // one slice: the thread's sums are final
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int b = 4 * bq + q;
      if (b >= a.nb) continue;
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const int c = c0 + 2 * jq + v;
        if (c < R) a.out[((size_t)blockIdx.y * a.nb + b) * a.rtot + a.off[m] + c] = acc[q][v];
      }
    }
    return;
  }
  // slices' sums added in slice order (the staged inputs are dead: reused)
  __syncthreads();
  float* red = xs;  // [slice][U][8]: thread t's 8 sums at red[8 t]
  *reinterpret_cast<float4*>(red + 8 * t) = make_float4(acc[0][0], acc[0][1], acc[1][0], acc[1][1]);
  *reinterpret_cast<float4*>(red + 8 * t + 4) = make_float4(acc[2][0], acc[2][1], acc[3][0], acc[3][1]);
  __syncthreads();
  const int ks = 16 >> lp;
  for (int o = t; o < 8 * U; o += blockDim.x) {
    const int uu = o >> 3, e = o & 7;
    const int b = 4 * (uu & ((1 << lp) - 1)) + (e >> 1), c = c0 + 2 * (uu >> lp) + (e & 1);
    float v = 0.f;
    for (int q = 0; q < ks; ++q) v += red[(q * U + uu) * 8 + e];
    if (b < a.nb && c < R) a.out[((size_t)blockIdx.y * a.nb + b) * a.rtot + a.off[m] + c] = v;
  }
}

// midT[j][b] = act(sum over splits of out[s][b][j]): tanh for w, sigmoid for g
// (transposed, 64 sessions per row, for the second stages).
__global__ void bt_adpr_kernel(float* midT, const float* part, int splits, int nb, int rtot, int used, int rw,
                               int ra, int rg) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * used) return;
  const int b = i / used, j = i - b * used;
  float s = 0.f;
#pragma unroll 8
  for (int q = 0; q < splits; ++q) s += part[((size_t)q * nb + b) * rtot + j];  // loads in flight together, adds in order
  if (j < rw) s = tanhf(s);
  else if (j >= rw + ra && j < rw + ra + rg) s = sigmoidf_(s);
  midT[(size_t)j * 64 + b] = s;
}

// ------------------------------------------------ adapter second stages
// Each adapter's rows are cut into chunks of at most kBtAdpChunkRows rows (the
// 320-row g2 of 2.9B into four), so every CTA does about the same work; chunk
// k writes out[slot_k][b][c] = sum over its rows r of mid[b][off_m + r] W2_m[r][c]
// (64 columns per CTA).  The first chunk of adapter m writes slot m, later
// chunks slots 4, 5, ...; a reader sums an adapter's slots in row order
// (bt_adp_at), so the result does not depend on scheduling.
constexpr int kBtAdpChunkRows = 96;
constexpr int kBtMaxChunks = 24;

struct BtAdpSlots {
  int n[4];     // chunks of adapter m
  int s[4][8];  // their output slots, in row order
};

struct BtAdpPlan {
  int n = 0, n_l0 = 0;  // chunks of a layer; of layer 0 (no v2: the v chunks come last)
  int m[kBtMaxChunks], r0[kBtMaxChunks], r1[kBtMaxChunks], slot[kBtMaxChunks];
  int slots = 4;        // output slots
  BtAdpSlots q;
};

// Adapter m's second-stage value at (row, ch): its chunk slots summed in order.
__device__ __forceinline__ float bt_adp_at(const float* adp2, const BtAdpSlots& q, int m, int rows, int row, int C,
                                           int ch) {
  float v = adp2[((size_t)q.s[m][0] * rows + row) * C + ch];
  for (int k = 1; k < q.n[m]; ++k) v += adp2[((size_t)q.s[m][k] * rows + row) * C + ch];
  return v;
}

struct BtAdp2Args {
  PackedView w[4];  // w2, a2, g2, v2: [R_m][C]
  int R[4], off[4];
  int fast[4];      // SG8, group >= 64, 16-byte aligned codes: vector tile loads
  int ck_m[kBtMaxChunks], ck_r0[kBtMaxChunks], ck_r1[kBtMaxChunks], ck_slot[kBtMaxChunks];
  const float* midT; // [rtot][64]
  float* out;       // [slots][nb][C]
  int C, nb, rtot;
};

constexpr int kBtAdp2Rc = 128;  // second-stage rows staged per round

__global__ void __launch_bounds__(kBtThreads) bt_adp2_kernel(BtAdp2Args a) {
  extern __shared__ __align__(16) float bt_sm[];
  const int ck = blockIdx.y, m = a.ck_m[ck], c0 = blockIdx.x * 64, t = threadIdx.x;
  const int R0 = a.ck_r0[ck], R1 = a.ck_r1[ck];
  const PackedView& W = a.w[m];
  float* ms = bt_sm;                  // [rc][64 sessions]
  float* ws = ms + kBtAdp2Rc * 64;    // [rc][64 columns]
  // threads: (row slice, column quad cq, session quad bq); 2^lp quads cover the
  // sessions (16 at 64), and the 16 >> lp slices take every (16 >> lp)-th row,
  // so few sessions still keep every thread's FMAs useful
  const int nq = (a.nb + 3) >> 2;
  const int lp = nq > 8 ? 4 : nq > 4 ? 3 : nq > 2 ? 2 : nq > 1 ? 1 : 0;
  const int U = 16 << lp, ks = 16 >> lp;  // threads per slice, slices
  const int u = t & (U - 1), bq = u & ((1 << lp) - 1), cq = u >> lp, sl = t >> (4 + lp);
  float acc[4][4] = {};
  // rows r0 .. r0 + rc of W (64 columns) dequantised into ws
  auto load_w = [&](int r0, int rc) {
    if (a.fast[m]) {
      for (int idx = t; idx < rc * 4; idx += blockDim.x) {
        const int r = idx >> 2, p = idx & 3;
        const uint64_t e0 = (uint64_t)(r0 + r) * a.C + c0 + 16 * p;
        const uint4 q = *reinterpret_cast<const uint4*>(W.payload + e0);
        const float2 pp = __ldg(reinterpret_cast<const float2*>(W.meta) + (e0 >> W.lg));
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        float* dst = ws + r * 64 + 16 * p;
#pragma unroll
        for (int u = 0; u < 16; ++u) dst[u] = sg8_dequant((qw[u >> 2] >> (8 * (u & 3))) & 0xffu, pp.x, pp.y);
      }
    } else {
      for (int idx = t; idx < rc * 64; idx += blockDim.x) {
        const int r = idx >> 6, j = idx & 63;
        ws[idx] = packed_at(W, r0 + r, c0 + j);
      }
    }
  };
  // the first chunk's weights do not depend on the previous kernel: before its wait
  load_w(R0, min(kBtAdp2Rc, R1 - R0));
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  for (int r0 = R0; r0 < R1; r0 += kBtAdp2Rc) {
    const int rc = min(kBtAdp2Rc, R1 - r0);
    if (r0 != R0) {
      __syncthreads();  // the previous chunk's ms / ws are no longer read
      load_w(r0, rc);
    }
    {
      // rows r0 .. r0 + rc of mid (64 sessions each): up to 8 float4 per thread, loads issued together
      const float4* src = reinterpret_cast<const float4*>(a.midT + (size_t)(a.off[m] + r0) * 64);
      float4 v[kBtAdp2Rc * 16 / kBtThreads];
#pragma unroll
      for (int q = 0; q < kBtAdp2Rc * 16 / kBtThreads; ++q) {
        const int idx = t + q * kBtThreads;
        if (idx < rc * 16) v[q] = src[idx];
      }
#pragma unroll
      for (int q = 0; q < kBtAdp2Rc * 16 / kBtThreads; ++q) {
        const int idx = t + q * kBtThreads;
        if (idx < rc * 16) reinterpret_cast<float4*>(ms)[idx] = v[q];
      }
    }
    __syncthreads();
    for (int r = sl; r < rc; r += ks) {
      const float4 mv = *reinterpret_cast<const float4*>(ms + r * 64 + 4 * bq);
      const float4 wv = *reinterpret_cast<const float4*>(ws + r * 64 + 4 * cq);
      const float mm[4] = {mv.x, mv.y, mv.z, mv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(mm[u], ww[v], acc[u][v]);
    }
  }
  if (lp == 4) {  // one slice: the thread's sums are final
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int b = 4 * bq + q;
      if (b >= a.nb) continue;
      *reinterpret_cast<float4*>(a.out + ((size_t)a.ck_slot[ck] * a.nb + b) * a.C + c0 + 4 * cq) =
          make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
    }
    return;
  }
  // slices' sums added in slice order (the staged mid rows are dead: reused)
  __syncthreads();
  float* red = ms;  // [slice][U][16]: thread t's 16 sums at red[16 t]
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<float4*>(red + 16 * t + 4 * q) = make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
  __syncthreads();
  for (int o = t; o < 4 * U; o += blockDim.x) {  // one float4 (session, column quad) per item
    const int uu = o >> 2, q = o & 3;
    const int b = 4 * (uu & ((1 << lp) - 1)) + q;
    float4 v = *reinterpret_cast<const float4*>(red + uu * 16 + 4 * q);
    for (int z = 1; z < ks; ++z) v = f4_add(v, *reinterpret_cast<const float4*>(red + (z * U + uu) * 16 + 4 * q));
    if (b < a.nb)
      *reinterpret_cast<float4*>(a.out + ((size_t)a.ck_slot[ck] * a.nb + b) * a.C + c0 + 4 * (uu >> lp)) = v;
  }
}

// ------------------------------------------------------------------ wkv
struct BtWkvArgs {
  const float* part[3];  // r, k, v GEMM pieces [pieces][nb][C]
  BtPieces pp[3];
  const float* adp2;     // [slots][nb][C]: w, a, g, v second-stage chunks (pre-activation)
  BtAdpSlots q;
  float* wkv;            // this layer's state [nb][H][64][64]
  float* vfirst;         // [nb][C]
  float* att_y;          // [nb][C]
  const float *w0, *a0, *v0, *k_k, *k_a, *r_k, *lnx_w, *lnx_b;
  int C, H, nb, layer0;
};

constexpr int kBtWkvSess = 4;  // sessions per CTA (64 threads each: thread = state row = channel)

// Named barrier 1 + j over the 64 threads of session slot j (ids as immediates).
__device__ __forceinline__ void bt_bar64(int j) {
  switch (j) {
    case 0: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
    default: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
  }
}

// Sum over the 64 threads of session slot j (two warps).
__device__ __forceinline__ float bt_sum64(float v, float* red, int j) {
  const int lane = threadIdx.x & 31, wg = (threadIdx.x >> 5) & 1;
  v = warp_sum(v);
  if (lane == 0) red[j * 2 + wg] = v;
  bt_bar64(j);
  const float r = red[j * 2] + red[j * 2 + 1];
  bt_bar64(j);
  return r;
}

// Sum over the 64 channel threads (warps 0 and 1) of a 256-thread CTA; every
// thread of the CTA must call it (it contains __syncthreads).
__device__ __forceinline__ float bt_csum64(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0 && w < 2) red[w] = v;
  __syncthreads();
  const float r = red[0] + red[1];
  __syncthreads();
  return r;
}

// Sum over the 16 lanes (a half-warp) that hold one state row.
__device__ __forceinline__ float bt_sum16(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  return v;
}

// Inputs of channel ch of one (session b, head): what threads 0..63 need
// before the state update (loaded one pair ahead, see bt_wkv_kernel).
struct BtWkvChan {
  float wv, av, gv, vg, vf, r, k, v;
};

__device__ __forceinline__ BtWkvChan bt_wkv_chan(const BtWkvArgs& a, int b, int ch) {
  BtWkvChan c;
  const int C = a.C;
  c.wv = bt_adp_at(a.adp2, a.q, 0, a.nb, b, C, ch);
  c.av = bt_adp_at(a.adp2, a.q, 1, a.nb, b, C, ch);
  c.gv = bt_adp_at(a.adp2, a.q, 2, a.nb, b, C, ch);
  c.vg = a.layer0 ? 0.f : bt_adp_at(a.adp2, a.q, 3, a.nb, b, C, ch);
  c.vf = a.layer0 ? 0.f : a.vfirst[(size_t)b * C + ch];
  c.r = bt_fold(a.part[0], a.pp[0], a.nb, C, b, ch);
  c.k = bt_fold(a.part[1], a.pp[1], a.nb, C, b, ch);
  c.v = bt_fold(a.part[2], a.pp[2], a.nb, C, b, ch);
  return c;
}

constexpr int kBtWkvCtasPerSm = 4;

// Sums of (x, y) over the 64 channel threads (warps 0 and 1) only: named
// barrier 1 over 64 threads, so the other warps are not held.
__device__ __forceinline__ float2 bt_chan_sum2(float x, float y, float2* red2) {
  x = warp_sum(x);
  y = warp_sum(y);
  if ((threadIdx.x & 31) == 0) red2[threadIdx.x >> 5] = make_float2(x, y);
  asm volatile("bar.sync 1, 64;" ::: "memory");
  const float2 r = make_float2(red2[0].x + red2[1].x, red2[0].y + red2[1].y);
  asm volatile("bar.sync 1, 64;" ::: "memory");
  return r;
}

// The same over warps 2 and 3 (the GroupNorm threads): named barrier 2.
__device__ __forceinline__ float2 bt_gn_sum2(float x, float y, float2* red2) {
  x = warp_sum(x);
  y = warp_sum(y);
  if ((threadIdx.x & 31) == 0) red2[(threadIdx.x >> 5) - 2] = make_float2(x, y);
  asm volatile("bar.sync 2, 64;" ::: "memory");
  const float2 r = make_float2(red2[0].x + red2[1].x, red2[0].y + red2[1].y);
  asm volatile("bar.sync 2, 64;" ::: "memory");
  return r;
}

// Persistent over (head, session) pairs taken head-major (q = h * nb + b) in a
// contiguous block per CTA, 256 threads per CTA, kBtWkvCtasPerSm CTAs per SM.
//   - the next pair's state (16 KB) is copied into the other shared-memory
//     stage with cp.async while this pair is computed, and threads 0..63 load
//     its channel inputs into registers: ~128 KB of state reads per SM in flight;
//   - the head's eight per-channel vectors are loaded when the head changes;
//   - thread t works on float4 f = t + 256 u (u < 4) of the state: rows
//     (t >> 4) + 16 u, columns 4 (t & 15) .. + 3; a row's dot products are
//     summed over its 16 lanes; the new state is stored straight to global
//     memory (512 contiguous bytes per warp instruction);
//   - channel sums (k norm; GroupNorm mean with the bonus; variance) run on the
//     64 channel threads under a 64-thread barrier; two CTA barriers per pair.
__global__ void __launch_bounds__(kBtThreads, kBtWkvCtasPerSm) bt_wkv_kernel(BtWkvArgs a) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  extern __shared__ __align__(16) float4 bt_stage[];  // [2][1024]
  __shared__ float2 red2[2], gred2[2];
  __shared__ __align__(16) float vd[64], vkk[64], vka[64], vk[64], vr[64], vv[64], sy[64];
  // GroupNorm inputs of the last updated pair (its bonus term and gate), double-buffered by pair parity
  __shared__ float gbon[2][64], gv[2][64], ggate[2][64];
  const int t = threadIdx.x, i = t & 63;
  const bool chan = t < 64, gnw = t >= 64 && t < 128;
  const int npairs = a.nb * a.H;  // <= 64 * 64: the products below fit 32 bits
  const int q0 = (int)((unsigned)blockIdx.x * (unsigned)npairs / gridDim.x);
  const int q1 = (int)((unsigned)(blockIdx.x + 1) * (unsigned)npairs / gridDim.x);
  if (q0 >= q1) return;
  // pair q = (head q / nb, session q % nb); its state is block (b, h) of
  // [nb][H][64][64].  (b, h) are advanced pair by pair: no division by the
  // runtime session count in the loop
  auto state_of = [&](int b, int h) -> float4* {
    return reinterpret_cast<float4*>(a.wkv + ((size_t)b * a.H + h) * 4096);
  };
  auto advance = [&](int& b, int& h) {
    if (++b == a.nb) {
      b = 0;
      ++h;
    }
  };
  // GroupNorm over a head (eps 64e-5), bonus, gate of pair (b, h), by warps
  // 2-3 while warps 0-1 prepare the next pair's channel vectors
  auto group_norm = [&](int b, int h, int par) {
    const int ch = h * 64 + i;
    const float y = sy[i];
    const float2 mb = bt_gn_sum2(y, gbon[par][i], gred2);
    const float mean = mb.x / 64.f;
    const float dv = y - mean;
    const float var = bt_gn_sum2(dv * dv, 0.f, gred2).x / 64.f;
    float o = dv * rsqrtf(var + 64e-5f) * a.lnx_w[ch] + a.lnx_b[ch];
    o = o + mb.y * gv[par][i];
    a.att_y[(size_t)b * a.C + ch] = o * ggate[par][i];
  };
  int b = q0 % a.nb, h = q0 / a.nb;  // pair q
  int pb = b, ph = h;                 // pair q - 1
  {
    const float4* src = state_of(b, h);
#pragma unroll
    for (int u = 0; u < 4; ++u) cp_async16(&bt_stage[t + 256 * u], &src[t + 256 * u]);
    cp_async_commit();
  }
  BtWkvChan cur{};
  if (chan) cur = bt_wkv_chan(a, b, h * 64 + i);
  int vh = -1;  // head whose vectors are in registers
  float kkw = 0.f, a0v = 0.f, v0v = 0.f, w0v = 0.f, kav = 0.f, rkv = 0.f;
  for (int q = q0, it = 0; q < q1; ++q, ++it) {
    const int st = it & 1, nx = q + 1, par = it & 1;
    const int ch = h * 64 + i;
    int bn = b, hn = h;  // pair nx
    advance(bn, hn);
    if (nx < q1) {
      const float4* src = state_of(bn, hn);
#pragma unroll
      for (int u = 0; u < 4; ++u) cp_async16(&bt_stage[(st ^ 1) * 1024 + t + 256 * u], &src[t + 256 * u]);
    }
    cp_async_commit();  // an empty group when there is no next pair
    if (chan) {
      BtWkvChan nxt{};
      if (nx < q1) nxt = bt_wkv_chan(a, bn, hn * 64 + i);
      if (h != vh) {
        vh = h;
        kkw = a.k_k[ch], a0v = a.a0[ch], w0v = a.w0[ch], kav = a.k_a[ch], rkv = a.r_k[ch];
        v0v = a.layer0 ? 0.f : a.v0[ch];
      }
      float v = cur.v;
      const float kkv = cur.k * kkw;
      const float aa = sigmoidf_(a0v + cur.av);
      if (a.layer0) a.vfirst[(size_t)b * a.C + ch] = v;
      else v = v + (cur.vf - v) * sigmoidf_(v0v + cur.vg);
      const float nrm = sqrtf(bt_chan_sum2(kkv * kkv, 0.f, red2).x);
      const float kk = kkv / fmaxf(nrm, 1e-12f);
      const float kn = cur.k * (1.0f + (aa - 1.0f) * kav);
      vd[i] = expf(-0.606531f * sigmoidf_(w0v + cur.wv));
      vkk[i] = -kk;
      vka[i] = kk * aa;
      vk[i] = kn;
      vr[i] = cur.r;
      vv[i] = v;
      gbon[par][i] = cur.r * kn * rkv;
      gv[par][i] = v;
      ggate[par][i] = cur.gv;
      cur = nxt;
    } else if (gnw && it > 0) {
      group_norm(pb, ph, par ^ 1);  // the previous pair (its sy is complete)
    }
    cp_async_wait_group<1>();  // this pair's stage (the group before the prefetch just issued)
    __syncthreads();
    // rows:  sa = S (-kk);  S = S diag(d) + sa (kk a)^T + v_row k^T;  y_row = S r
    {
      const int cg = t & 15, row0 = t >> 4;
      const float4 nkk = reinterpret_cast<const float4*>(vkk)[cg];
      const float4 d4 = reinterpret_cast<const float4*>(vd)[cg];
      const float4 a4 = reinterpret_cast<const float4*>(vka)[cg];
      const float4 k4 = reinterpret_cast<const float4*>(vk)[cg];
      const float4 r4 = reinterpret_cast<const float4*>(vr)[cg];
      float4* S = state_of(b, h);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int row = row0 + 16 * u;
        const float4 s4 = bt_stage[st * 1024 + t + 256 * u];
        float sa = s4.x * nkk.x;
        sa = fmaf(s4.y, nkk.y, sa);
        sa = fmaf(s4.z, nkk.z, sa);
        sa = fmaf(s4.w, nkk.w, sa);
        sa = bt_sum16(sa);
        const float vrow = vv[row];
        float4 n;
        n.x = s4.x * d4.x + sa * a4.x + vrow * k4.x;
        n.y = s4.y * d4.y + sa * a4.y + vrow * k4.y;
        n.z = s4.z * d4.z + sa * a4.z + vrow * k4.z;
        n.w = s4.w * d4.w + sa * a4.w + vrow * k4.w;
        float y = n.x * r4.x;
        y = fmaf(n.y, r4.y, y);
        y = fmaf(n.z, r4.z, y);
        y = fmaf(n.w, r4.w, y);
        y = bt_sum16(y);
        S[t + 256 * u] = n;
        if (cg == 0) sy[row] = y;
      }
    }
    __syncthreads();  // sy complete; stage st and the vectors are free again
    pb = b;
    ph = h;
    b = bn;
    h = hn;
  }
  if (gnw) group_norm(pb, ph, (q1 - 1 - q0) & 1);  // the last pair
  cp_async_wait_all();
}

// ------------------------------------------------------------ ffn input
struct BtFfnArgs {
  const float* x;       // [nb][C] layer input
  float* xm;            // [nb][C] x + attention (written)
  const float* part;    // output-projection pieces
  BtPieces pp;
  const float *ln_w, *ln_b, *mix;
  float* state;         // ffn_x[l] [nb][C]
  uint8_t* dig;
  float2* cs;
  int C, nb, bp, lfk;
  const float* add;     // tensor parallel: all-reduced output projection [nb][C], or null (fold `part`)
};

__global__ void __launch_bounds__(kBtRowThreads) bt_ffn_kernel(BtFfnArgs a) {
  __shared__ float red[32];
  extern __shared__ __align__(16) float bt_sm[];
  const int b = blockIdx.x, C = a.C, t = threadIdx.x, i = 4 * t;
  const bool act = i < C;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w4 = z4, b4 = z4, m4 = z4;
  if (act) {  // weights: before the dependency wait
    w4 = ldg4(a.ln_w + i);
    b4 = ldg4(a.ln_b + i);
    m4 = ldg4(a.mix + i);
  }
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  float* xl = bt_sm;
  float4 x4 = z4, p4 = z4;
  if (act) {
    const size_t o = (size_t)b * C + i;
    p4 = ldcg4(a.state + o);
    const float4 att = a.add ? ldcg4(a.add + o) : bt_fold4(a.part, a.pp, a.nb, C, b, i);
    x4 = f4_add(ldcg4(a.x + o), att);
    *reinterpret_cast<float4*>(a.xm + o) = x4;
  }
  const float4 y4 = bt_ln4(x4, act, w4, b4, C, red);
  if (act) {
    *reinterpret_cast<float4*>(a.state + (size_t)b * C + i) = y4;
    *reinterpret_cast<float4*>(xl + i) = f4_lerp(y4, p4, m4);
  }
  __syncthreads();
  bt_digits_block(xl, C, a.lfk, a.dig, a.cs, b, a.bp);
}

// h = relu(key)^2 and its digit rows: one warp per (session, group).
__global__ void __launch_bounds__(kBtThreads) bt_hdig_kernel(uint8_t* dig, float2* cs, const float* part, BtPieces pp,
                                                             int nb, int F, int bp, int lfk) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int G = F >> lfk;
  if (gw >= nb * G) return;
  const int b = gw / G, g = gw - b * G;
  const int per = 1 << (lfk - 5);
  const int n0 = (g << lfk) + lane * per;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (per == 4) {  // one 16-byte load per piece for the lane's four values
    const float4 y = bt_fold4(part, pp, nb, F, b, n0);
    v[0] = y.x > 0.f ? y.x * y.x : 0.f;
    v[1] = y.y > 0.f ? y.y * y.y : 0.f;
    v[2] = y.z > 0.f ? y.z * y.z : 0.f;
    v[3] = y.w > 0.f ? y.w * y.w : 0.f;
  } else {
    for (int u = 0; u < per; ++u) {
      const float y = bt_fold(part, pp, nb, F, b, n0 + u);
      v[u] = y > 0.f ? y * y : 0.f;
    }
  }
  bg_emit_group(v, per, dig, cs, (size_t)F, (size_t)n0, b, bp, g);
}

// ------------------------------------------------------------- argmax
// ============================================================ prefill rows
// Sequence prefill runs the same layer with rows = (session s, position j) of a
// chunk of P positions: row = s * P + j.  Rows are independent everywhere
// except the token shift (prev of (s, j) is the LayerNorm output of (s, j-1), or
// the state for j = 0) and WKV7 (positions in order), handled below.

// LayerNorm of every row: x[row] (+ folded pieces of the previous layer's
// value projection onto xm) -> x[row] and xln[row].
struct BtLnRowsArgs {
  float* x;           // [rows][C]
  const float* xm;    // fold source, or null (x complete)
  const float* part;
  BtPieces pp;
  const float *ln_w, *ln_b;
  float* xln;         // [rows][C]
  int C, rows;
};

__global__ void __launch_bounds__(kBtRowThreads) bt_lnrows_kernel(BtLnRowsArgs a) {
  __shared__ float red[32];
  const int row = blockIdx.x, C = a.C, i = 4 * threadIdx.x;
  const bool act = i < C;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w4 = z4, b4 = z4, x4 = z4;
  if (act) {  // weights: before the dependency wait
    w4 = ldg4(a.ln_w + i);
    b4 = ldg4(a.ln_b + i);
  }
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  if (act) {
    const size_t o = (size_t)row * C + i;
    if (a.part) {
      x4 = f4_add(ldcg4(a.xm + o), bt_fold4(a.part, a.pp, a.rows, C, row, i));
      *reinterpret_cast<float4*>(a.x + o) = x4;
    } else {
      x4 = ldcg4(a.x + o);
    }
  }
  const float4 y4 = bt_ln4(x4, act, w4, b4, C, red);
  if (act) *reinterpret_cast<float4*>(a.xln + (size_t)row * C + i) = y4;
}

// Token-shift mixes of every row.  mode 0 (time mix): six mixes; digit rows of
// r, k, v and fp32 w/a/g/v adapter inputs.  mode 1 (channel mix): the key mix's
// digit rows.  The CTA of row (s, 0) reads the state of session s and then
// stores the LayerNorm output of (s, P-1) as the new state.
struct BtMixRowsArgs {
  const float* xln;    // [rows][C]
  float* state;        // [nb][C]
  const float* mix[6]; // mode 0: x_r, x_w, x_k, x_v, x_a, x_g; mode 1: mix[0] = x_k
  uint8_t* dig[3];
  float2* cs[3];
  float* xa4;          // [4][rows][C] (mode 0)
  int C, rows, P, bp, lfk, mode;
};

__global__ void __launch_bounds__(kBtRowThreads) bt_mixrows_kernel(BtMixRowsArgs a) {
  extern __shared__ __align__(16) float bt_sm[];
  const int row = blockIdx.x, C = a.C, s = row / a.P, j = row - s * a.P, i = 4 * threadIdx.x;
  const bool act = i < C;
  const int nd = a.mode == 0 ? 3 : 1;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 m4[6];
#pragma unroll
  for (int k = 0; k < 6; ++k) m4[k] = z4;
  if (act)  // the mixes (weights): before the dependency wait
#pragma unroll
    for (int k = 0; k < 6; ++k)
      if (k < (a.mode == 0 ? 6 : 1)) m4[k] = ldg4(a.mix[k] + i);
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  float* mixed = bt_sm;  // [3][C]
  if (act) {
    const float4 z = ldcg4(a.xln + (size_t)row * C + i);
    const float4 p = j > 0 ? ldcg4(a.xln + (size_t)(row - 1) * C + i) : ldcg4(a.state + (size_t)s * C + i);
    if (j == 0)  // the chunk's last LayerNorm output becomes the session's state
      *reinterpret_cast<float4*>(a.state + (size_t)s * C + i) = ldcg4(a.xln + (size_t)(row + a.P - 1) * C + i);
    if (a.mode == 0) {
      *reinterpret_cast<float4*>(mixed + i) = f4_lerp(z, p, m4[0]);          // r
      *reinterpret_cast<float4*>(mixed + C + i) = f4_lerp(z, p, m4[2]);      // k
      const float4 vv = f4_lerp(z, p, m4[3]);
      *reinterpret_cast<float4*>(mixed + 2 * C + i) = vv;                   // v
      float* xw = a.xa4 + (size_t)row * C + i;
      const size_t ps = (size_t)a.rows * C;
      *reinterpret_cast<float4*>(xw) = f4_lerp(z, p, m4[1]);                // w
      *reinterpret_cast<float4*>(xw + ps) = f4_lerp(z, p, m4[4]);           // a
      *reinterpret_cast<float4*>(xw + 2 * ps) = f4_lerp(z, p, m4[5]);       // g
      *reinterpret_cast<float4*>(xw + 3 * ps) = vv;                         // v
    } else {
      *reinterpret_cast<float4*>(mixed + i) = f4_lerp(z, p, m4[0]);
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int G = C >> a.lfk, per = 1 << (a.lfk - 5);
  for (int w = warp; w < nd * G; w += nw) {
    const int m = w / G, g = w - m * G;
    const float* src = mixed + (size_t)m * C + ((size_t)g << a.lfk) + lane * per;
    float v[4] = {src[0], src[1], per == 4 ? src[2] : 0.f, per == 4 ? src[3] : 0.f};
    bg_emit_group(v, per, a.dig[m], a.cs[m], (size_t)C, ((size_t)g << a.lfk) + lane * per, row, a.bp, g);
  }
}

// x + attention output for every row, then LayerNorm 2 -> xln2.
struct BtFfnLnArgs {
  const float* x;
  float* xm;
  const float* part;
  BtPieces pp;
  const float *ln_w, *ln_b;
  float* xln;
  int C, rows;
};

__global__ void __launch_bounds__(kBtRowThreads) bt_ffnln_kernel(BtFfnLnArgs a) {
  __shared__ float red[32];
  const int row = blockIdx.x, C = a.C, i = 4 * threadIdx.x;
  const bool act = i < C;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w4 = z4, b4 = z4, x4 = z4;
  if (act) {  // weights: before the dependency wait
    w4 = ldg4(a.ln_w + i);
    b4 = ldg4(a.ln_b + i);
  }
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  if (act) {
    const size_t o = (size_t)row * C + i;
    x4 = f4_add(ldcg4(a.x + o), bt_fold4(a.part, a.pp, a.rows, C, row, i));
    *reinterpret_cast<float4*>(a.xm + o) = x4;
  }
  const float4 y4 = bt_ln4(x4, act, w4, b4, C, red);
  if (act) *reinterpret_cast<float4*>(a.xln + (size_t)row * C + i) = y4;
}

// WKV7 over the P positions of a chunk, in order, state rows in registers:
// CTA = (head, 4 sessions), 64 threads per session (thread = state row = channel).
struct BtWkvRowsArgs {
  const float* part[3];
  BtPieces pp[3];
  const float* adp2;   // [slots][rows][C]
  BtAdpSlots q;
  float* wkv;          // this layer's state [nb][H][64][64]
  float* vfirst;       // [rows][C]
  float* att_y;        // [rows][C]
  const float *w0, *a0, *v0, *k_k, *k_a, *r_k, *lnx_w, *lnx_b;
  int C, H, nb, rows, P, layer0;
};

__global__ void __launch_bounds__(kBtThreads, 2) bt_wkvrows_kernel(BtWkvRowsArgs a) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  __shared__ float red[2 * kBtWkvSess];
  __shared__ __align__(16) float vecs[kBtWkvSess][5][64];
  const int h = blockIdx.x, t = threadIdx.x, js = t >> 6, i = t & 63;
  const int s = blockIdx.y * kBtWkvSess + js;
  if (s >= a.nb) return;  // whole 64-thread group: it owns its named barrier
  const int C = a.C, ch = h * 64 + i;
  float4* Srow = reinterpret_cast<float4*>(a.wkv + ((size_t)s * a.H + h) * 4096 + (size_t)i * 64);
  float4 s4[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) s4[u] = Srow[u];
  const float kkw = a.k_k[ch], a0 = a.a0[ch], ka = a.k_a[ch], w0 = a.w0[ch], rk = a.r_k[ch], lw = a.lnx_w[ch],
              lb = a.lnx_b[ch], v0 = a.layer0 ? 0.f : a.v0[ch];
  float* vd = vecs[js][0];
  float* vkk = vecs[js][1];
  float* vka = vecs[js][2];
  float* vk = vecs[js][3];
  float* vr = vecs[js][4];
  for (int j = 0; j < a.P; ++j) {
    const int row = s * a.P + j;
    const float wv = bt_adp_at(a.adp2, a.q, 0, a.rows, row, C, ch);
    const float av = bt_adp_at(a.adp2, a.q, 1, a.rows, row, C, ch);
    const float gv = bt_adp_at(a.adp2, a.q, 2, a.rows, row, C, ch);
    float vv = 0.f, vf = 0.f;
    if (!a.layer0) {
      vv = bt_adp_at(a.adp2, a.q, 3, a.rows, row, C, ch);
      vf = a.vfirst[(size_t)row * C + ch];
    }
    const float r = bt_fold(a.part[0], a.pp[0], a.rows, C, row, ch);
    const float k = bt_fold(a.part[1], a.pp[1], a.rows, C, row, ch);
    float v = bt_fold(a.part[2], a.pp[2], a.rows, C, row, ch);
    const float kkv = k * kkw;
    const float nrm = sqrtf(bt_sum64(kkv * kkv, red, js));
    const float aa = sigmoidf_(a0 + av);
    const float kk = kkv / fmaxf(nrm, 1e-12f);
    const float kn = k * (1.0f + (aa - 1.0f) * ka);
    if (a.layer0) a.vfirst[(size_t)row * C + ch] = v;
    else v = v + (vf - v) * sigmoidf_(v0 + vv);
    vd[i] = expf(-0.606531f * sigmoidf_(w0 + wv));
    vkk[i] = -kk;
    vka[i] = kk * aa;
    vk[i] = kn;
    vr[i] = r;
    bt_bar64(js);
    float sa = 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float4 n4 = reinterpret_cast<const float4*>(vkk)[u];
      sa = fmaf(s4[u].x, n4.x, sa);
      sa = fmaf(s4[u].y, n4.y, sa);
      sa = fmaf(s4[u].z, n4.z, sa);
      sa = fmaf(s4[u].w, n4.w, sa);
    }
    float y = 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float4 d4 = reinterpret_cast<const float4*>(vd)[u];
      const float4 a4 = reinterpret_cast<const float4*>(vka)[u];
      const float4 k4 = reinterpret_cast<const float4*>(vk)[u];
      const float4 r4 = reinterpret_cast<const float4*>(vr)[u];
      float4 n;
      n.x = s4[u].x * d4.x + sa * a4.x + v * k4.x;
      n.y = s4[u].y * d4.y + sa * a4.y + v * k4.y;
      n.z = s4[u].z * d4.z + sa * a4.z + v * k4.z;
      n.w = s4[u].w * d4.w + sa * a4.w + v * k4.w;
      y = fmaf(n.x, r4.x, y);
      y = fmaf(n.y, r4.y, y);
      y = fmaf(n.z, r4.z, y);
      y = fmaf(n.w, r4.w, y);
      s4[u] = n;
    }
    const float mean = bt_sum64(y, red, js) / 64.f;
    const float dv = y - mean;
    const float var = bt_sum64(dv * dv, red, js) / 64.f;
    const float bonus = bt_sum64(r * kn * rk, red, js);  // also orders this position's reads of vecs
    float o = dv * rsqrtf(var + 64e-5f) * lw + lb;
    o = o + bonus * v;
    a.att_y[(size_t)row * C + ch] = o * gv;
  }
#pragma unroll
  for (int u = 0; u < 16; ++u) Srow[u] = s4[u];
}

// Head input of each session after a prefill chunk: the last position's
// residual stream (with the last value projection folded in), in decode rows.
__global__ void bt_pick_last_kernel(float* xs, const float* xm, const float* part, BtPieces pp, int C, int rows,
                                    int P, int nb) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * C) return;
  const int s = i / C, c = i - s * C, row = s * P + P - 1;
  xs[(size_t)s * C + c] = xm[(size_t)row * C + c] + bt_fold(part, pp, rows, C, row, c);
}

// Per-session first-maximum argmax of the logits; with `loc` set (tensor
// parallel: this rank holds vocabulary [v0, v0 + V)) the session's best
// (value, global index) goes to loc[b] for the cross-rank merge instead.
__global__ void __launch_bounds__(1024) bt_argmax_kernel(float* logits, const float* part, BtPieces pp, int nb,
                                                         int V, int* tok, int* hist, const int* step, int hist_cap,
                                                         int v0, float2* loc) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int b = blockIdx.x;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int n = threadIdx.x; n < V; n += blockDim.x) {
    const float v = bt_fold(part, pp, nb, V, b, n);
    logits[(size_t)b * V + n] = v;
    if (v > best || (v == best && n < besti)) {
      best = v;
      besti = n;
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
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    bv[wid] = best;
    bi[wid] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float cb = -INFINITY;
    int ci = 0x7fffffff;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
      if (bv[w] > cb || (bv[w] == cb && bi[w] < ci)) {
        cb = bv[w];
        ci = bi[w];
      }
    if (ci == 0x7fffffff) ci = 0;  // every logit NaN
    if (loc) {
      loc[b] = make_float2(cb, __int_as_float(ci + v0));
      return;
    }
    tok[b] = ci;
    const int s = *step;
    hist[(size_t)((s % hist_cap + hist_cap) % hist_cap) * nb + b] = ci;
  }
}

// Merge the ranks' per-session bests all[r][b] (ranks hold increasing
// vocabulary ranges): the largest value, the smallest index among equals.
__global__ void bt_argmax_merge_kernel(const float2* all, int ranks, int nb, int* tok, int* hist, const int* step,
                                       int hist_cap) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int r = 0; r < ranks; ++r) {
    const float2 c = all[(size_t)r * nb + b];
    const int ci = __float_as_int(c.y);
    if (c.x > best || (c.x == best && ci < bi)) {
      best = c.x;
      bi = ci;
    }
  }
  if (bi == 0x7fffffff) bi = 0;
  tok[b] = bi;
  const int s = *step;
  hist[(size_t)((s % hist_cap + hist_cap) % hist_cap) * nb + b] = bi;
}

}  // namespace rwkvb

namespace rwkvb {

// ------------------------------------------------ LUT2 batched product
// y[b][n] = sum_k W[n][k] x[b][k] for a TR2\x04 W (2-bit codes, one 4-entry fp16
// codebook per 64 consecutive elements, row-aligned groups) on the CUDA cores:
// LUT2 centroids are not an affine code grid, so the integer tcgen05 product of
// the SG8 path does not apply.  The batched engine's inputs are its digit rows
// (x = c_f (X0 + X1/254 + X2/254^2) per 64-column group, stored X + 127), the
// same rows the SG8 product reads; they are turned back into fp32 here.
// A CTA owns 64 rows and a contiguous range of 64-column chunks (k split `ks`
// ways); per chunk the 64 x 64 weight tile is decoded once into shared memory
// and every thread accumulates a 4-row x 4-session register tile.  Output:
// piece p (= the CTA's k split) of the engine's pieces layout [ks][nb][rows],
// summed in piece order by the readers like the SG8 product's pieces.
constexpr int kL2Rows = 64;
constexpr int kL2Kc = 64;
constexpr int kL2Threads = 256;
constexpr int kL2Stride = 68;  // padded row stride of the shared tiles (float4 aligned)
constexpr int kL2MaxJobs = 3;

struct BtL2Job {
  const uint32_t* codes;  // 2-bit codes, 16 per word, row-major
  const uint2* recs;      // per 64-element group: 4 fp16 centroids
  float* out;             // pieces [ks][nb][rows]
  const uint8_t* dig;     // digit rows [3 bp + 1][K]
  const float* cs;        // [K / 64][2 bp]: c_f, then sum x
  int rows, K, ks, cta0;  // k splits; first CTA of the job
};

struct BtL2Args {
  BtL2Job job[kL2MaxJobs];
  int njobs, nb, bp;
};

__global__ void __launch_bounds__(kL2Threads) bt_l2gemm_kernel(BtL2Args a) {
  pdl_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  pdl_launch_dependents();
  __shared__ __align__(16) float ws[kL2Kc * kL2Stride];  // [k][row]
  __shared__ __align__(16) float xs[kL2Kc * kL2Stride];  // [k][session]
  int j = 0;
  while (j + 1 < a.njobs && (int)blockIdx.x >= a.job[j + 1].cta0) ++j;
  const BtL2Job J = a.job[j];
  const int local = (int)blockIdx.x - J.cta0, tile = local / J.ks, piece = local - tile * J.ks;
  const int nch = J.K / kL2Kc;
  const int ch0 = (int)((long long)nch * piece / J.ks), ch1 = (int)((long long)nch * (piece + 1) / J.ks);
  const int t = threadIdx.x, r0 = tile * kL2Rows;
  const int rq = t & 15, bq = t >> 4;  // rows 4 rq .. +3, sessions 4 bq .. +3
  const int drow = t & 63, dq = t >> 6;  // decode / staging: row or session, 16-column quarter
  const int words = J.K >> 4;
  float acc[4][4] = {};
  for (int ch = ch0; ch < ch1; ++ch) {
    const int k0 = ch * kL2Kc;
    // weights: row drow, columns k0 + 16 dq .. +15 (one code word)
    {
      const int row = r0 + drow;
      const uint32_t w = __ldg(J.codes + (size_t)row * words + (k0 >> 4) + dq);
      const uint2 rec = __ldg(J.recs + (((size_t)row * J.K + k0) >> 6));
      const float2 c01 = __half22float2(*reinterpret_cast<const __half2*>(&rec.x));
      const float2 c23 = __half22float2(*reinterpret_cast<const __half2*>(&rec.y));
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const uint32_t c = (w >> (2 * u)) & 3u;
        const float v = c == 0 ? c01.x : (c == 1 ? c01.y : (c == 2 ? c23.x : c23.y));
        ws[(16 * dq + u) * kL2Stride + drow] = v;
      }
    }
    // inputs: session drow, columns k0 + 16 dq .. +15, from the three digit rows
    {
      const int b = drow;
      float xv[16];
      if (b < a.nb) {
        const uint4 d0 = *reinterpret_cast<const uint4*>(J.dig + (size_t)b * J.K + k0 + 16 * dq);
        const uint4 d1 = *reinterpret_cast<const uint4*>(J.dig + (size_t)(a.bp + b) * J.K + k0 + 16 * dq);
        const uint4 d2 = *reinterpret_cast<const uint4*>(J.dig + (size_t)(2 * a.bp + b) * J.K + k0 + 16 * dq);
        const float cf = J.cs[(size_t)ch * 2 * a.bp + b];
        const uint32_t w0[4] = {d0.x, d0.y, d0.z, d0.w}, w1[4] = {d1.x, d1.y, d1.z, d1.w},
                       w2[4] = {d2.x, d2.y, d2.z, d2.w};
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float x0 = (float)(int)((w0[u >> 2] >> (8 * (u & 3))) & 0xffu) - 127.f;
          const float x1 = (float)(int)((w1[u >> 2] >> (8 * (u & 3))) & 0xffu) - 127.f;
          const float x2 = (float)(int)((w2[u >> 2] >> (8 * (u & 3))) & 0xffu) - 127.f;
          xv[u] = cf * (x0 + (x1 + x2 * kInv254) * kInv254);
        }
      } else {
#pragma unroll
        for (int u = 0; u < 16; ++u) xv[u] = 0.f;
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) xs[(16 * dq + u) * kL2Stride + b] = xv[u];
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kL2Kc; ++k) {
      const float4 wv = *reinterpret_cast<const float4*>(ws + k * kL2Stride + 4 * rq);
      const float4 xv = *reinterpret_cast<const float4*>(xs + k * kL2Stride + 4 * bq);
      const float wr[4] = {wv.x, wv.y, wv.z, wv.w}, xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(wr[i], xr[q], acc[i][q]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int b = 4 * bq + q;
    if (b >= a.nb) continue;
    float* o = J.out + ((size_t)piece * a.nb + b) * J.rows + r0 + 4 * rq;
    *reinterpret_cast<float4*>(o) = make_float4(acc[0][q], acc[1][q], acc[2][q], acc[3][q]);
  }
}

}  // namespace rwkvb

namespace rwkvb {

// --------------------------------------------- tensor-parallel peer exchange
// Every rank owns one exchange buffer (CUDA IPC-mapped into the other ranks'
// processes), identically laid out on every rank:
//   flags [ninst][kBtMaxRanks][kBtXCtas] u32: written by the peers (epoch)
//   data  [2 L][nb][C] f32: this rank's folded partial projection per all-reduce
//   amax  [nb] float2: this rank's per-session (best logit, global index bits)
// An all-reduce (instance i): every CTA folds its chunk of this rank's GEMM
// pieces into data[i], releases flags[i][rank][cta] = epoch in every peer,
// waits (bounded) until every peer released flags[i][peer][cta], and sums the
// chunk over all ranks in rank order -- the same value on every rank.  Peers'
// data are read with plain loads through the IPC mapping (no multicast).
// A slot is rewritten one step later only after every peer has released a later
// instance of that step, i.e. after the peer has finished reading it.
constexpr int kBtMaxRanks = 8;
constexpr int kBtXCtas = 128;
constexpr int kBtXThreads = 256;

struct BtXPeers {
  char* base[kBtMaxRanks];  // exchange buffer of rank r as mapped in this process
};

struct BtXLayout {
  size_t flags = 0, data = 0, amax = 0, bytes = 0;
  int ninst = 0;
};

inline BtXLayout bt_x_layout(int L, int nb, int C) {
  BtXLayout x;
  x.ninst = 2 * L + 1;
  x.flags = 0;
  x.data = ((size_t)x.ninst * kBtMaxRanks * kBtXCtas * 4 + 255) & ~size_t(255);
  x.amax = x.data + (((size_t)2 * L * nb * C * 4 + 255) & ~size_t(255));
  x.bytes = x.amax + (((size_t)nb * 8 + 255) & ~size_t(255));
  return x;
}

__device__ __forceinline__ void bt_fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void bt_st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t bt_ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t* bt_x_flag(char* base, size_t flags_off, int inst, int src, int cta) {
  return reinterpret_cast<uint32_t*>(base + flags_off) + ((size_t)inst * kBtMaxRanks + src) * kBtXCtas + cta;
}

// Wall-time bound of one peer-exchange wait: well above the skew between the
// rank processes' launches of their step graphs (scheduling, host jitter).
constexpr uint64_t kTpWaitLimitNs = 5000000000ull;  // 5 s

// Thread 0: release this CTA's flag of instance `inst` in every peer, then wait
// (bounded by `limit_ns` of wall time) for every peer's flag; false when a wait
// gave up (error word set).  Once an exchange of the step has given up, the
// later ones return at once instead of each waiting out the limit; the error
// word stays set until the host reads and clears it.  The release is one
// system-scope acq_rel fence followed by relaxed flag stores (the PTX release
// pattern): the CTA's data writes, ordered before the fence by the caller's
// __syncthreads, are visible to every peer that observes a flag.
__device__ bool bt_x_handshake(const BtXPeers& P, size_t flags_off, int inst, int cta, int rank, int size, uint32_t ep,
                               uint64_t limit_ns, int* err) {
  if (*reinterpret_cast<volatile int*>(err) & kErrTimeout) return false;
  bt_fence_acq_rel_sys();
  for (int r = 0; r < size; ++r)
    if (r != rank) bt_st_relaxed_sys(bt_x_flag(P.base[r], flags_off, inst, rank, cta), ep);
  uint64_t t0 = 0;  // the wall clock is read only once a flag was not there at the first poll
  for (int r = 0; r < size; ++r) {
    if (r == rank) continue;
    const uint32_t* f = bt_x_flag(P.base[rank], flags_off, inst, r, cta);
    while (bt_ld_acquire_sys(f) != ep) {
      if (t0 == 0) t0 = globaltimer_ns();
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicOr(err, kErrTimeout);
        return false;
      }
      __nanosleep(128);
    }
  }
  return true;
}

struct BtXReduceArgs {
  BtXPeers peers;
  const float* part;  // this rank's GEMM pieces [pieces][nb][C]
  BtPieces pp;
  float* out;         // [nb][C]: the sum over ranks
  const unsigned long long* epoch;
  int* err;
  size_t flags_off, data_off;
  int nb, C, rank, size, inst;
  uint64_t limit_ns;
};

__global__ void __launch_bounds__(kBtXThreads) bt_xreduce_kernel(BtXReduceArgs a) {
  __shared__ int s_ok;
  const int n = a.nb * a.C, c = blockIdx.x;
  const int e0 = (int)((long long)n * c / kBtXCtas), e1 = (int)((long long)n * (c + 1) / kBtXCtas);
  pdl_wait();  // programmatic dependent launch: the GEMM pieces and the step's epoch are visible
  pdl_launch_dependents();
  const uint32_t ep = (uint32_t)*a.epoch;
  float* mine = reinterpret_cast<float*>(a.peers.base[a.rank] + a.data_off) + (size_t)a.inst * n;
  for (int i = e0 + (int)threadIdx.x; i < e1; i += blockDim.x) {
    const int b = i / a.C, col = i - b * a.C;
    mine[i] = bt_fold(a.part, a.pp, a.nb, a.C, b, col);
  }
  __syncthreads();
  if (threadIdx.x == 0)
    s_ok = bt_x_handshake(a.peers, a.flags_off, a.inst, c, a.rank, a.size, ep, a.limit_ns, a.err) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  for (int i = e0 + (int)threadIdx.x; i < e1; i += blockDim.x) {
    float v = 0.f;
    for (int r = 0; r < a.size; ++r)
      v += __ldcg(reinterpret_cast<const float*>(a.peers.base[r] + a.data_off) + (size_t)a.inst * n + i);
    a.out[i] = v;
  }
}

struct BtXArgmaxArgs {
  BtXPeers peers;
  const unsigned long long* epoch;
  int* err;
  int *tok, *hist;
  const int* step;
  size_t flags_off, amax_off;
  int nb, rank, size, inst, hist_cap;
  uint64_t limit_ns;
};

// One CTA: every rank's per-session bests (written to its own amax slot by
// bt_argmax_kernel) merged first-maximum-wins in rank order.
__global__ void __launch_bounds__(kBtXThreads) bt_xargmax_kernel(BtXArgmaxArgs a) {
  __shared__ int s_ok;
  pdl_wait();  // programmatic dependent launch: this rank's bests and the step's epoch are visible
  pdl_launch_dependents();
  const uint32_t ep = (uint32_t)*a.epoch;
  if (threadIdx.x == 0)
    s_ok = bt_x_handshake(a.peers, a.flags_off, a.inst, 0, a.rank, a.size, ep, a.limit_ns, a.err) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const int st = *a.step;
  for (int b = threadIdx.x; b < a.nb; b += blockDim.x) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < a.size; ++r) {
      const float2 c = __ldcg(reinterpret_cast<const float2*>(a.peers.base[r] + a.amax_off) + b);
      const int ci = __float_as_int(c.y);
      if (c.x > best || (c.x == best && ci < bi)) {
        best = c.x;
        bi = ci;
      }
    }
    if (bi == 0x7fffffff) bi = 0;
    a.tok[b] = bi;
    a.hist[(size_t)((st % a.hist_cap + a.hist_cap) % a.hist_cap) * a.nb + b] = bi;
  }
}

}  // namespace rwkvb

// ------------------------------------------------------------ host engine
namespace rwkvb {
namespace {

struct BtLayer {
  PackedView ad1[4], ad2[4];  // w1 a1 g1 v1, w2 a2 g2 v2
  const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  const float* mix[6];
  const float *w0, *a0, *v0, *k_k, *k_a, *r_k, *lnx_w, *lnx_b, *ffn_x_k;
  BgArgs rkv, o, key, value;
  BtL2Args l2rkv, l2o, l2key, l2value;  // LUT2 engines, CUDA-core products (flag bit 2)
  LmArgs lmrkv, lmo, lmkey, lmvalue;     // LUT2 engines, tcgen05 products
  rwkvb_packed big[6];  // att r, k, v, o, ffn key, ffn value (for further launch plans)
};

// Sequence prefill: rows = (session, position) of a chunk of P positions, with
// its own activation buffers, digit rows and GEMM launch plans.
struct BtPrefill {
  int P = 0, rows = 0, bp = 0, nrows = 0;
  void* arena = nullptr;
  float *x = nullptr, *xm = nullptr, *xln = nullptr, *xln2 = nullptr, *xa4 = nullptr, *adp1 = nullptr;
  float *mid = nullptr, *adp2 = nullptr, *vfirst = nullptr, *att_y = nullptr, *xhead = nullptr;
  float *part_r = nullptr, *part_k = nullptr, *part_v = nullptr, *part_o = nullptr, *part_key = nullptr;
  float* part_val = nullptr;
  uint8_t *dig_r = nullptr, *dig_k = nullptr, *dig_v = nullptr, *dig_y = nullptr, *dig_f = nullptr, *dig_h = nullptr;
  float2 *cs_r = nullptr, *cs_k = nullptr, *cs_v = nullptr, *cs_y = nullptr, *cs_f = nullptr, *cs_h = nullptr;
  int *tok = nullptr, *step = nullptr;
  std::vector<BgArgs> rkv, o, key, value;
  int g_rkv = 0, g_o = 0, g_key = 0, g_value = 0;
  size_t smem_bg = 0;
  BtPieces pp_rkv[3], pp_o, pp_key, pp_value;
  int* np_dev = nullptr;  // piece-count tables of the pp_* above
  cudaGraphExec_t exec = nullptr;
};

constexpr size_t kBtAdp1Smem = sizeof(float) * (kBtAdpKc * kBtXsStride + kBtAdpKc * kBtAdpCols);

bool bt_aligned16(const uint8_t* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool bt_fast_adp1(const PackedView& w, int R) {
  return w.kind == RWKVB_KIND_SG8 && w.lg >= 5 && R % 32 == 0 && bt_aligned16(w.payload);
}

bool bt_fast_adp2(const PackedView& w, int C) {
  return w.kind == RWKVB_KIND_SG8 && w.lg >= 6 && C % 64 == 0 && bt_aligned16(w.payload);
}

bool bt_desc_ok(const rwkvb_packed& p, int rows, int cols) {
  return p.data && p.rows == rows && p.cols == cols && p.group_size > 0 &&
         (p.kind == RWKVB_KIND_SG8 || (p.kind >= RWKVB_KIND_LUT2_F32 && p.kind <= RWKVB_KIND_LUT2_IN_RES));
}

}  // namespace
}  // namespace rwkvb

struct rwkvb_batch {
  int dev = 0, sms = 0;
  int nb = 0, bp = 0, nrows = 0, lfk = 7, group = 128;
  int L = 0, C = 0, H = 0, F = 0, V = 0, rw = 0, ra = 0, rg = 0, rv = 0, rtot = 0;
  int adp_splits = 0, hist_cap = 1024;
  bool lut2 = false;     // TR2\x04 projections and head: CUDA-core products (bt_l2gemm_kernel)
  bool l2_cores = false;  // LUT2 products on CUDA cores instead of tcgen05 (flag bit 2)
  rwkvb::BtL2Args l2head;
  rwkvb::LmArgs lmhead;
  int l2g_rkv = 0, l2g_o = 0, l2g_key = 0, l2g_value = 0, l2g_head = 0;
  int lmg_rkv = 0, lmg_o = 0, lmg_key = 0, lmg_value = 0, lmg_head = 0;
  size_t smem_lm = 0;
  bool pdl = true;       // programmatic dependent launch between the step's kernels
  rwkvb::BtAdpPlan adp;  // adapter second-stage chunks
  std::vector<rwkvb::BtLayer> layers;
  rwkvb::PackedView emb;
  const float *ln0_w = nullptr, *ln0_b = nullptr, *lnout_w = nullptr, *lnout_b = nullptr;
  rwkvb::BgArgs head;
  int g_rkv = 0, g_o = 0, g_key = 0, g_value = 0, g_head = 0;
  size_t smem_bg = 0;
  rwkvb::BtPieces pp_rkv[3], pp_o, pp_key, pp_value, pp_head;
  int* np_dev = nullptr;  // piece-count tables of the pp_* above
  void* arena = nullptr;
  float *att_x = nullptr, *wkv = nullptr, *ffn_x = nullptr, *x = nullptr, *xm = nullptr, *xa4 = nullptr;
  float *adp1 = nullptr, *mid = nullptr, *adp2 = nullptr, *vfirst = nullptr, *att_y = nullptr, *logits = nullptr;
  float *part_r = nullptr, *part_k = nullptr, *part_v = nullptr, *part_o = nullptr, *part_key = nullptr;
  float *part_val = nullptr, *part_head = nullptr;
  uint8_t *dig_r = nullptr, *dig_k = nullptr, *dig_v = nullptr, *dig_y = nullptr, *dig_f = nullptr;
  uint8_t *dig_h = nullptr, *dig_o = nullptr;
  float2 *cs_r = nullptr, *cs_k = nullptr, *cs_v = nullptr, *cs_y = nullptr, *cs_f = nullptr, *cs_h = nullptr;
  float2* cs_o = nullptr;
  int *tok = nullptr, *hist = nullptr, *step = nullptr, *err = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool use_graph = true;
  int launches = 0;
  rwkvb::BtPrefill* pf = nullptr;
  // tensor parallel: this rank holds attention channels [., . + Ca) (H = Ca / 64
  // heads), F FFN rows and vocabulary [V0, V0 + V) of Vfull; partial output and
  // value projections are all-reduced (collective kind 0), per-session argmax
  // bests all-gathered (kind 1) through the host's collective callback
  int Ca = 0, Vfull = 0, V0 = 0, tp_rank = 0, tp_size = 1;
  rwkvb_collective_fn collective = nullptr;
  void* collective_user = nullptr;
  float *ored = nullptr, *vred = nullptr;
  float2 *amax_loc = nullptr, *amax_all = nullptr;
  // peer-memory exchange instead of the collective callback (tp->peer set)
  bool xp = false;
  rwkvb::BtXPeers xpeers{};
  rwkvb::BtXLayout xl;
  unsigned long long* epoch = nullptr;
  uint64_t tp_wait_ns = 0;  // wall-time bound of one exchange wait
};

namespace rwkvb {
namespace {

// Chunks of the adapter second stages: adapter m (w, a, g, v; v last so that
// layer 0 uses a prefix) in ceil(R_m / kBtAdpChunkRows) near-equal row ranges.
bool bt_adp_plan(const int (&R)[4], BtAdpPlan& P) {
  P = BtAdpPlan();
  int extra = 0;
  for (int m = 0; m < 4; ++m) {
    const int n = (R[m] + kBtAdpChunkRows - 1) / kBtAdpChunkRows;
    if (n < 1 || n > 8 || P.n + n > kBtMaxChunks) return false;
    P.q.n[m] = n;
    for (int k = 0; k < n; ++k) {
      const int c = P.n++;
      P.m[c] = m;
      P.r0[c] = (int)((long long)R[m] * k / n);
      P.r1[c] = (int)((long long)R[m] * (k + 1) / n);
      P.slot[c] = k == 0 ? m : 4 + extra++;
      P.q.s[m][k] = P.slot[c];
    }
    if (m == 2) P.n_l0 = P.n;
  }
  P.slots = 4 + extra;
  return true;
}

// Fill the chunk fields of an adapter second-stage launch; returns the chunk count.
int bt_adp2_chunks(const BtAdpPlan& P, bool layer0, BtAdp2Args& a) {
  const int n = layer0 ? P.n_l0 : P.n;
  for (int c = 0; c < n; ++c) {
    a.ck_m[c] = P.m[c];
    a.ck_r0[c] = P.r0[c];
    a.ck_r1[c] = P.r1[c];
    a.ck_slot[c] = P.slot[c];
  }
  return n;
}

BtPieces bt_pieces(const BgArgs& a, int job, int grid) {
  BtPieces p;
  p.stage0 = a.mat[job].stage0;
  p.G = a.mat[job].k / 128;
  p.total = a.total;
  p.ncta = grid;
  p.np = nullptr;
  return p;
}

// LUT2 batched product (bt_l2gemm_kernel): TR2\x04 row-major, 64-element groups.
bool bt_l2_ok(const rwkvb_packed& w) {
  if (w.kind != RWKVB_KIND_LUT2_F16 || w.group_size != 64 || !w.data) return false;
  if (w.rows <= 0 || w.cols <= 0 || w.rows % kL2Rows || w.cols % kL2Kc) return false;
  const PackedView v = make_view(w);
  const uint64_t n = (uint64_t)w.rows * w.cols, need = 8 + n / 64 * 8 + n / 4;
  return w.bytes >= need && (reinterpret_cast<uintptr_t>(v.payload) & 3u) == 0 &&
         (reinterpret_cast<uintptr_t>(v.meta) & 7u) == 0;
}

// Launch plan of one LUT2 product launch over `njobs` matrices; the k split
// gives about two CTAs per SM and at most `pmax` pieces.
int bt_l2_setup(BtL2Args* a, const rwkvb_packed* const* w, float* const* out, const uint8_t* const* dig,
                const float2* const* cs, int njobs, int nb, int sms, int pmax, int* grid, int* ks_out) {
  if (njobs < 1 || njobs > kL2MaxJobs || nb < 1 || nb > kBgMaxSessions) return RWKVB_EARG;
  std::memset(a, 0, sizeof(*a));
  a->njobs = njobs, a->nb = nb, a->bp = bg_padded_sessions(nb);
  int tiles = 0, nch = 1 << 30;
  for (int j = 0; j < njobs; ++j) {
    if (!bt_l2_ok(*w[j])) return RWKVB_EUNSUPPORTED;
    tiles += w[j]->rows / kL2Rows;
    nch = std::min(nch, w[j]->cols / kL2Kc);
  }
  const int ks = std::max(1, std::min({(2 * sms + tiles - 1) / tiles, nch, pmax}));
  int cta = 0;
  for (int j = 0; j < njobs; ++j) {
    const PackedView v = make_view(*w[j]);
    BtL2Job& J = a->job[j];
    J.codes = reinterpret_cast<const uint32_t*>(v.payload);
    J.recs = reinterpret_cast<const uint2*>(v.meta);
    J.out = out[j];
    J.dig = dig[j];
    J.cs = reinterpret_cast<const float*>(cs[j]);
    J.rows = w[j]->rows, J.K = w[j]->cols, J.ks = ks, J.cta0 = cta;
    cta += (w[j]->rows / kL2Rows) * ks;
  }
  *grid = cta;
  *ks_out = ks;
  return RWKVB_OK;
}

// Pieces of a LUT2 product: every row's tile has `ks` pieces in k-split order.
BtPieces bt_l2_pieces(int ks) {
  BtPieces p;
  p.stage0 = 0, p.G = ks, p.total = 1 << 20, p.ncta = 1 << 20;
  p.np = nullptr;
  return p;
}

// tcgen05 LUT2 product (l2mma_kernel) launch plan over `njobs` matrices whose
// digit rows / group scales are dig[j] / cs[j]; the grid is the SM count
// unless that would give a tile more than `pcap` pieces.
struct LmJob {
  const rwkvb_packed* w;
  float* out;
  const uint8_t* dig;
  const float2* cs;
};

int lm_pmax(const LmArgs& a, int n) {
  int pmax = 1;
  for (int j = 0; j < a.nmat; ++j) {
    const LmMat& M = a.mat[j];
    const int G = M.k / 64;
    for (int t = 0; t < M.tiles; ++t) {
      const long long f = M.stage0 + (long long)t * G;
      pmax = std::max(pmax, bg_cta_of(f + G - 1, a.total, n) - bg_cta_of(f, a.total, n) + 1);
    }
  }
  return pmax;
}

int lm_setup(LmArgs* a, const LmJob* jobs, int njobs, int nb, int sms, int pcap, int* grid, size_t* smem,
             int* err_word) {
  if (njobs < 1 || njobs > kLmMaxMats || nb < 1 || nb > kBgMaxSessions || pcap < 1) return RWKVB_EARG;
  std::memset(a, 0, sizeof(*a));
  a->nb = nb;
  a->bp = bg_padded_sessions(nb);
  const int nrows = bg_digit_rows(nb);
  int total = 0;
  for (int j = 0; j < njobs; ++j) {
    const rwkvb_packed& w = *jobs[j].w;
    if (!bt_l2_ok(w) || w.rows % 128 || w.cols % 128) return RWKVB_EUNSUPPORTED;
    const PackedView v = make_view(w);
    // TMA bases: 16-byte aligned codes and records (payloads are placed 16-byte
    // aligned and an even group count keeps the records so)
    if ((reinterpret_cast<uintptr_t>(v.payload) | reinterpret_cast<uintptr_t>(v.meta)) & 15u)
      return RWKVB_EUNSUPPORTED;
    LmMat& M = a->mat[j];
    M.out = jobs[j].out;
    M.cs = reinterpret_cast<const float*>(jobs[j].cs);
    M.rows = w.rows;
    M.k = w.cols;
    M.tiles = w.rows / 128;
    M.stage0 = total;
    total += M.tiles * (w.cols / 64);
    const uint64_t cdims[2] = {(uint64_t)w.cols / 4, (uint64_t)w.rows}, cstr[1] = {(uint64_t)w.cols / 4};
    const uint64_t rdims[2] = {(uint64_t)w.cols / 8, (uint64_t)w.rows}, rstr[1] = {(uint64_t)w.cols / 8};
    const uint64_t ddims[2] = {(uint64_t)w.cols, (uint64_t)nrows}, dstr[1] = {(uint64_t)w.cols};
    const uint32_t box16[2] = {16, 128}, dbox[2] = {64, (uint32_t)(3 * a->bp)};
    int st = encode_u8_map(&a->cmap[j], 2, v.payload, cdims, cstr, box16, false);
    if (st == RWKVB_OK) st = encode_u8_map(&a->rmap[j], 2, v.meta, rdims, rstr, box16, false);
    if (st == RWKVB_OK) st = encode_u8_map(&a->dmap[j], 2, jobs[j].dig, ddims, dstr, dbox, false);
    if (st != RWKVB_OK) return st;
  }
  a->nmat = njobs;
  a->total = total;
  // operand slot: A tile | B tile (3 bp rows); raw slot: codes | records |
  // digit rows | scales
  a->op_bytes = (kLmATile + 384 * a->bp + 1023) & ~1023;
  a->r_dig = 4096;
  a->r_cs = a->r_dig + 192 * a->bp;
  a->raw_bytes = (a->r_cs + 4 * a->bp + 127) & ~127;
  a->tx_bytes = (uint32_t)(2048 + 2048 + 192 * a->bp + 4 * a->bp);
  const size_t room = kBgSmemBudget - 1024 - (size_t)kLmOps * a->op_bytes;
  a->rstages = (int)std::min<size_t>(kLmMaxRaw, room / (size_t)a->raw_bytes);
  if (a->rstages < 2) return RWKVB_EUNSUPPORTED;
  a->idesc = idesc_f16f16_f32(128, 3 * a->bp);
  a->err = err_word;
  int n = std::min(sms, total);
  if ((long long)total * n >= (1ll << 31)) return RWKVB_EUNSUPPORTED;  // the kernel splits stages in 32-bit arithmetic
  while (n > 1 && lm_pmax(*a, n) > pcap) --n;
  *grid = n;
  *smem = (size_t)kLmOps * a->op_bytes + (size_t)a->rstages * a->raw_bytes + 1024;
  return RWKVB_OK;
}

BtPieces lm_pieces(const LmArgs& a, int j, int grid) {
  BtPieces p;
  p.stage0 = a.mat[j].stage0, p.G = a.mat[j].k / 64, p.total = a.total, p.ncta = grid;
  p.np = nullptr;
  return p;
}

// Tabulate the per-tile piece counts of each (pieces, output rows) job into
// one device buffer (*dev, owned by the caller) and point the jobs at it.
int bt_np_upload(const std::vector<std::pair<BtPieces*, int>>& jobs, int** dev) {
  std::vector<int> host;
  std::vector<size_t> off;
  for (const auto& j : jobs) {
    off.push_back(host.size());
    const BtPieces& p = *j.first;
    const int tiles = (j.second + 127) / 128;
    for (int t = 0; t < tiles; ++t) {
      const long long f = p.stage0 + (long long)t * p.G;
      host.push_back(bg_cta_of(f + p.G - 1, p.total, p.ncta) - bg_cta_of(f, p.total, p.ncta) + 1);
    }
  }
  if (cudaMalloc((void**)dev, sizeof(int) * std::max<size_t>(host.size(), 1)) != cudaSuccess) {
    cudaGetLastError();
    *dev = nullptr;
    return RWKVB_EALLOC;
  }
  const int st = cuda_status(cudaMemcpy(*dev, host.data(), sizeof(int) * host.size(), cudaMemcpyHostToDevice));
  if (st != RWKVB_OK) return st;
  for (size_t i = 0; i < jobs.size(); ++i) jobs[i].first->np = *dev + off[i];
  return RWKVB_OK;
}

// One projection launch of the step: the SG8 tcgen05 GEMM, or for LUT2
// engines the tcgen05 LUT2 GEMM (or its CUDA-core counterpart, flag bit 2).
int bt_product(rwkvb_batch* e, const BgArgs& bg, int bg_grid, const BtL2Args& l2, int l2_grid, const LmArgs& lm,
               int lm_grid, cudaStream_t s) {
  if (!e->lut2) return bg_launch(bg, bg_grid, e->smem_bg, s, e->pdl);
  if (e->l2_cores) return bt_go(e->pdl, bt_l2gemm_kernel, dim3(l2_grid), dim3(kL2Threads), 0, s, l2);
  return bt_go(e->pdl, l2mma_kernel, dim3(lm_grid), dim3(kLmThreads), e->smem_lm, s, lm);
}

// ln_out of x (+ folded value pieces onto xm when `part` is set), the head
// GEMM and the per-session first-maximum argmax (-> e->tok, e->logits).
int bt_record_head(rwkvb_batch* e, float* x, const float* xm, const float* part, const BtPieces& pp, cudaStream_t s,
                   const float* add = nullptr) {
  const int C = e->C, nb = e->nb;
  BtInArgs a;
  std::memset(&a, 0, sizeof(a));
  a.x = x;
  a.xm = xm;
  a.part = part;
  a.pp = pp;
  a.add = add;
  a.ln_w = e->lnout_w;
  a.ln_b = e->lnout_b;
  a.state = nullptr;
  a.dig[0] = e->dig_o;
  a.cs[0] = e->cs_o;
  a.C = C, a.nb = nb, a.bp = e->bp, a.lfk = e->lfk;
  bt_go(e->pdl, bt_in_kernel, dim3(nb), dim3(kBtRowThreads), sizeof(float) * 5 * C, s, a);
  int st = cuda_status(cudaGetLastError());
  if (st == RWKVB_OK)
    st = !e->lut2     ? bg_launch(e->head, e->g_head, e->smem_bg, s, e->pdl)
         : e->l2_cores ? bt_go(e->pdl, bt_l2gemm_kernel, dim3(e->l2g_head), dim3(kL2Threads), 0, s, e->l2head)
                       : bt_go(e->pdl, l2mma_kernel, dim3(e->lmg_head), dim3(kLmThreads), e->smem_lm, s, e->lmhead);
  if (st != RWKVB_OK) return st;
  const bool tp = e->tp_size > 1;
  float2* loc = !tp ? nullptr
                    : (e->xp ? reinterpret_cast<float2*>(e->xpeers.base[e->tp_rank] + e->xl.amax) : e->amax_loc);
  bt_go(e->pdl, bt_argmax_kernel, dim3(nb), dim3(1024), 0, s, e->logits, e->part_head, e->pp_head, nb, e->V, e->tok, e->hist, e->step,
                                       e->hist_cap, e->V0, loc);
  st = cuda_status(cudaGetLastError());
  if (st != RWKVB_OK || !tp) return st;
  if (e->xp) {
    BtXArgmaxArgs x;
    std::memset(&x, 0, sizeof(x));
    x.peers = e->xpeers;
    x.epoch = e->epoch;
    x.err = e->err;
    x.tok = e->tok, x.hist = e->hist, x.step = e->step;
    x.flags_off = e->xl.flags, x.amax_off = e->xl.amax;
    x.nb = nb, x.rank = e->tp_rank, x.size = e->tp_size, x.inst = e->xl.ninst - 1, x.hist_cap = e->hist_cap;
    x.limit_ns = e->tp_wait_ns;
    return bt_go(e->pdl, bt_xargmax_kernel, dim3(1), dim3(kBtXThreads), 0, s, x);
  }
  e->collective(1, e->amax_loc, e->amax_all, (int64_t)sizeof(float2) * nb, s, e->collective_user);
  bt_go(e->pdl, bt_argmax_merge_kernel, dim3((nb + 127) / 128), dim3(128), 0, s, e->amax_all, e->tp_size, nb, e->tok, e->hist, e->step,
                                                          e->hist_cap);
  return cuda_status(cudaGetLastError());
}

// Tensor parallel: fold a projection's pieces into `red` [nb][C] and all-reduce
// it: in one peer-exchange kernel (instance `inst` of the step), or by the fold
// kernel and the host's collective callback.
int bt_reduce(rwkvb_batch* e, float* red, const float* part, const BtPieces& pp, cudaStream_t s, int inst) {
  if (e->xp) {
    BtXReduceArgs x;
    std::memset(&x, 0, sizeof(x));
    x.peers = e->xpeers;
    x.part = part;
    x.pp = pp;
    x.out = red;
    x.epoch = e->epoch;
    x.err = e->err;
    x.flags_off = e->xl.flags, x.data_off = e->xl.data;
    x.nb = e->nb, x.C = e->C, x.rank = e->tp_rank, x.size = e->tp_size, x.inst = inst;
    x.limit_ns = e->tp_wait_ns;
    return bt_go(e->pdl, bt_xreduce_kernel, dim3(kBtXCtas), dim3(kBtXThreads), 0, s, x);
  }
  const int n = e->nb * e->C;
  bg_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(red, part, e->nb, e->C, pp.stage0, pp.G, pp.total, pp.ncta);
  const int st = cuda_status(cudaGetLastError());
  if (st != RWKVB_OK) return st;
  e->collective(0, red, red, (int64_t)sizeof(float) * n, s, e->collective_user);
  return RWKVB_OK;
}

// Launch one token step of every session (tokens already in e->tok).
int bt_record_step(rwkvb_batch* e, cudaStream_t s) {
  const int C = e->C, Ca = e->Ca, nb = e->nb;
  const bool tp = e->tp_size > 1;
  int n = 0;
#define BT_CHECK()                                                                           \
  do {                                                                                       \
    const int st_ = cuda_status(cudaGetLastError());                                         \
    if (st_ != RWKVB_OK) {                                                                   \
      if (std::getenv("RWKVB_DEBUG")) std::fprintf(stderr, "rwkvb: batched launch at line %d\n", __LINE__); \
      return st_;                                                                            \
    }                                                                                        \
    ++n;                                                                                     \
  } while (0)
  {
    BtEmbedArgs a{e->emb, e->ln0_w, e->ln0_b, e->tok, e->x, e->step, e->err, C, e->Vfull, e->xp ? e->epoch : nullptr};
    bt_go(e->pdl, bt_embed_kernel, dim3(nb), dim3(kBtThreads), sizeof(float) * C, s, a);
    BT_CHECK();
  }
  for (int l = 0; l < e->L; ++l) {
    const BtLayer& ly = e->layers[l];
    const bool l0 = l == 0;
    {
      BtInArgs a;
      std::memset(&a, 0, sizeof(a));
      a.x = e->x;
      a.xm = e->xm;
      a.part = (l0 || tp) ? nullptr : e->part_val;
      a.add = (!l0 && tp) ? e->vred : nullptr;
      a.pp = e->pp_value;
      a.ln_w = ly.ln1_w;
      a.ln_b = ly.ln1_b;
      a.state = e->att_x + (size_t)l * nb * C;
      for (int j = 0; j < 6; ++j) a.mix[j] = ly.mix[j];
      a.dig[0] = e->dig_r, a.dig[1] = e->dig_k, a.dig[2] = e->dig_v;
      a.cs[0] = e->cs_r, a.cs[1] = e->cs_k, a.cs[2] = e->cs_v;
      a.xa4 = e->xa4;
      a.C = C, a.nb = nb, a.bp = e->bp, a.lfk = e->lfk;
      bt_go(e->pdl, bt_in_kernel, dim3(nb), dim3(kBtRowThreads), sizeof(float) * 5 * C, s, a);
      BT_CHECK();
    }
    if (bt_product(e, ly.rkv, e->g_rkv, ly.l2rkv, e->l2g_rkv, ly.lmrkv, e->lmg_rkv, s) != RWKVB_OK) return RWKVB_ECUDA;
    ++n;
    const int nm = l0 ? 3 : 4;
    {
      BtAdp1Args a;
      std::memset(&a, 0, sizeof(a));
      const int Rm[4] = {e->rw, e->ra, e->rg, e->rv};
      int off = 0, blk = 0;
      for (int m = 0; m < 4; ++m) {
        a.w[m] = ly.ad1[m];
        a.R[m] = Rm[m];
        a.off[m] = off;
        a.blk0[m] = blk;
        off += Rm[m];
        if (m < nm) blk += (Rm[m] + kBtAdpCols - 1) / kBtAdpCols;
      }
      a.blk0[nm] = blk;
      a.nm = nm;
      for (int m = 0; m < nm; ++m) a.fast[m] = bt_fast_adp1(a.w[m], a.R[m]);
      a.xa4 = e->xa4;
      a.out = e->adp1;
      a.C = C, a.nb = nb, a.rtot = e->rtot;
      bt_go(e->pdl, bt_adp1_kernel, dim3(blk, e->adp_splits), dim3(kBtThreads), kBtAdp1Smem, s, a);
      BT_CHECK();
      const int used = l0 ? e->rw + e->ra + e->rg : e->rtot;
      bt_go(e->pdl, bt_adpr_kernel, dim3((nb * used + 255) / 256), dim3(256), 0, s, e->mid, e->adp1, e->adp_splits, nb, e->rtot, used,
                                                              e->rw, e->ra, e->rg);
      BT_CHECK();
    }
    {
      BtAdp2Args a;
      std::memset(&a, 0, sizeof(a));
      const int Rm[4] = {e->rw, e->ra, e->rg, e->rv};
      int off = 0;
      for (int m = 0; m < 4; ++m) {
        a.w[m] = ly.ad2[m];
        a.R[m] = Rm[m];
        a.off[m] = off;
        off += Rm[m];
      }
      for (int m = 0; m < nm; ++m) a.fast[m] = bt_fast_adp2(a.w[m], C);
      const int nck = bt_adp2_chunks(e->adp, l0, a);
      a.midT = e->mid;
      a.out = e->adp2;
      a.C = Ca, a.nb = nb, a.rtot = e->rtot;
      bt_go(e->pdl, bt_adp2_kernel, dim3(Ca / 64, nck), dim3(kBtThreads), sizeof(float) * 2 * kBtAdp2Rc * 64, s, a);
      BT_CHECK();
    }
    {
      BtWkvArgs a;
      std::memset(&a, 0, sizeof(a));
      a.part[0] = e->part_r, a.part[1] = e->part_k, a.part[2] = e->part_v;
      for (int j = 0; j < 3; ++j) a.pp[j] = e->pp_rkv[j];
      a.adp2 = e->adp2;
      a.q = e->adp.q;
      a.wkv = e->wkv + (size_t)l * nb * e->H * 4096;
      a.vfirst = e->vfirst;
      a.att_y = e->att_y;
      a.w0 = ly.w0, a.a0 = ly.a0, a.v0 = ly.v0, a.k_k = ly.k_k, a.k_a = ly.k_a, a.r_k = ly.r_k;
      a.lnx_w = ly.lnx_w, a.lnx_b = ly.lnx_b;
      a.C = Ca, a.H = e->H, a.nb = nb, a.layer0 = l0 ? 1 : 0;
      const int pairs = nb * e->H, grid = std::min(pairs, e->sms * kBtWkvCtasPerSm);
      bt_go(e->pdl, bt_wkv_kernel, dim3(grid), dim3(kBtThreads), 2 * 1024 * sizeof(float4), s, a);
      BT_CHECK();
    }
    if (bg_digits(e->dig_y, e->cs_y, e->att_y, Ca, Ca, nb, e->group, s, e->pdl) != RWKVB_OK) return RWKVB_ECUDA;
    ++n;
    if (bt_product(e, ly.o, e->g_o, ly.l2o, e->l2g_o, ly.lmo, e->lmg_o, s) != RWKVB_OK) return RWKVB_ECUDA;
    ++n;
    if (tp) {
      if (bt_reduce(e, e->ored, e->part_o, e->pp_o, s, 2 * l) != RWKVB_OK) return RWKVB_ECUDA;
      ++n;
    }
    {
      BtFfnArgs a{e->x, e->xm, e->part_o, e->pp_o, ly.ln2_w, ly.ln2_b, ly.ffn_x_k,
                  e->ffn_x + (size_t)l * nb * C, e->dig_f, e->cs_f, C, nb, e->bp, e->lfk, tp ? e->ored : nullptr};
      bt_go(e->pdl, bt_ffn_kernel, dim3(nb), dim3(kBtRowThreads), sizeof(float) * C, s, a);
      BT_CHECK();
    }
    if (bt_product(e, ly.key, e->g_key, ly.l2key, e->l2g_key, ly.lmkey, e->lmg_key, s) != RWKVB_OK) return RWKVB_ECUDA;
    ++n;
    {
      const int warps = nb * (e->F >> e->lfk);
      bt_go(e->pdl, bt_hdig_kernel, dim3((warps + 7) / 8), dim3(kBtThreads), 0, s, e->dig_h, e->cs_h, e->part_key, e->pp_key, nb, e->F,
                                                           e->bp, e->lfk);
      BT_CHECK();
    }
    if (bt_product(e, ly.value, e->g_value, ly.l2value, e->l2g_value, ly.lmvalue, e->lmg_value, s) != RWKVB_OK) return RWKVB_ECUDA;
    ++n;
    if (tp) {
      if (bt_reduce(e, e->vred, e->part_val, e->pp_value, s, 2 * l + 1) != RWKVB_OK) return RWKVB_ECUDA;
      ++n;
    }
  }
  {
    const int st = tp ? bt_record_head(e, e->x, e->xm, nullptr, e->pp_value, s, e->vred)
                      : bt_record_head(e, e->x, e->xm, e->part_val, e->pp_value, s);
    if (st != RWKVB_OK) return st;
    n += tp ? 4 : 3;
  }
#undef BT_CHECK
  e->launches = n;
  return RWKVB_OK;
}

// Capture the step into e->exec (once).  Under tensor parallelism the host
// collective callback is called during the capture, on the capture stream.
int bt_capture_step(rwkvb_batch* e) {
  if (e->exec) return RWKVB_OK;
  cudaStream_t cs = nullptr;
  if (cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking) != cudaSuccess) return RWKVB_ECUDA;
  cudaGraph_t g = nullptr;
  int st = cuda_status(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  if (st == RWKVB_OK) {
    st = bt_record_step(e, cs);
    const cudaError_t ce = cudaStreamEndCapture(cs, &g);
    if (st == RWKVB_OK) st = cuda_status(ce);
  }
  if (st == RWKVB_OK) st = cuda_status(cudaGraphInstantiate(&e->exec, g, 0));
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(cs);
  if (st != RWKVB_OK) {
    cudaGetLastError();
    e->exec = nullptr;
  }
  return st;
}

int bt_run_step(rwkvb_batch* e, cudaStream_t s) {
  if (!e->use_graph) return bt_record_step(e, s);
  const int st = bt_capture_step(e);
  if (st != RWKVB_OK) return st;
  return cuda_status(cudaGraphLaunch(e->exec, s));
}

int bt_check_err(rwkvb_batch* e, cudaStream_t s) {
  int h = 0;
  cudaError_t err = cudaMemcpyAsync(&h, e->err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_status(err);
  if (h) {
    cudaMemsetAsync(e->err, 0, sizeof(int), s);
    cudaStreamSynchronize(s);
    return (h & kErrTimeout) ? RWKVB_ETIMEOUT : RWKVB_EARG;
  }
  return RWKVB_OK;
}

// Build the prefill plan: chunk P = 64 / nb positions (at least 2).
int bt_prefill_setup(rwkvb_batch* e) {
  if (e->pf) return RWKVB_OK;
  if (e->tp_size > 1) return RWKVB_EUNSUPPORTED;  // positions then run as (tensor-parallel) decode steps
  if (e->lut2) return RWKVB_EUNSUPPORTED;          // LUT2 engines: every position as a decode step
  const int P = kBgMaxSessions / e->nb;
  if (P < 2) return RWKVB_EUNSUPPORTED;
  BtPrefill* f = new (std::nothrow) BtPrefill();
  if (!f) return RWKVB_EALLOC;
  const int rows = e->nb * P, C = e->C, F = e->F, V = e->V;
  f->P = P, f->rows = rows, f->bp = bg_padded_sessions(rows), f->nrows = bg_digit_rows(rows);
  const size_t rC = (size_t)rows * C;
  const int Pk = C / 128, Pf = F / 128;
  struct Item {
    void** p;
    size_t bytes;
  };
  const size_t csC = 8 * (size_t)(C / e->group) * f->bp, csF = 8 * (size_t)(F / e->group) * f->bp;
  std::vector<Item> items = {
      {(void**)&f->x, 4 * rC},          {(void**)&f->xm, 4 * rC},
      {(void**)&f->xln, 4 * rC},        {(void**)&f->xln2, 4 * rC},
      {(void**)&f->xa4, 4 * 4 * rC},    {(void**)&f->adp1, 4 * (size_t)e->adp_splits * rows * e->rtot},
      {(void**)&f->mid, 4 * (size_t)64 * e->rtot}, {(void**)&f->adp2, 4 * (size_t)e->adp.slots * rC},
      {(void**)&f->vfirst, 4 * rC},     {(void**)&f->att_y, 4 * rC},
      {(void**)&f->xhead, 4 * (size_t)e->nb * C},
      {(void**)&f->part_r, 4 * (size_t)Pk * rC}, {(void**)&f->part_k, 4 * (size_t)Pk * rC},
      {(void**)&f->part_v, 4 * (size_t)Pk * rC}, {(void**)&f->part_o, 4 * (size_t)Pk * rC},
      {(void**)&f->part_key, 4 * (size_t)Pk * rows * F}, {(void**)&f->part_val, 4 * (size_t)Pf * rC},
      {(void**)&f->dig_r, (size_t)f->nrows * C}, {(void**)&f->dig_k, (size_t)f->nrows * C},
      {(void**)&f->dig_v, (size_t)f->nrows * C}, {(void**)&f->dig_y, (size_t)f->nrows * C},
      {(void**)&f->dig_f, (size_t)f->nrows * C}, {(void**)&f->dig_h, (size_t)f->nrows * F},
      {(void**)&f->cs_r, csC}, {(void**)&f->cs_k, csC}, {(void**)&f->cs_v, csC}, {(void**)&f->cs_y, csC},
      {(void**)&f->cs_f, csC}, {(void**)&f->cs_h, csF},
      {(void**)&f->tok, 4 * (size_t)rows}, {(void**)&f->step, 16},
  };
  (void)V;
  size_t total = 0;
  std::vector<size_t> offs;
  for (const Item& it : items) {
    offs.push_back(total);
    total += (it.bytes + 1023) & ~size_t(1023);
  }
  if (cudaMalloc(&f->arena, total) != cudaSuccess) {
    cudaGetLastError();
    delete f;
    return RWKVB_EALLOC;
  }
  cudaMemset(f->arena, 0, total);
  for (size_t i = 0; i < items.size(); ++i) *items[i].p = (char*)f->arena + offs[i];
  int st = RWKVB_OK;
  uint8_t* digs[] = {f->dig_r, f->dig_k, f->dig_v, f->dig_y, f->dig_f};
  for (uint8_t* d : digs)
    if (st == RWKVB_OK) st = bg_digits_init(d, C, rows, nullptr);
  if (st == RWKVB_OK) st = bg_digits_init(f->dig_h, F, rows, nullptr);
  if (st == RWKVB_OK) st = cuda_status(cudaDeviceSynchronize());
  const BgDigits d_rkv[3] = {{f->dig_r, f->cs_r, C}, {f->dig_k, f->cs_k, C}, {f->dig_v, f->cs_v, C}};
  const BgDigits d_y{f->dig_y, f->cs_y, C}, d_f{f->dig_f, f->cs_f, C}, d_h{f->dig_h, f->cs_h, F};
  int pieces = 0;
  size_t smem = 0;
  for (int l = 0; l < e->L && st == RWKVB_OK; ++l) {
    const BtLayer& ly = e->layers[l];
    BgArgs rkv, o, key, value;
    const BgJob jr[3] = {{&ly.big[0], 0, f->part_r}, {&ly.big[1], 1, f->part_k}, {&ly.big[2], 2, f->part_v}};
    st = bg_setup(&rkv, jr, 3, d_rkv, 3, rows, e->sms, &f->g_rkv, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    f->smem_bg = std::max(f->smem_bg, smem);
    const BgJob jo{&ly.big[3], 0, f->part_o};
    if (st == RWKVB_OK) st = bg_setup(&o, &jo, 1, &d_y, 1, rows, e->sms, &f->g_o, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    const BgJob jk{&ly.big[4], 0, f->part_key};
    if (st == RWKVB_OK) st = bg_setup(&key, &jk, 1, &d_f, 1, rows, e->sms, &f->g_key, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    const BgJob jv{&ly.big[5], 0, f->part_val};
    if (st == RWKVB_OK) st = bg_setup(&value, &jv, 1, &d_h, 1, rows, e->sms, &f->g_value, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pf) st = RWKVB_EUNSUPPORTED;
    if (st == RWKVB_OK && l == 0) {
      for (int j = 0; j < 3; ++j) f->pp_rkv[j] = bt_pieces(rkv, j, f->g_rkv);
      f->pp_o = bt_pieces(o, 0, f->g_o);
      f->pp_key = bt_pieces(key, 0, f->g_key);
      f->pp_value = bt_pieces(value, 0, f->g_value);
    }
    f->rkv.push_back(rkv), f->o.push_back(o), f->key.push_back(key), f->value.push_back(value);
  }
  if (st == RWKVB_OK)
    st = bt_np_upload({{&f->pp_rkv[0], C}, {&f->pp_rkv[1], C}, {&f->pp_rkv[2], C}, {&f->pp_o, C},
                       {&f->pp_key, e->F}, {&f->pp_value, C}},
                      &f->np_dev);
  if (st == RWKVB_OK) st = bg_allow_smem(f->smem_bg);
  if (st == RWKVB_OK) {
    const void* fns[] = {(const void*)bt_mixrows_kernel, (const void*)bt_lnrows_kernel, (const void*)bt_ffnln_kernel};
    const int sm[] = {(int)(sizeof(float) * 5 * C), (int)(sizeof(float) * C), (int)(sizeof(float) * C)};
    for (int i = 0; i < 3 && st == RWKVB_OK; ++i)
      st = cuda_status(cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, sm[i]));
  }
  if (st != RWKVB_OK) {
    cudaFree(f->arena);
    if (f->np_dev) cudaFree(f->np_dev);
    delete f;
    return st;
  }
  e->pf = f;
  return RWKVB_OK;
}

// One prefill chunk of every session (tokens in pf->tok, row order s * P + j).
int bt_record_prefill(rwkvb_batch* e, cudaStream_t s) {
  BtPrefill& f = *e->pf;
  const int C = e->C, rows = f.rows, nb = e->nb;
#define PF_CHECK()                                  \
  do {                                              \
    const int st_ = cuda_status(cudaGetLastError()); \
    if (st_ != RWKVB_OK) return st_;                \
  } while (0)
  {
    BtEmbedArgs a{e->emb, e->ln0_w, e->ln0_b, f.tok, f.x, f.step, e->err, C, e->Vfull, nullptr};
    bt_go(e->pdl, bt_embed_kernel, dim3(rows), dim3(kBtThreads), sizeof(float) * C, s, a);
    PF_CHECK();
  }
  for (int l = 0; l < e->L; ++l) {
    const BtLayer& ly = e->layers[l];
    const bool l0 = l == 0;
    {
      BtLnRowsArgs a{f.x, l0 ? nullptr : f.xm, l0 ? nullptr : f.part_val, f.pp_value, ly.ln1_w, ly.ln1_b, f.xln,
                     C, rows};
      bt_go(e->pdl, bt_lnrows_kernel, dim3(rows), dim3(kBtRowThreads), sizeof(float) * C, s, a);
      PF_CHECK();
    }
    {
      BtMixRowsArgs a;
      std::memset(&a, 0, sizeof(a));
      a.xln = f.xln;
      a.state = e->att_x + (size_t)l * nb * C;
      for (int j = 0; j < 6; ++j) a.mix[j] = ly.mix[j];
      a.dig[0] = f.dig_r, a.dig[1] = f.dig_k, a.dig[2] = f.dig_v;
      a.cs[0] = f.cs_r, a.cs[1] = f.cs_k, a.cs[2] = f.cs_v;
      a.xa4 = f.xa4;
      a.C = C, a.rows = rows, a.P = f.P, a.bp = f.bp, a.lfk = e->lfk, a.mode = 0;
      bt_go(e->pdl, bt_mixrows_kernel, dim3(rows), dim3(kBtRowThreads), sizeof(float) * 5 * C, s, a);
      PF_CHECK();
    }
    if (bg_launch(f.rkv[l], f.g_rkv, f.smem_bg, s, e->pdl) != RWKVB_OK) return RWKVB_ECUDA;
    const int nm = l0 ? 3 : 4;
    {
      BtAdp1Args a;
      std::memset(&a, 0, sizeof(a));
      const int Rm[4] = {e->rw, e->ra, e->rg, e->rv};
      int off = 0, blk = 0;
      for (int m = 0; m < 4; ++m) {
        a.w[m] = ly.ad1[m];
        a.R[m] = Rm[m];
        a.off[m] = off;
        a.blk0[m] = blk;
        off += Rm[m];
        if (m < nm) blk += (Rm[m] + kBtAdpCols - 1) / kBtAdpCols;
      }
      a.blk0[nm] = blk;
      a.nm = nm;
      for (int m = 0; m < nm; ++m) a.fast[m] = bt_fast_adp1(a.w[m], a.R[m]);
      a.xa4 = f.xa4;
      a.out = f.adp1;
      a.C = C, a.nb = rows, a.rtot = e->rtot;
      bt_go(e->pdl, bt_adp1_kernel, dim3(blk, e->adp_splits), dim3(kBtThreads), kBtAdp1Smem, s, a);
      PF_CHECK();
      const int used = l0 ? e->rw + e->ra + e->rg : e->rtot;
      bt_go(e->pdl, bt_adpr_kernel, dim3((rows * used + 255) / 256), dim3(256), 0, s, f.mid, f.adp1, e->adp_splits, rows, e->rtot, used,
                                                                e->rw, e->ra, e->rg);
      PF_CHECK();
    }
    {
      BtAdp2Args a;
      std::memset(&a, 0, sizeof(a));
      const int Rm[4] = {e->rw, e->ra, e->rg, e->rv};
      int off = 0;
      for (int m = 0; m < 4; ++m) {
        a.w[m] = ly.ad2[m];
        a.R[m] = Rm[m];
        a.off[m] = off;
        off += Rm[m];
      }
      for (int m = 0; m < nm; ++m) a.fast[m] = bt_fast_adp2(a.w[m], C);
      const int nck = bt_adp2_chunks(e->adp, l0, a);
      a.midT = f.mid;
      a.out = f.adp2;
      a.C = C, a.nb = rows, a.rtot = e->rtot;
      bt_go(e->pdl, bt_adp2_kernel, dim3(C / 64, nck), dim3(kBtThreads), sizeof(float) * 2 * kBtAdp2Rc * 64, s, a);
      PF_CHECK();
    }
    {
      BtWkvRowsArgs a;
      std::memset(&a, 0, sizeof(a));
      a.part[0] = f.part_r, a.part[1] = f.part_k, a.part[2] = f.part_v;
      for (int j = 0; j < 3; ++j) a.pp[j] = f.pp_rkv[j];
      a.adp2 = f.adp2;
      a.q = e->adp.q;
      a.wkv = e->wkv + (size_t)l * nb * e->H * 4096;
      a.vfirst = f.vfirst;
      a.att_y = f.att_y;
      a.w0 = ly.w0, a.a0 = ly.a0, a.v0 = ly.v0, a.k_k = ly.k_k, a.k_a = ly.k_a, a.r_k = ly.r_k;
      a.lnx_w = ly.lnx_w, a.lnx_b = ly.lnx_b;
      a.C = C, a.H = e->H, a.nb = nb, a.rows = rows, a.P = f.P, a.layer0 = l0 ? 1 : 0;
      bt_go(e->pdl, bt_wkvrows_kernel, dim3(e->H, (nb + kBtWkvSess - 1) / kBtWkvSess), dim3(kBtThreads), 0, s, a);
      PF_CHECK();
    }
    if (bg_digits(f.dig_y, f.cs_y, f.att_y, C, C, rows, e->group, s, e->pdl) != RWKVB_OK) return RWKVB_ECUDA;
    if (bg_launch(f.o[l], f.g_o, f.smem_bg, s, e->pdl) != RWKVB_OK) return RWKVB_ECUDA;
    {
      BtFfnLnArgs a{f.x, f.xm, f.part_o, f.pp_o, ly.ln2_w, ly.ln2_b, f.xln2, C, rows};
      bt_go(e->pdl, bt_ffnln_kernel, dim3(rows), dim3(kBtRowThreads), sizeof(float) * C, s, a);
      PF_CHECK();
    }
    {
      BtMixRowsArgs a;
      std::memset(&a, 0, sizeof(a));
      a.xln = f.xln2;
      a.state = e->ffn_x + (size_t)l * nb * C;
      a.mix[0] = ly.ffn_x_k;
      a.dig[0] = f.dig_f;
      a.cs[0] = f.cs_f;
      a.C = C, a.rows = rows, a.P = f.P, a.bp = f.bp, a.lfk = e->lfk, a.mode = 1;
      bt_go(e->pdl, bt_mixrows_kernel, dim3(rows), dim3(kBtRowThreads), sizeof(float) * 5 * C, s, a);
      PF_CHECK();
    }
    if (bg_launch(f.key[l], f.g_key, f.smem_bg, s, e->pdl) != RWKVB_OK) return RWKVB_ECUDA;
    {
      const int warps = rows * (e->F >> e->lfk);
      bt_go(e->pdl, bt_hdig_kernel, dim3((warps + 7) / 8), dim3(kBtThreads), 0, s, f.dig_h, f.cs_h, f.part_key, f.pp_key, rows, e->F, f.bp,
                                                           e->lfk);
      PF_CHECK();
    }
    if (bg_launch(f.value[l], f.g_value, f.smem_bg, s, e->pdl) != RWKVB_OK) return RWKVB_ECUDA;
  }
  bt_go(e->pdl, bt_pick_last_kernel, dim3((nb * C + 255) / 256), dim3(256), 0, s, f.xhead, f.xm, f.part_val, f.pp_value, C, rows, f.P, nb);
  PF_CHECK();
#undef PF_CHECK
  return RWKVB_OK;
}

int bt_run_prefill_chunk(rwkvb_batch* e, cudaStream_t s) {
  BtPrefill& f = *e->pf;
  if (e->use_graph && !f.exec) {
    cudaStream_t cs = nullptr;
    if (cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking) != cudaSuccess) return RWKVB_ECUDA;
    cudaGraph_t g = nullptr;
    int st = cuda_status(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    if (st == RWKVB_OK) {
      st = bt_record_prefill(e, cs);
      const cudaError_t ce = cudaStreamEndCapture(cs, &g);
      if (st == RWKVB_OK) st = cuda_status(ce);
    }
    if (st == RWKVB_OK) st = cuda_status(cudaGraphInstantiate(&f.exec, g, 0));
    if (g) cudaGraphDestroy(g);
    cudaStreamDestroy(cs);
    if (st != RWKVB_OK) {
      f.exec = nullptr;
      return st;
    }
  }
  if (e->use_graph) return cuda_status(cudaGraphLaunch(f.exec, s));
  return bt_record_prefill(e, s);
}

}  // namespace
}  // namespace rwkvb

extern "C" int rwkvb_batch_prefill(rwkvb_batch* e, const int32_t* tokens, int32_t n, void* stream) {
  if (!e || (!tokens && n > 0) || n < 0) return RWKVB_EARG;
  for (size_t i = 0; i < (size_t)n * e->nb; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->Vfull) return RWKVB_EARG;
  if (n == 0) return RWKVB_OK;
  cudaStream_t s = (cudaStream_t)stream;
  int st = bt_prefill_setup(e);
  const int P = st == RWKVB_OK ? e->pf->P : 1;
  if (st == RWKVB_EUNSUPPORTED) st = RWKVB_OK;  // chunk of one: every position is a decode step
  if (st != RWKVB_OK) return st;
  const int nb = e->nb, full = P > 1 ? n / P : 0;
  std::vector<int32_t> chunk((size_t)nb * (P > 1 ? P : 1));
  for (int c = 0; c < full && st == RWKVB_OK; ++c) {
    for (int b = 0; b < nb; ++b)
      for (int j = 0; j < P; ++j) chunk[(size_t)b * P + j] = tokens[(size_t)b * n + (size_t)c * P + j];
    st = cuda_status(cudaMemcpyAsync(e->pf->tok, chunk.data(), sizeof(int32_t) * nb * P, cudaMemcpyHostToDevice, s));
    if (st == RWKVB_OK) st = bt_run_prefill_chunk(e, s);
    if (st == RWKVB_OK) st = cuda_status(cudaStreamSynchronize(s));  // the host chunk buffer is reused
  }
  const int done = full * P;
  if (st == RWKVB_OK && done == n) {
    BtPrefill& f = *e->pf;
    st = bt_record_head(e, f.xhead, nullptr, nullptr, f.pp_value, s);
  }
  std::vector<int32_t> step(nb);
  for (int pos = done; pos < n && st == RWKVB_OK; ++pos) {
    for (int b = 0; b < nb; ++b) step[b] = tokens[(size_t)b * n + pos];
    st = rwkvb_batch_forward(e, step.data(), s);
    if (st == RWKVB_OK) st = cuda_status(cudaStreamSynchronize(s));
  }
  return st;
}

namespace rwkvb {
namespace {
int bt_create(const rwkvb_model_desc* m, int32_t batch, uint32_t flags, const rwkvb_tp_desc* tp, rwkvb_batch** out) {
  if (!m || !out || !m->layers || batch <= 0 || batch > kBgMaxSessions) return RWKVB_EARG;
  *out = nullptr;
  // V: vocabulary rows of this engine's head (a shard under tensor parallelism); Vfull: embedding rows
  const int L = m->n_layer, C = m->n_embd, N = m->head_size, F = m->ffn, Vfull = m->vocab, V = m->head.rows;
  const int Ca = m->layers[0].att_r.rows;  // attention channels held here
  if (L <= 0 || C <= 0 || F <= 0 || V <= 0 || N != 64 || C % 128 || F % 128 || V % 128 || Ca <= 0 || Ca % 128)
    return RWKVB_EUNSUPPORTED;
  if (C > 4 * kBtRowThreads) return RWKVB_EUNSUPPORTED;  // per-session row kernels: one float4 per thread
  if (!tp && (Ca != C || V != Vfull)) return RWKVB_EARG;
  if (tp && (tp->size < 2 || tp->rank < 0 || tp->rank >= tp->size || (!tp->collective && !tp->peer) ||
             tp->vocab_offset < 0 || tp->vocab_offset + V > Vfull || (tp->peer && tp->size > kBtMaxRanks)))
    return RWKVB_EARG;
  // projections and head all SG8 (tcgen05 products) or all TR2\x04 (CUDA-core products)
  const bool l2 = m->head.kind == RWKVB_KIND_LUT2_F16;
  auto big_ok = [&](const rwkvb_packed& w) { return l2 ? bt_l2_ok(w) : bg_matrix_ok(w); };
  if (l2 && tp) return RWKVB_EUNSUPPORTED;
  if (!bt_desc_ok(m->emb, Vfull, C) || !big_ok(m->head) || m->head.cols != C)
    return (m->head.kind == RWKVB_KIND_SG8 || l2) ? RWKVB_EUNSUPPORTED : RWKVB_EARG;
  if (!m->ln0_w || !m->ln0_b || !m->ln_out_w || !m->ln_out_b) return RWKVB_EARG;
  const rwkvb_layer_desc& l0 = m->layers[0];
  const int rw = l0.w1.cols, ra = l0.a1.cols, rg = l0.g1.cols;
  const int rv = L > 1 ? m->layers[1].v1.cols : 0;
  const uint32_t group = m->head.group_size;
  for (int i = 0; i < L; ++i) {
    const rwkvb_layer_desc& s = m->layers[i];
    const rwkvb_packed* big[] = {&s.att_r, &s.att_k, &s.att_v, &s.att_o, &s.ffn_key, &s.ffn_value};
    for (const rwkvb_packed* p : big)
      if (!big_ok(*p) || p->group_size != group) return RWKVB_EUNSUPPORTED;
    if (s.att_r.rows != Ca || s.att_r.cols != C || s.att_k.rows != Ca || s.att_k.cols != C || s.att_v.rows != Ca ||
        s.att_v.cols != C || s.att_o.rows != C || s.att_o.cols != Ca || s.ffn_key.rows != F ||
        s.ffn_key.cols != C || s.ffn_value.rows != C || s.ffn_value.cols != F)
      return RWKVB_EARG;
    if (!bt_desc_ok(s.w1, C, rw) || !bt_desc_ok(s.w2, rw, Ca) || !bt_desc_ok(s.a1, C, ra) ||
        !bt_desc_ok(s.a2, ra, Ca) || !bt_desc_ok(s.g1, C, rg) || !bt_desc_ok(s.g2, rg, Ca))
      return RWKVB_EARG;
    if (i > 0 && (!bt_desc_ok(s.v1, C, rv) || !bt_desc_ok(s.v2, rv, Ca))) return RWKVB_EARG;
    const float* vecs[] = {s.ln1_w, s.ln1_b, s.ln2_w, s.ln2_b, s.x_r, s.x_w, s.x_k, s.x_v, s.x_a, s.x_g,
                           s.w0, s.a0, s.k_k, s.k_a, s.r_k, s.lnx_w, s.lnx_b, s.ffn_x_k};
    for (const float* p : vecs)
      if (!p) return RWKVB_EARG;
    if (i > 0 && !s.v0) return RWKVB_EARG;
  }
  if (rw <= 0 || ra <= 0 || rg <= 0) return RWKVB_EUNSUPPORTED;

  rwkvb_batch* e = new (std::nothrow) rwkvb_batch();
  if (!e) return RWKVB_EALLOC;
  cudaGetDevice(&e->dev);
  e->sms = device_sms();
  e->use_graph = !(flags & 0x1u);
  e->lut2 = l2;
  e->l2_cores = l2 && (flags & 0x4u);
  // bit 1: no programmatic dependent launch; off under tensor parallelism (collectives between kernels)
  e->pdl = !(flags & 0x2u) && !tp;
  // bits 16..19: exchange wait limit in units of 100 ms (0: the 5 s default)
  e->tp_wait_ns = ((flags >> 16) & 0xFu) ? (uint64_t)((flags >> 16) & 0xFu) * 100000000ull : rwkvb::kTpWaitLimitNs;
  e->nb = batch;
  e->bp = bg_padded_sessions(batch);
  e->nrows = bg_digit_rows(batch);
  e->group = (int)group;
  e->lfk = group == 64 ? 6 : 7;
  e->L = L, e->C = C, e->H = Ca / 64, e->F = F, e->V = V;
  e->Ca = Ca, e->Vfull = Vfull;
  if (tp) {
    e->tp_rank = tp->rank, e->tp_size = tp->size, e->V0 = tp->vocab_offset;
    e->collective = tp->collective, e->collective_user = tp->user;
    if (tp->peer) {
      e->xp = true;
      e->xl = bt_x_layout(L, batch, C);
      for (int r = 0; r < tp->size; ++r) {
        if (!tp->peer[r]) {
          delete e;
          return RWKVB_EARG;
        }
        e->xpeers.base[r] = static_cast<char*>(tp->peer[r]);
      }
    }
  }
  e->rw = rw, e->ra = ra, e->rg = rg, e->rv = rv, e->rtot = rw + ra + rg + rv;
  {
    const int R[4] = {rw, ra, rg, rv};
    if (!bt_adp_plan(R, e->adp)) {
      delete e;
      return RWKVB_EUNSUPPORTED;
    }
  }
  e->adp_splits = C / kBtAdpKc;
  e->emb = make_view(m->emb);
  e->ln0_w = m->ln0_w, e->ln0_b = m->ln0_b, e->lnout_w = m->ln_out_w, e->lnout_b = m->ln_out_b;

  // ---------------------------------------------------------------- arena
  const size_t nbC = (size_t)batch * C;
  const int bp = e->bp, nr = e->nrows;
  // generous piece bounds: a tile never spans more CTAs than its stages
  const int Pk = C / 128, Pf = F / 128;
  struct Item {
    void** p;
    size_t bytes;
  };
  std::vector<Item> items = {
      {(void**)&e->att_x, 4 * (size_t)L * nbC},
      {(void**)&e->wkv, 4 * (size_t)L * batch * e->H * 4096},
      {(void**)&e->ffn_x, 4 * (size_t)L * nbC},
      {(void**)&e->x, 4 * nbC},
      {(void**)&e->xm, 4 * nbC},
      {(void**)&e->xa4, 4 * 4 * nbC},
      {(void**)&e->adp1, 4 * (size_t)e->adp_splits * batch * e->rtot},
      {(void**)&e->mid, 4 * (size_t)64 * e->rtot},
      {(void**)&e->adp2, 4 * (size_t)e->adp.slots * nbC},
      {(void**)&e->vfirst, 4 * nbC},
      {(void**)&e->att_y, 4 * nbC},
      {(void**)&e->logits, 4 * (size_t)batch * V},
      {(void**)&e->part_r, 4 * (size_t)Pk * nbC},
      {(void**)&e->part_k, 4 * (size_t)Pk * nbC},
      {(void**)&e->part_v, 4 * (size_t)Pk * nbC},
      {(void**)&e->part_o, 4 * (size_t)Pk * nbC},
      {(void**)&e->part_key, 4 * (size_t)Pk * batch * F},
      {(void**)&e->part_val, 4 * (size_t)Pf * nbC},
      {(void**)&e->part_head, 4 * (size_t)Pk * batch * V},
      {(void**)&e->dig_r, (size_t)nr * C},
      {(void**)&e->dig_k, (size_t)nr * C},
      {(void**)&e->dig_v, (size_t)nr * C},
      {(void**)&e->dig_y, (size_t)nr * C},
      {(void**)&e->dig_f, (size_t)nr * C},
      {(void**)&e->dig_h, (size_t)nr * F},
      {(void**)&e->dig_o, (size_t)nr * C},
      {(void**)&e->cs_r, 8 * (size_t)(C / group) * bp},
      {(void**)&e->cs_k, 8 * (size_t)(C / group) * bp},
      {(void**)&e->cs_v, 8 * (size_t)(C / group) * bp},
      {(void**)&e->cs_y, 8 * (size_t)(C / group) * bp},
      {(void**)&e->cs_f, 8 * (size_t)(C / group) * bp},
      {(void**)&e->cs_h, 8 * (size_t)(F / group) * bp},
      {(void**)&e->cs_o, 8 * (size_t)(C / group) * bp},
      {(void**)&e->tok, 4 * (size_t)batch},
      {(void**)&e->hist, 4 * (size_t)e->hist_cap * batch},
      {(void**)&e->step, 16},
      {(void**)&e->err, 16},
      {(void**)&e->ored, 4 * nbC},
      {(void**)&e->vred, 4 * nbC},
      {(void**)&e->amax_loc, 8 * (size_t)batch},
      {(void**)&e->amax_all, 8 * (size_t)batch * e->tp_size},
      {(void**)&e->epoch, 16},
  };
  size_t total = 0;
  std::vector<size_t> offs;
  for (const Item& it : items) {
    offs.push_back(total);
    total += (it.bytes + 1023) & ~size_t(1023);
  }
  if (cudaMalloc(&e->arena, total) != cudaSuccess) {
    cudaGetLastError();
    delete e;
    return RWKVB_EALLOC;
  }
  cudaMemset(e->arena, 0, total);
  for (size_t i = 0; i < items.size(); ++i) *items[i].p = (char*)e->arena + offs[i];
  {
    // constant rows (the ones row at 3 * bp * K) laid out for each GEMM's own K
    uint8_t* digs[] = {e->dig_r, e->dig_k, e->dig_v, e->dig_f, e->dig_o};
    int st = RWKVB_OK;
    for (uint8_t* d : digs)
      if (st == RWKVB_OK) st = bg_digits_init(d, C, batch, nullptr);
    if (st == RWKVB_OK) st = bg_digits_init(e->dig_y, Ca, batch, nullptr);
    if (st == RWKVB_OK) st = bg_digits_init(e->dig_h, F, batch, nullptr);
    if (st == RWKVB_OK) st = cuda_status(cudaMemset(e->step, 0xff, sizeof(int)));
    if (st == RWKVB_OK) st = cuda_status(cudaDeviceSynchronize());
    if (st != RWKVB_OK) {
      cudaFree(e->arena);
      delete e;
      return st;
    }
  }

  // ------------------------------------------------------- GEMM launch plans
  const BgDigits d_rkv[3] = {{e->dig_r, e->cs_r, C}, {e->dig_k, e->cs_k, C}, {e->dig_v, e->cs_v, C}};
  const BgDigits d_y{e->dig_y, e->cs_y, Ca}, d_f{e->dig_f, e->cs_f, C}, d_h{e->dig_h, e->cs_h, F},
      d_o{e->dig_o, e->cs_o, C};
  int pieces = 0, st = RWKVB_OK;
  size_t smem = 0;
  for (int i = 0; i < L && st == RWKVB_OK; ++i) {
    const rwkvb_layer_desc& s = m->layers[i];
    BtLayer ly;
    std::memset(&ly, 0, sizeof(ly));
    const rwkvb_packed* a1[4] = {&s.w1, &s.a1, &s.g1, &s.v1};
    const rwkvb_packed* a2[4] = {&s.w2, &s.a2, &s.g2, &s.v2};
    for (int j = 0; j < 4; ++j) {
      if (j == 3 && i == 0) continue;
      ly.ad1[j] = make_view(*a1[j]);
      ly.ad2[j] = make_view(*a2[j]);
    }
    ly.ln1_w = s.ln1_w, ly.ln1_b = s.ln1_b, ly.ln2_w = s.ln2_w, ly.ln2_b = s.ln2_b;
    ly.mix[0] = s.x_r, ly.mix[1] = s.x_w, ly.mix[2] = s.x_k, ly.mix[3] = s.x_v, ly.mix[4] = s.x_a, ly.mix[5] = s.x_g;
    ly.w0 = s.w0, ly.a0 = s.a0, ly.v0 = s.v0, ly.k_k = s.k_k, ly.k_a = s.k_a, ly.r_k = s.r_k;
    ly.lnx_w = s.lnx_w, ly.lnx_b = s.lnx_b, ly.ffn_x_k = s.ffn_x_k;
    ly.big[0] = s.att_r, ly.big[1] = s.att_k, ly.big[2] = s.att_v, ly.big[3] = s.att_o;
    ly.big[4] = s.ffn_key, ly.big[5] = s.ffn_value;
    if (l2) {
      int ks = 0;
      const rwkvb_packed* wr[3] = {&s.att_r, &s.att_k, &s.att_v};
      float* orkv[3] = {e->part_r, e->part_k, e->part_v};
      const uint8_t* drkv[3] = {e->dig_r, e->dig_k, e->dig_v};
      const float2* crkv[3] = {e->cs_r, e->cs_k, e->cs_v};
      st = bt_l2_setup(&ly.l2rkv, wr, orkv, drkv, crkv, 3, batch, e->sms, Pk, &e->l2g_rkv, &ks);
      if (i == 0)
        for (int j = 0; j < 3; ++j) e->pp_rkv[j] = bt_l2_pieces(ks);
      const rwkvb_packed* wo = &s.att_o;
      float* oo = e->part_o;
      const uint8_t* dy = e->dig_y;
      const float2* cy = e->cs_y;
      if (st == RWKVB_OK) st = bt_l2_setup(&ly.l2o, &wo, &oo, &dy, &cy, 1, batch, e->sms, Pk, &e->l2g_o, &ks);
      if (i == 0) e->pp_o = bt_l2_pieces(ks);
      const rwkvb_packed* wk = &s.ffn_key;
      float* ok = e->part_key;
      const uint8_t* df = e->dig_f;
      const float2* cf = e->cs_f;
      if (st == RWKVB_OK) st = bt_l2_setup(&ly.l2key, &wk, &ok, &df, &cf, 1, batch, e->sms, Pk, &e->l2g_key, &ks);
      if (i == 0) e->pp_key = bt_l2_pieces(ks);
      const rwkvb_packed* wv = &s.ffn_value;
      float* ov = e->part_val;
      const uint8_t* dh = e->dig_h;
      const float2* ch = e->cs_h;
      if (st == RWKVB_OK)
        st = bt_l2_setup(&ly.l2value, &wv, &ov, &dh, &ch, 1, batch, e->sms, Pf, &e->l2g_value, &ks);
      if (i == 0) e->pp_value = bt_l2_pieces(ks);
      if (!e->l2_cores) {
        size_t sm = 0;
        const LmJob jr[3] = {{&s.att_r, e->part_r, e->dig_r, e->cs_r},
                             {&s.att_k, e->part_k, e->dig_k, e->cs_k},
                             {&s.att_v, e->part_v, e->dig_v, e->cs_v}};
        const LmJob jo{&s.att_o, e->part_o, e->dig_y, e->cs_y}, jk{&s.ffn_key, e->part_key, e->dig_f, e->cs_f},
            jv{&s.ffn_value, e->part_val, e->dig_h, e->cs_h};
        if (st == RWKVB_OK) st = lm_setup(&ly.lmrkv, jr, 3, batch, e->sms, Pk, &e->lmg_rkv, &sm, e->err);
        e->smem_lm = std::max(e->smem_lm, sm);
        if (st == RWKVB_OK) st = lm_setup(&ly.lmo, &jo, 1, batch, e->sms, Pk, &e->lmg_o, &sm, e->err);
        e->smem_lm = std::max(e->smem_lm, sm);
        if (st == RWKVB_OK) st = lm_setup(&ly.lmkey, &jk, 1, batch, e->sms, Pk, &e->lmg_key, &sm, e->err);
        e->smem_lm = std::max(e->smem_lm, sm);
        if (st == RWKVB_OK) st = lm_setup(&ly.lmvalue, &jv, 1, batch, e->sms, Pf, &e->lmg_value, &sm, e->err);
        e->smem_lm = std::max(e->smem_lm, sm);
        if (i == 0 && st == RWKVB_OK) {
          for (int j = 0; j < 3; ++j) e->pp_rkv[j] = lm_pieces(ly.lmrkv, j, e->lmg_rkv);
          e->pp_o = lm_pieces(ly.lmo, 0, e->lmg_o);
          e->pp_key = lm_pieces(ly.lmkey, 0, e->lmg_key);
          e->pp_value = lm_pieces(ly.lmvalue, 0, e->lmg_value);
        }
      }
      e->layers.push_back(ly);
      continue;
    }
    const BgJob jr[3] = {{&s.att_r, 0, e->part_r}, {&s.att_k, 1, e->part_k}, {&s.att_v, 2, e->part_v}};
    st = bg_setup(&ly.rkv, jr, 3, d_rkv, 3, batch, e->sms, &e->g_rkv, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    const BgJob jo{&s.att_o, 0, e->part_o};
    if (st == RWKVB_OK) st = bg_setup(&ly.o, &jo, 1, &d_y, 1, batch, e->sms, &e->g_o, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    const BgJob jk{&s.ffn_key, 0, e->part_key};
    if (st == RWKVB_OK) st = bg_setup(&ly.key, &jk, 1, &d_f, 1, batch, e->sms, &e->g_key, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    const BgJob jv{&s.ffn_value, 0, e->part_val};
    if (st == RWKVB_OK)
      st = bg_setup(&ly.value, &jv, 1, &d_h, 1, batch, e->sms, &e->g_value, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pf) st = RWKVB_EUNSUPPORTED;
    e->smem_bg = smem;
    if (i == 0 && st == RWKVB_OK) {
      for (int j = 0; j < 3; ++j) e->pp_rkv[j] = bt_pieces(ly.rkv, j, e->g_rkv);
      e->pp_o = bt_pieces(ly.o, 0, e->g_o);
      e->pp_key = bt_pieces(ly.key, 0, e->g_key);
      e->pp_value = bt_pieces(ly.value, 0, e->g_value);
    }
    e->layers.push_back(ly);
  }
  if (st == RWKVB_OK && l2) {
    int ks = 0;
    const rwkvb_packed* wh = &m->head;
    float* oh = e->part_head;
    const uint8_t* doo = e->dig_o;
    const float2* co = e->cs_o;
    st = bt_l2_setup(&e->l2head, &wh, &oh, &doo, &co, 1, batch, e->sms, Pk, &e->l2g_head, &ks);
    e->pp_head = bt_l2_pieces(ks);
    if (st == RWKVB_OK && !e->l2_cores) {
      size_t sm = 0;
      const LmJob jh{&m->head, e->part_head, e->dig_o, e->cs_o};
      st = lm_setup(&e->lmhead, &jh, 1, batch, e->sms, Pk, &e->lmg_head, &sm, e->err);
      e->smem_lm = std::max(e->smem_lm, sm);
      e->pp_head = lm_pieces(e->lmhead, 0, e->lmg_head);
    }
    if (st == RWKVB_OK && !e->l2_cores)
      st = cuda_status(
          cudaFuncSetAttribute(l2mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)e->smem_lm));
  } else if (st == RWKVB_OK) {
    const BgJob jh{&m->head, 0, e->part_head};
    st = bg_setup(&e->head, &jh, 1, &d_o, 1, batch, e->sms, &e->g_head, &pieces, &smem, e->err);
    if (st == RWKVB_OK && pieces > Pk) st = RWKVB_EUNSUPPORTED;
    e->pp_head = bt_pieces(e->head, 0, e->g_head);
  }
  if (st == RWKVB_OK)
    st = bt_np_upload({{&e->pp_rkv[0], Ca}, {&e->pp_rkv[1], Ca}, {&e->pp_rkv[2], Ca}, {&e->pp_o, C},
                       {&e->pp_key, F}, {&e->pp_value, C}, {&e->pp_head, V}},
                      &e->np_dev);
  if (st == RWKVB_OK) {
    // every kernel must be launchable with the block size the step uses
    struct {
      const void* fn;
      int threads;
      const char* name;
    } ks[] = {{(const void*)bgemm_kernel, kBgThreads, "bgemm_kernel"},
              {(const void*)bt_embed_kernel, kBtThreads, "bt_embed_kernel"},
              {(const void*)bt_in_kernel, kBtRowThreads, "bt_in_kernel"},
              {(const void*)bt_adp1_kernel, kBtThreads, "bt_adp1_kernel"},
              {(const void*)bt_adp2_kernel, kBtThreads, "bt_adp2_kernel"},
              {(const void*)bt_wkv_kernel, kBtThreads, "bt_wkv_kernel"},
              {(const void*)bt_ffn_kernel, kBtRowThreads, "bt_ffn_kernel"},
              {(const void*)bt_hdig_kernel, kBtThreads, "bt_hdig_kernel"},
              {(const void*)bt_argmax_kernel, 1024, "bt_argmax_kernel"},
              {(const void*)bt_l2gemm_kernel, kL2Threads, "bt_l2gemm_kernel"},
              {(const void*)l2mma_kernel, kLmThreads, "l2mma_kernel"}};
    for (const auto& k : ks) {
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, k.fn) != cudaSuccess || fa.maxThreadsPerBlock < k.threads) {
        if (std::getenv("RWKVB_DEBUG"))
          std::fprintf(stderr, "rwkvb: %s: max %d threads per block (needs %d), %d registers\n", k.name,
                       fa.maxThreadsPerBlock, k.threads, fa.numRegs);
        cudaGetLastError();
        st = RWKVB_EUNSUPPORTED;
      }
    }
  }
  if (st == RWKVB_OK && !l2) st = bg_allow_smem(e->smem_bg);
  if (st == RWKVB_OK)
    st = cuda_status(
        cudaFuncSetAttribute(bt_adp1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBtAdp1Smem));
  if (st == RWKVB_OK) {
    const cudaError_t ce =
        cudaFuncSetAttribute(bt_adp2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * 2 * kBtAdp2Rc * 64));
    st = cuda_status(ce);
    if (st == RWKVB_OK)
      st = cuda_status(cudaFuncSetAttribute(bt_in_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)(sizeof(float) * 5 * C)));
  }
  if (st != RWKVB_OK) {
    cudaFree(e->arena);
    if (e->np_dev) cudaFree(e->np_dev);
    delete e;
    return st;
  }
  *out = e;
  return RWKVB_OK;
}
}  // namespace
}  // namespace rwkvb

extern "C" int rwkvb_batch_create(const rwkvb_model_desc* m, int32_t batch, uint32_t flags, rwkvb_batch** out) {
  return bt_create(m, batch, flags, nullptr, out);
}

extern "C" int rwkvb_batch_create_tp(const rwkvb_model_desc* local, int32_t batch, const rwkvb_tp_desc* tp,
                                     uint32_t flags, rwkvb_batch** out) {
  if (!tp) return RWKVB_EARG;
  return bt_create(local, batch, flags, tp, out);
}

extern "C" int rwkvb_batch_tp_exchange_bytes(const rwkvb_model_desc* local, int32_t batch, uint64_t* bytes) {
  if (!local || !bytes || batch < 1 || batch > kBgMaxSessions) return RWKVB_EARG;
  *bytes = (uint64_t)bt_x_layout(local->n_layer, batch, local->n_embd).bytes;
  return RWKVB_OK;
}

extern "C" int rwkvb_ipc_alloc(uint64_t bytes, void** dev_ptr, uint8_t* handle) {
  if (!dev_ptr || !handle || bytes == 0) return RWKVB_EARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  cudaIpcMemHandle_t h;
  int st = cuda_status(cudaMemset(p, 0, bytes));
  if (st == RWKVB_OK) st = cuda_status(cudaIpcGetMemHandle(&h, p));
  if (st != RWKVB_OK) {
    cudaFree(p);
    return st;
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return RWKVB_OK;
}

extern "C" int rwkvb_ipc_free(void* dev_ptr) { return dev_ptr ? cuda_status(cudaFree(dev_ptr)) : RWKVB_EARG; }

extern "C" int rwkvb_ipc_open(const uint8_t* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return RWKVB_EARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int rwkvb_ipc_close(void* dev_ptr) {
  return dev_ptr ? cuda_status(cudaIpcCloseMemHandle(dev_ptr)) : RWKVB_EARG;
}

extern "C" int rwkvb_batch_prepare(rwkvb_batch* e, void* stream) {
  (void)stream;
  if (!e) return RWKVB_EARG;
  return e->use_graph ? bt_capture_step(e) : RWKVB_OK;
}

extern "C" int rwkvb_batch_destroy(rwkvb_batch* e) {
  if (!e) return RWKVB_EARG;
  cudaDeviceSynchronize();
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->pf) {
    if (e->pf->exec) cudaGraphExecDestroy(e->pf->exec);
    if (e->pf->arena) cudaFree(e->pf->arena);
    if (e->pf->np_dev) cudaFree(e->pf->np_dev);
    delete e->pf;
  }
  if (e->arena) cudaFree(e->arena);
  if (e->np_dev) cudaFree(e->np_dev);
  delete e;
  return RWKVB_OK;
}

extern "C" int rwkvb_batch_buffers(rwkvb_batch* e, float** att_x, float** wkv, float** ffn_x, float** logits) {
  if (!e) return RWKVB_EARG;
  if (att_x) *att_x = e->att_x;
  if (wkv) *wkv = e->wkv;
  if (ffn_x) *ffn_x = e->ffn_x;
  if (logits) *logits = e->logits;
  return RWKVB_OK;
}

extern "C" int rwkvb_batch_reset(rwkvb_batch* e, void* stream) {
  if (!e) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t nbC = (size_t)e->nb * e->C;
  cudaError_t err = cudaMemsetAsync(e->att_x, 0, sizeof(float) * e->L * nbC, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->wkv, 0, sizeof(float) * (size_t)e->L * e->nb * e->H * 4096, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->ffn_x, 0, sizeof(float) * e->L * nbC, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->err, 0, sizeof(int), s);
  return cuda_status(err);
}

extern "C" int rwkvb_batch_forward(rwkvb_batch* e, const int32_t* tokens, void* stream) {
  if (!e || !tokens) return RWKVB_EARG;
  for (int i = 0; i < e->nb; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->Vfull) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  int st = cuda_status(cudaMemcpyAsync(e->tok, tokens, sizeof(int32_t) * e->nb, cudaMemcpyHostToDevice, s));
  if (st == RWKVB_OK) st = bt_run_step(e, s);
  return st;
}

extern "C" int rwkvb_batch_decode_greedy_async(rwkvb_batch* e, int32_t n, int32_t* out_dev, void* stream) {
  if (!e || n < 0 || (n > 0 && !out_dev)) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  int st = RWKVB_OK;
  for (int done = 0; done < n && st == RWKVB_OK;) {
    const int chunk = (n - done) < e->hist_cap ? (n - done) : e->hist_cap;
    st = cuda_status(cudaMemsetAsync(e->step, 0xff, sizeof(int), s));
    for (int i = 0; i < chunk && st == RWKVB_OK; ++i) st = bt_run_step(e, s);
    if (st == RWKVB_OK)
      st = cuda_status(cudaMemcpyAsync(out_dev + (size_t)done * e->nb, e->hist, sizeof(int32_t) * chunk * e->nb,
                                       cudaMemcpyDeviceToDevice, s));
    done += chunk;
  }
  return st;
}

extern "C" int rwkvb_batch_decode_greedy(rwkvb_batch* e, int32_t n, int32_t* out_host, void* stream) {
  if (!e || n < 0 || (n > 0 && !out_host)) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  int32_t* dev = nullptr;
  if (n > 0 && cudaMallocAsync((void**)&dev, sizeof(int32_t) * (size_t)n * e->nb, s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  int st = rwkvb_batch_decode_greedy_async(e, n, dev, s);
  if (st == RWKVB_OK && n > 0)
    st = cuda_status(
        cudaMemcpyAsync(out_host, dev, sizeof(int32_t) * (size_t)n * e->nb, cudaMemcpyDeviceToHost, s));
  if (dev) cudaFreeAsync(dev, s);
  const int st2 = cuda_status(cudaStreamSynchronize(s));
  if (st == RWKVB_OK) st = st2;
  if (st == RWKVB_OK) st = bt_check_err(e, s);
  return st;
}

extern "C" int rwkvb_batch_launches_per_step(rwkvb_batch* e, int32_t* out) {
  if (!e || !out) return RWKVB_EARG;
  // embed; per layer 12 (ln1/shift/digits, r/k/v GEMM, adapter stage 1, its
  // activation, stage 2, WKV, y digits, output GEMM, ln2/digits, key GEMM,
  // relu^2 digits, value GEMM) + 2 reductions under tensor parallelism; head
  // input, head GEMM, argmax (+ merge)
  *out = e->tp_size > 1 ? 1 + 14 * e->L + 4 : 1 + 12 * e->L + 3;
  return RWKVB_OK;
}
