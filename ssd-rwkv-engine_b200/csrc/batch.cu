// Batched decode: the tcgen05 SG8 GEMM (bgemm.cuh) behind the op-level entry
// rwkvb_gemm_sg8_f32, and the host plan shared with the batched engine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "bgemm.cuh"
#include "common.cuh"
#include "internal.h"

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
    a->cs[d] = dg[d].cs;
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
  const size_t stage_bytes = (size_t)kBgTileBytes + (size_t)a->nrows * 128;
  a->stages = (int)std::min<size_t>(kBgMaxStages, (kBgSmemBudget - 1024) / stage_bytes);
  if (a->stages < 2) return RWKVB_EUNSUPPORTED;
  a->idesc = idesc_u8u8_s32(128, a->nrows);
  a->spin_limit = 1u << 22;
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

int bg_launch(const BgArgs& a, int grid, size_t smem, cudaStream_t s) {
  int st = bg_allow_smem(smem);
  if (st != RWKVB_OK) return st;
  bgemm_kernel<<<grid, kBgThreads, smem, s>>>(a);
  return cuda_status(cudaGetLastError());
}

// Constant rows of a digit matrix: zero everything, then the ones row (3 bp).
int bg_digits_init(uint8_t* rows, int k, int nb, cudaStream_t s) {
  const int bp = bg_padded_sessions(nb), nrows = bg_digit_rows(nb);
  cudaError_t e = cudaMemsetAsync(rows, 0, (size_t)nrows * k, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(rows + (size_t)3 * bp * k, 1, (size_t)k, s);
  return cuda_status(e);
}

int bg_digits(uint8_t* rows, float2* cs, const float* x, int ldx, int k, int nb, int group, cudaStream_t s) {
  const int lfk = group == 64 ? 6 : 7;
  const int warps = nb * (k >> lfk);
  bg_digits_kernel<<<(warps + 7) / 8, 256, 0, s>>>(rows, cs, x, ldx, k, nb, bg_padded_sessions(nb), lfk);
  return cuda_status(cudaGetLastError());
}

}  // namespace rwkvb

using namespace rwkvb;

extern "C" int rwkvb_gemm_sg8_f32(float* y, const rwkvb_packed* w, const float* x, int32_t batch, int32_t* err_word,
                                  void* stream) {
  if (!y || !w || !x || batch <= 0 || batch > kBgMaxSessions) return RWKVB_EARG;
  if (!bg_matrix_ok(*w)) return w->kind == RWKVB_KIND_SG8 ? RWKVB_EUNSUPPORTED : RWKVB_EARG;
  if (reinterpret_cast<uintptr_t>(x) % 16) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int K = w->cols, N = w->rows, nb = batch;
  const int bp = bg_padded_sessions(nb), nrows = bg_digit_rows(nb);
  const size_t dig_bytes = (size_t)nrows * K;
  const size_t cs_bytes = sizeof(float2) * (size_t)(K / w->group_size) * bp;
  uint8_t* dig = nullptr;
  const size_t cs_off = (dig_bytes + 255) & ~size_t(255);
  const size_t err_off = (cs_off + cs_bytes + 255) & ~size_t(255);
  if (cudaMallocAsync((void**)&dig, err_off + 256, s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  float2* cs = reinterpret_cast<float2*>(dig + cs_off);
  if (!err_word) {  // no caller word: timeouts still stop the kernel, unreported
    err_word = reinterpret_cast<int32_t*>(dig + err_off);
    cudaMemsetAsync(err_word, 0, sizeof(int32_t), s);
  }
  BgDigits dg{dig, cs, K};
  BgArgs a;
  int grid = 0, pieces = 0;
  size_t smem = 0;
  BgJob job{w, 0, nullptr};
  int st = bg_setup(&a, &job, 1, &dg, 1, nb, device_sms(), &grid, &pieces, &smem, err_word);
  float* part = nullptr;
  if (st == RWKVB_OK && cudaMallocAsync((void**)&part, sizeof(float) * (size_t)pieces * nb * N, s) != cudaSuccess) {
    cudaGetLastError();
    st = RWKVB_EALLOC;
  }
  if (st == RWKVB_OK) {
    a.mat[0].out = part;
    st = bg_digits_init(dig, K, nb, s);
    if (st == RWKVB_OK) st = bg_digits(dig, cs, x, K, K, nb, (int)w->group_size, s);
    if (st == RWKVB_OK) st = bg_launch(a, grid, smem, s);
    if (st == RWKVB_OK) {
      bg_reduce_kernel<<<(nb * N + 255) / 256, 256, 0, s>>>(y, part, nb, N, 0, K / 128, a.total, grid);
      st = cuda_status(cudaGetLastError());
    }
  }
  if (part) cudaFreeAsync(part, s);
  cudaFreeAsync(dig, s);
  return st;
}
