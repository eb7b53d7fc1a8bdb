// Op-level C-ABI entry points: dequant, GEMV family, fused adapters, fused
// channel mix, WKV7.  Each mirrors one export of the reference's native
// library (rwkv_ssd/native/lut2_gather.c); see include/rwkv_b200.h.
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "wkv7.cuh"

namespace rwkvb {

// ------------------------------------------------------------------ dequant
__global__ void dequant_kernel(PackedView w, float* out, uint64_t numel) {
  for (uint64_t o = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; o < numel;
       o += (uint64_t)gridDim.x * blockDim.x) {
    if (w.kind == RWKVB_KIND_SG8) {
      out[o] = sg8_elem(w, o);
    } else {
      // out is in checkpoint order; input-major kinds encode the transpose.
      uint64_t e = o;
      if (lut2_input_major(w.kind)) {
        uint64_t r = o / (uint64_t)w.cols, c = o - r * (uint64_t)w.cols;
        e = c * (uint64_t)w.rows + r;
      }
      out[o] = lut2_elem(w, e);
    }
  }
}

// --------------------------------------------------------------------- GEMV
// y[row] = W[row, :] @ x for rows [blockIdx.x * rpc, ...).  blockIdx.y selects
// one of up to 3 (W, x, y) triples (batched QKV).
struct GemvArgs {
  PackedView w[4];
  const float* x[4];
  float* y[4];
  int mode[4];
  int lg[4];
  int rpc;   // rows per CTA
  int epi;   // 0 store, 1 relu^2
};

__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int m = blockIdx.y;
  const PackedView& W = a.w[m];
  const int r0 = blockIdx.x * a.rpc;
  const int r1 = min(W.rows, r0 + a.rpc);
  if (r0 >= r1) return;
  const int K = W.cols;
  float* sx = smem;
  float* sxc = smem + ((K + 15) & ~15);
  const float* x = a.x[m];
  if (a.mode[m] == 1) {
    stage_input(K, sx, sxc, [&](int i) { return __ldg(x + i); });
  } else {
    for (int i = threadIdx.x; i < K; i += blockDim.x) sx[i] = __ldg(x + i);
    __syncthreads();
  }
  float* y = a.y[m];
  const int epi = a.epi;
  packed_rows(W, a.mode[m], a.lg[m], sx, sxc, r0, r1, [&](int row, float v) {
    if (epi == 1) v = v > 0.f ? v * v : 0.f;
    y[row] = v;
  });
}

static size_t gemv_smem(int K) { return (size_t)(((K + 15) & ~15) + (K + 15) / 16 + 4) * sizeof(float); }

int launch_gemv(const PackedView* w, const float* const* x, float* const* y, int n, int epi,
                cudaStream_t s) {
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  int max_rows = 0, max_k = 0;
  for (int m = 0; m < n; ++m) {
    a.w[m] = w[m];
    a.x[m] = x[m];
    a.y[m] = y[m];
    a.mode[m] = gemv_mode(w[m]);
    a.lg[m] = ilog2u(w[m].group);
    max_rows = w[m].rows > max_rows ? w[m].rows : max_rows;
    max_k = w[m].cols > max_k ? w[m].cols : max_k;
  }
  int sms = device_sms();
  int target = (2 * sms + n - 1) / n;
  int rpc = (max_rows + target - 1) / target;
  rpc = rpc < 1 ? 1 : rpc;
  a.rpc = rpc;
  a.epi = epi;
  size_t sm = gemv_smem(max_k);
  if (sm > kMaxSmem) return RWKVB_EUNSUPPORTED;
  if (sm > 48 * 1024) {
    int st = allow_big_smem((const void*)gemv_kernel);
    if (st != RWKVB_OK) return st;
  }
  dim3 grid((max_rows + rpc - 1) / rpc, n);
  gemv_kernel<<<grid, 256, sm, s>>>(a);
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------- per-tensor LUT2 (TR2\x01) W @ x
// One warp per row, the reference's row walk (lut2_gather.c:186-210): row r
// reads its codes from byte (r * cols) / 4 on, four per byte, low bits first.
__global__ void __launch_bounds__(256) lut2_tensor_gemv_kernel(PackedView w, const float* x, float* y) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= w.rows) return;
  const int K = w.cols;
  const float* cb = reinterpret_cast<const float*>(w.meta);
  const float c0 = __ldg(cb), c1 = __ldg(cb + 1), c2 = __ldg(cb + 2), c3 = __ldg(cb + 3);
  const uint8_t* prow = w.payload + (((uint64_t)row * (uint64_t)K) >> 2);
  float acc = 0.f;
  for (int j = lane; 4 * j < K; j += 32) {
    const uint32_t b = __ldg(prow + j);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int col = 4 * j + u;
      if (col < K) {
        const uint32_t code = (b >> (2 * u)) & 3u;
        const float v = code == 0 ? c0 : (code == 1 ? c1 : (code == 2 ? c2 : c3));
        acc = fmaf(v, __ldg(x + col), acc);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

// ------------------------------------------------- activation-INT8 SG8 GEMV
// Per input group (one warp each): int8 codes q, scale and the fp32 group sum,
// following the reference's quantiser (lut2_gather.c:636-689): scale =
// max|x| / 127 (1 when max|x| <= 1e-12), q = x * (1 / scale) rounded half away
// from zero by truncating +-0.5, clamped to +-127; the sum in column order.
__global__ void i8_quant_kernel(const float* __restrict__ x, int g, int groups, int8_t* __restrict__ q,
                                float* __restrict__ scale, float* __restrict__ sum_x) {
  const int grp = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (grp >= groups) return;
  const float* xg = x + (size_t)grp * g;
  float m = 0.f;
  for (int i = lane; i < g; i += 32) m = fmaxf(m, fabsf(__ldg(xg + i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float sc = m > 1.0e-12f ? __fdiv_rn(m, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, sc);
  for (int i = lane; i < g; i += 32) {
    const float v = __fmul_rn(__ldg(xg + i), inv);
    int qi = v >= 0.f ? __float2int_rz(__fadd_rn(v, 0.5f)) : __float2int_rz(__fsub_rn(v, 0.5f));
    qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
    q[(size_t)grp * g + i] = (int8_t)qi;
  }
  if (lane == 0) {
    float sx = 0.f;
    for (int i = 0; i < g; ++i) sx = __fadd_rn(sx, __ldg(xg + i));
    scale[grp] = sc;
    sum_x[grp] = sx;
  }
}

__device__ __forceinline__ int dp4a_u8s8(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

struct I8Args {
  PackedView w[3];
  const int8_t* q[3];
  const float* scale[3];
  const float* sum_x[3];
  float* y[3];
};

// One warp per row (blockIdx.y selects the map): lane l takes groups l, l + 32,
// ...; per group the exact integer dot of the u8 codes and int8 activations,
// then min * sum(x) + (max - min) / 255 * scale * dot.
__global__ void __launch_bounds__(256) i8_gemv_kernel(I8Args a, int g) {
  const int m = blockIdx.y;
  const PackedView& w = a.w[m];
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= w.rows) return;
  const int K = w.cols, groups = K / g;
  const size_t rg = (size_t)row * (size_t)groups;  // first weight group of the row
  float acc = 0.f;
  for (int gi = lane; gi < groups; gi += 32) {
    const uint32_t* wq = reinterpret_cast<const uint32_t*>(w.payload + (rg + gi) * (size_t)g);
    const uint32_t* xq = reinterpret_cast<const uint32_t*>(a.q[m] + (size_t)gi * g);
    int dot = 0;
    for (int i = 0; i < (g >> 2); ++i) dot = dp4a_u8s8(__ldg(wq + i), __ldg(xq + i), dot);
    const float2 p = ldg_f2(w.meta + (rg + gi) * 8);
    acc += p.x * __ldg(a.sum_x[m] + gi) + (p.y - p.x) * kInv255 * __ldg(a.scale[m] + gi) * (float)dot;
  }
  acc = warp_sum(acc);
  if (lane == 0) a.y[m][row] = acc;
}

// ----------------------------------------------------- transposed (x @ W)
// part[split][j] over rows [split*ch, ...) of W [R, C] row-major.
__global__ void transposed_partial_kernel(PackedView w, const float* x, int ch, float* part) {
  const int s = blockIdx.x;
  const int i0 = s * ch, i1 = min(w.rows, i0 + ch);
  const int j0 = blockIdx.y * 256, j1 = min(w.cols, j0 + 256);
  if (i0 >= i1 || j0 >= j1) return;
  transposed_partial(w, x, i0, i1, j0, j1, part + (size_t)s * w.cols + j0);
}

// out[j] = act(bias[j] + sum_s part[s][j]); act 0 none, 1 tanh, 2 sigmoid.
__global__ void reduce_act_kernel(const float* part, int splits, int n, const float* bias, int act, float* out) {
  int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  float acc = 0.f;
  for (int s = 0; s < splits; ++s) acc += part[(size_t)s * n + j];
  if (bias) acc = bias[j] + acc;
  if (act == 1) acc = tanhf(acc);
  if (act == 2) acc = sigmoidf_(acc);
  out[j] = acc;
}

int launch_transposed(const PackedView& w, const float* x, float* y, const float* bias, int act,
                      float* scratch, cudaStream_t s) {
  // scratch >= splits * w.cols floats (splits <= 64)
  int splits = w.rows >= 512 ? 32 : (w.rows >= 64 ? 8 : 1);
  int ch = (w.rows + splits - 1) / splits;
  splits = (w.rows + ch - 1) / ch;
  dim3 grid(splits, (w.cols + 255) / 256);
  transposed_partial_kernel<<<grid, 256, 0, s>>>(w, x, ch, scratch);
  reduce_act_kernel<<<(w.cols + 255) / 256, 256, 0, s>>>(scratch, splits, w.cols, bias, act, y);
  return cuda_status(cudaGetLastError());
}

// --------------------------------------------------------------------- WKV7
__global__ void __launch_bounds__(256) wkv7_kernel(float* state, float* y, const float* r, const float* w,
                                                   const float* k, const float* v, const float* kk,
                                                   const float* a, int n_head, int mode) {
  __shared__ __align__(16) float sr[64], sd[64], sk[64], sv[64], skk[64], ska[64];
  const int bh = blockIdx.x;  // batch * n_head + head
  const size_t off = (size_t)bh * 64;
  if (threadIdx.x < 64) {
    int t = threadIdx.x;
    float wv = w[off + t];
    sd[t] = mode == 0 ? expf(-0.606531f * sigmoidf_(wv)) : expf(-expf(wv));
    sr[t] = r[off + t];
    sk[t] = k[off + t];
    sv[t] = v[off + t];
    skk[t] = kk[off + t];
    ska[t] = kk[off + t] * a[off + t];
  }
  __syncthreads();
  wkv7_head64(state + (size_t)bh * 4096, sr, sd, sk, sv, skk, ska, y + off);
}

}  // namespace rwkvb

using namespace rwkvb;

// ======================================================================= ABI
extern "C" int rwkvb_version(void) { return RWKVB_ABI_VERSION; }

extern "C" const char* rwkvb_status_string(int st) {
  switch (st) {
    case RWKVB_OK: return "ok";
    case RWKVB_EARG: return "invalid argument or malformed packed blob";
    case RWKVB_EALLOC: return "device allocation failed";
    case RWKVB_ECUDA: return "CUDA runtime error";
    case RWKVB_ETIMEOUT: return "bounded device wait timed out";
    case RWKVB_EUNSUPPORTED: return "unsupported shape or configuration";
    case RWKVB_ESCRATCH: return "request exceeds the fixed static scratch buffer";
    default: return "unknown status";
  }
}

extern "C" int rwkvb_packed_init(rwkvb_packed* out, const uint8_t* header, uint64_t blob_bytes,
                                 const uint8_t* device_blob, int32_t rows, int32_t cols) {
  if (!out || !header || rows <= 0 || cols <= 0 || blob_bytes < 8) return RWKVB_EARG;
  uint32_t group;
  memcpy(&group, header + 4, 4);
  const bool per_tensor = header[0] == 'T' && header[1] == 'R' && header[2] == '2' && header[3] == 1;
  if (group == 0 && !per_tensor) return RWKVB_EARG;
  uint64_t numel = (uint64_t)rows * (uint64_t)cols;
  uint64_t groups = per_tensor ? 1 : (numel + group - 1) / group;
  uint32_t kind;
  if (header[0] == 'S' && header[1] == 'G' && header[2] == '8' && header[3] == 1) {
    kind = RWKVB_KIND_SG8;
    if (blob_bytes != 8 + groups * 8 + numel) return RWKVB_EARG;  // pack_codec.py:136
  } else if (header[0] == 'T' && header[1] == 'R' && header[2] == '2' && header[3] >= 3 && header[3] <= 7) {
    kind = header[3];
    if (blob_bytes < 8 + groups * rwkvb_lut2_record_bytes(kind) + (numel + 3) / 4) return RWKVB_EARG;
  } else if (header[0] == 'T' && header[1] == 'R' && header[2] == '2' && header[3] == 1) {
    // per-tensor LUT2: the whole tensor is the one "group" of its codebook
    // (bytes 4..8 are codebook[0], not a group size); _lut2_inner_view checks
    // the 20-byte header (trinity_codec.py:306-323)
    kind = RWKVB_KIND_LUT2_TENSOR;
    if (numel > 0xffffffffull || blob_bytes < 20 + (numel + 3) / 4) return RWKVB_EARG;
    group = (uint32_t)numel;
  } else {
    return RWKVB_EARG;
  }
  out->data = device_blob;
  out->bytes = blob_bytes;
  out->kind = kind;
  out->group_size = group;
  out->rows = rows;
  out->cols = cols;
  return RWKVB_OK;
}

static bool packed_ok(const rwkvb_packed* w) {
  return w && w->data && w->rows > 0 && w->cols > 0 && w->group_size > 0 &&
         (w->kind == RWKVB_KIND_SG8 || (w->kind >= 3 && w->kind <= 7) || w->kind == RWKVB_KIND_LUT2_TENSOR);
}

extern "C" int rwkvb_dequant_f32(float* out, const rwkvb_packed* w, void* stream) {
  if (!out || !packed_ok(w)) return RWKVB_EARG;
  uint64_t numel = (uint64_t)w->rows * w->cols;
  int blocks = (int)((numel + 255) / 256);
  int cap = device_sms() * 16;
  blocks = blocks > cap ? cap : blocks;
  dequant_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(make_view(*w), out, numel);
  return cuda_status(cudaGetLastError());
}

extern "C" int rwkvb_gemv_f32(float* y, const rwkvb_packed* w, const float* x, void* stream) {
  if (!y || !x || !packed_ok(w)) return RWKVB_EARG;
  PackedView v = make_view(*w);
  if (v.kind == RWKVB_KIND_LUT2_TENSOR) {
    lut2_tensor_gemv_kernel<<<(v.rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(v, x, y);
    return cuda_status(cudaGetLastError());
  }
  return launch_gemv(&v, &x, &y, 1, 0, (cudaStream_t)stream);
}

extern "C" int rwkvb_tmix_gemv_f32(float* y_out, const rwkvb_packed* const* w, const float* const* x, int32_t n,
                                   void* stream) {
  if (!y_out || !w || !x || n < 1 || n > 4) return RWKVB_EARG;
  PackedView v[4];
  float* ys[4];
  for (int m = 0; m < n; ++m) {
    if (!packed_ok(w[m]) || !x[m]) return RWKVB_EARG;
    if (w[m]->rows != w[0]->rows || w[m]->cols != w[0]->cols) return RWKVB_EARG;
    v[m] = make_view(*w[m]);
    ys[m] = y_out + (size_t)m * w[0]->rows;
  }
  return launch_gemv(v, x, ys, n, 0, (cudaStream_t)stream);
}

// Activation-INT8 SG8 maps (1 or 3): quantise every input, then the integer
// GEMV; scratch [K] int8 + [2 * groups] fp32 per map, stream-ordered.
static int i8_maps(const rwkvb_packed* const* w, const float* const* x, float* const* y, int n, cudaStream_t s) {
  const int K = w[0]->cols, g = (int)w[0]->group_size, groups = K / g;
  const size_t per = ((size_t)K + 255) / 256 * 256 + (size_t)groups * 8;
  uint8_t* scratch = nullptr;
  if (cudaMallocAsync((void**)&scratch, per * n, s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  I8Args a;
  memset(&a, 0, sizeof(a));
  int st = RWKVB_OK;
  for (int m = 0; m < n && st == RWKVB_OK; ++m) {
    uint8_t* base = scratch + per * m;
    int8_t* q = reinterpret_cast<int8_t*>(base);
    float* sc = reinterpret_cast<float*>(base + ((size_t)K + 255) / 256 * 256);
    float* sx = sc + groups;
    i8_quant_kernel<<<(groups + 7) / 8, 256, 0, s>>>(x[m], g, groups, q, sc, sx);
    st = cuda_status(cudaGetLastError());
    a.w[m] = make_view(*w[m]);
    a.q[m] = q;
    a.scale[m] = sc;
    a.sum_x[m] = sx;
    a.y[m] = y[m];
  }
  if (st == RWKVB_OK) {
    i8_gemv_kernel<<<dim3((w[0]->rows + 7) / 8, n), 256, 0, s>>>(a, g);
    st = cuda_status(cudaGetLastError());
  }
  cudaFreeAsync(scratch, s);
  return st;
}

static bool i8_ok(const rwkvb_packed* w) {
  return packed_ok(w) && w->kind == RWKVB_KIND_SG8 && w->cols % (int)w->group_size == 0 && w->group_size % 4 == 0;
}

extern "C" int rwkvb_gemv_sg8_i8_f32(float* y, const rwkvb_packed* w, const float* x, void* stream) {
  if (!y || !x || !packed_ok(w) || w->kind != RWKVB_KIND_SG8) return RWKVB_EARG;
  if (!i8_ok(w) || ((uintptr_t)make_view(*w).payload & 3u)) return rwkvb_gemv_f32(y, w, x, stream);  // float path
  return i8_maps(&w, &x, &y, 1, (cudaStream_t)stream);
}

extern "C" int rwkvb_tmix_qkv_i8_gemv_f32(float* y_out, const rwkvb_packed* const* w3, const float* const* x3,
                                          void* stream) {
  if (!y_out || !w3 || !x3) return RWKVB_EARG;
  bool fast = true;
  for (int m = 0; m < 3; ++m) {
    if (!packed_ok(w3[m]) || !x3[m] || w3[m]->kind != RWKVB_KIND_SG8) return RWKVB_EARG;
    if (w3[m]->rows != w3[0]->rows || w3[m]->cols != w3[0]->cols) return RWKVB_EARG;
    fast = fast && i8_ok(w3[m]) && w3[m]->group_size == w3[0]->group_size &&
           !((uintptr_t)make_view(*w3[m]).payload & 3u);
  }
  if (!fast) return rwkvb_tmix_qkv_gemv_f32(y_out, w3, x3, stream);  // the reference's float fallback
  float* ys[3] = {y_out, y_out + w3[0]->rows, y_out + 2 * (size_t)w3[0]->rows};
  return i8_maps(w3, x3, ys, 3, (cudaStream_t)stream);
}

extern "C" int rwkvb_tmix_qkv_gemv_f32(float* y_out, const rwkvb_packed* const* w3, const float* const* x3,
                                       void* stream) {
  if (!y_out || !w3 || !x3) return RWKVB_EARG;
  PackedView v[3];
  float* ys[3];
  for (int m = 0; m < 3; ++m) {
    if (!packed_ok(w3[m]) || !x3[m]) return RWKVB_EARG;
    if (w3[m]->rows != w3[0]->rows || w3[m]->cols != w3[0]->cols) return RWKVB_EARG;
    v[m] = make_view(*w3[m]);
    ys[m] = y_out + (size_t)m * w3[0]->rows;
  }
  return launch_gemv(v, x3, ys, 3, 0, (cudaStream_t)stream);
}

extern "C" int rwkvb_transposed_gemv_f32(float* y, const rwkvb_packed* w, const float* x, void* stream) {
  if (!y || !x || !packed_ok(w) || w->kind != RWKVB_KIND_SG8) return RWKVB_EARG;
  cudaStream_t s = (cudaStream_t)stream;
  float* scratch = nullptr;
  if (cudaMallocAsync((void**)&scratch, sizeof(float) * 64 * (size_t)w->cols, s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  int st = launch_transposed(make_view(*w), x, y, nullptr, 0, scratch, s);
  cudaFreeAsync(scratch, s);
  return st;
}

extern "C" int rwkvb_tmix_adapters_f32(float* w_out, float* a_out, float* g_out, float* v_out,
                                       const rwkvb_packed* const* mats, const float* const* xs,
                                       const float* a0, int has_v, void* stream) {
  if (!w_out || !a_out || !g_out || !mats || !xs || !a0) return RWKVB_EARG;
  int nm = has_v ? 8 : 6;
  for (int m = 0; m < nm; ++m)
    if (!packed_ok(mats[m]) || mats[m]->kind != RWKVB_KIND_SG8) return RWKVB_EARG;
  if (has_v && (!v_out || !xs[3])) return RWKVB_EARG;
  const int C = mats[1]->cols;
  for (int p = 0; p < nm / 2; ++p) {
    const rwkvb_packed* first = mats[2 * p];
    const rwkvb_packed* second = mats[2 * p + 1];
    if (!xs[p] || first->rows != C || second->cols != C || first->cols != second->rows) return RWKVB_EARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int max_rank = 0;
  for (int p = 0; p < nm / 2; ++p) max_rank = mats[2 * p]->cols > max_rank ? mats[2 * p]->cols : max_rank;
  float* scratch = nullptr;
  size_t part = 64 * (size_t)(C > max_rank ? C : max_rank);
  if (cudaMallocAsync((void**)&scratch, sizeof(float) * (part + 4 * (size_t)max_rank), s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  float* mid = scratch + part;
  float* outs[4] = {w_out, a_out, g_out, v_out};
  // act after stage 1: w tanh, a none, g sigmoid, v none (lut2_gather.c:1072-1077)
  const int act1[4] = {1, 0, 2, 0};
  int st = RWKVB_OK;
  for (int p = 0; p < nm / 2 && st == RWKVB_OK; ++p) {
    PackedView f = make_view(*mats[2 * p]);
    PackedView g = make_view(*mats[2 * p + 1]);
    st = launch_transposed(f, xs[p], mid + p * max_rank, nullptr, act1[p], scratch, s);
    if (st == RWKVB_OK)
      st = launch_transposed(g, mid + p * max_rank, outs[p], p == 1 ? a0 : nullptr, p == 1 ? 2 : 0, scratch, s);
  }
  cudaFreeAsync(scratch, s);
  return st;
}

extern "C" int rwkvb_cmix_gemv_f32(float* y, const rwkvb_packed* key, const rwkvb_packed* value, const float* x,
                                   void* stream) {
  if (!y || !x || !packed_ok(key) || !packed_ok(value)) return RWKVB_EARG;
  if (value->cols != key->rows) return RWKVB_EARG;  // lut2_gather.c:515-518
  cudaStream_t s = (cudaStream_t)stream;
  float* h = nullptr;
  if (cudaMallocAsync((void**)&h, sizeof(float) * (size_t)key->rows, s) != cudaSuccess) {
    cudaGetLastError();
    return RWKVB_EALLOC;
  }
  PackedView kv = make_view(*key), vv = make_view(*value);
  int st = launch_gemv(&kv, &x, &h, 1, 1, s);
  const float* hc = h;
  if (st == RWKVB_OK) st = launch_gemv(&vv, &hc, &y, 1, 0, s);
  cudaFreeAsync(h, s);
  return st;
}

extern "C" int rwkvb_wkv7_f32(float* state, float* y, const float* r, const float* w, const float* k,
                              const float* v, const float* kk, const float* a, int batch, int n_head,
                              int head_size, int decay_mode, void* stream) {
  if (!state || !y || !r || !w || !k || !v || !kk || !a || batch <= 0 || n_head <= 0) return RWKVB_EARG;
  if (head_size != 64 || (decay_mode != 0 && decay_mode != 1)) return RWKVB_EUNSUPPORTED;
  wkv7_kernel<<<batch * n_head, 256, 0, (cudaStream_t)stream>>>(state, y, r, w, k, v, kk, a, n_head, decay_mode);
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------------- no-allocation channel mix
// The intermediate of rwkvb_cmix_gemv_f32_noalloc: one fixed buffer per device
// (a __device__ variable is instantiated in every device's context).
static __device__ __align__(256) float g_cmix_scratch[RWKVB_CMIX_NOALLOC_MAX_FFN];

namespace {
constexpr int kMaxDevices = 64;
struct ScratchSlot {
  float* ptr;
  unsigned long long ctx_id;  // unique id of the context the address belongs to
};
ScratchSlot g_cmix_scratch_slot[kMaxDevices];
std::mutex g_cmix_scratch_mu;

typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);

// Unique id of the calling thread's current context (never reused within the
// process, unlike the context handle); false when none is current or the
// driver entry points are unavailable.
bool current_ctx_id(unsigned long long* id) {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && p)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess && p)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    cudaGetLastError();
  });
  if (!get_cur || !get_id) return false;
  void* ctx = nullptr;
  if (get_cur(&ctx) != 0 || !ctx) return false;
  return get_id(ctx, id) == 0;
}

// Address of g_cmix_scratch in the current device's context.  Resolved once
// per context: a device reset (cudaDeviceReset) replaces the context and the
// address is resolved again in the new one.
int cmix_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return RWKVB_EUNSUPPORTED;
  unsigned long long id = 0;
  const bool known = current_ctx_id(&id);
  std::lock_guard<std::mutex> lock(g_cmix_scratch_mu);
  ScratchSlot& s = g_cmix_scratch_slot[dev];
  if (s.ptr && known && s.ctx_id == id) {
    *out = s.ptr;
    return RWKVB_OK;
  }
  float* p = nullptr;
  e = cudaGetSymbolAddress((void**)&p, g_cmix_scratch);
  if (e != cudaSuccess) return cuda_status(e);
  unsigned long long id2 = 0;
  if (current_ctx_id(&id2)) {  // the lookup made the context current if none was
    s.ptr = p;
    s.ctx_id = id2;
  } else {
    s.ptr = nullptr;  // no context id to key on: resolve again next call
  }
  *out = p;
  return RWKVB_OK;
}
}  // namespace

extern "C" int rwkvb_cmix_gemv_f32_noalloc(float* y, const rwkvb_packed* key, const rwkvb_packed* value,
                                           const float* x, void* stream) {
  if (!y || !x || !packed_ok(key) || !packed_ok(value)) return RWKVB_EARG;
  if (value->cols != key->rows) return RWKVB_EARG;
  if (key->rows > RWKVB_CMIX_NOALLOC_MAX_FFN) return RWKVB_ESCRATCH;
  float* h = nullptr;
  int st = cmix_scratch(&h);
  if (st != RWKVB_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  PackedView kv = make_view(*key), vv = make_view(*value);
  st = launch_gemv(&kv, &x, &h, 1, 1, s);
  const float* hc = h;
  if (st == RWKVB_OK) st = launch_gemv(&vv, &hc, &y, 1, 0, s);
  return st;
}
