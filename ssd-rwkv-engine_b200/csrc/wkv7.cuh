// WKV7 per-head recurrent state update (RWKV-7 time mix, rwkv7_linear.py:314-337).
#pragma once

#include "common.cuh"

namespace rwkvb {

// One head, N = 64, 256 threads.  S is the head's [64][64] fp32 state in global
// memory (row i = value index, column j = key index), updated in place:
//   sa[i] = sum_j S[i][j] * (-kk[j])
//   S[i][j] = S[i][j] * d[j] + sa[i] * ka[j] + v[i] * k[j]
//   y[i] = sum_j S[i][j] * r[j]
// Vectors live in shared memory.  Thread t owns row t/4, columns (t%4)*16..+16:
// the state is read and written exactly once, with 16-byte vector accesses.
// Each thread visits its four 4-column blocks starting at block (row & 3), so
// that a warp's 16-byte accesses to a shared-memory S (rows 256 bytes apart,
// all starting in the same bank) spread over all 32 banks; the sums over j run
// in that order.
// out != nullptr: the new state goes to `out` (global, same layout) instead of S.
__device__ __forceinline__ void wkv7_head64(float* __restrict__ S, const float* r, const float* d,
                                            const float* k, const float* v, const float* kk, const float* ka,
                                            float* y, float* out = nullptr) {
  const int t = threadIdx.x;
  const int i = t >> 2, q = (t & 3) << 4, rot = i & 3;
  float4* row = reinterpret_cast<float4*>(S + i * 64 + q);
  float s[16];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float4 a = row[(u + rot) & 3];
    s[4 * u] = a.x; s[4 * u + 1] = a.y; s[4 * u + 2] = a.z; s[4 * u + 3] = a.w;
  }
  // the same 16 entries of each vector, in the same block order, as four
  // 16-byte loads (q is a multiple of 16; the vectors are 16-byte aligned)
  auto ld16 = [&](const float* p, float (&o)[16]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 f = reinterpret_cast<const float4*>(p + q)[(u + rot) & 3];
      o[4 * u] = f.x; o[4 * u + 1] = f.y; o[4 * u + 2] = f.z; o[4 * u + 3] = f.w;
    }
  };
  float vkk[16];
  ld16(kk, vkk);
  float sa = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) sa = fmaf(s[j], -vkk[j], sa);
  sa += __shfl_xor_sync(0xffffffffu, sa, 1);
  sa += __shfl_xor_sync(0xffffffffu, sa, 2);
  const float vi = v[i];
  float vd[16], vka[16], vk[16], vr[16];
  ld16(d, vd);
  ld16(ka, vka);
  ld16(k, vk);
  ld16(r, vr);
  float yy = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float nv = s[j] * vd[j] + sa * vka[j] + vi * vk[j];
    s[j] = nv;
    yy = fmaf(nv, vr[j], yy);
  }
  yy += __shfl_xor_sync(0xffffffffu, yy, 1);
  yy += __shfl_xor_sync(0xffffffffu, yy, 2);
  float4* dst = out ? reinterpret_cast<float4*>(out + i * 64 + q) : row;
#pragma unroll
  for (int u = 0; u < 4; ++u) dst[(u + rot) & 3] = make_float4(s[4 * u], s[4 * u + 1], s[4 * u + 2], s[4 * u + 3]);
  if ((t & 3) == 0) y[i] = yy;
}

}  // namespace rwkvb
