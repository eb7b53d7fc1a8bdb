// Asynchronous data movement for the decode engine: mbarriers, 1-D TMA bulk
// copies into shared memory, cp.async 16-byte copies, programmatic dependent
// launch, and the ring-streamed SG8 GEMV built on them.
#pragma once

#include "common.cuh"

namespace rwkvb {

// Error flags written by device code (engine err word).
constexpr int kErrToken = 1;    // token id out of range
constexpr int kErrTimeout = 4;  // a bounded wait gave up

// ------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// -------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Non-blocking test of phase `parity` of `bar`.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` by polling (no suspension: the lowest
// wake-up latency, for the few threads on a pipeline's critical hand-off),
// giving up after `limit_ns` of wall time.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Wait for phase `parity` of `bar` to complete, giving up after `limit`
// polls (each poll may suspend the thread for a short hardware interval).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit = 1u << 22) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// One poll of phase `parity` of `bar` that may suspend the thread in hardware
// for up to `hint_ns` (it resumes as soon as the phase completes).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` with the thread suspended in hardware
// between polls (try_wait with a suspend-time hint: the thread resumes when
// the phase completes, or after at most `hint_ns`), giving up after
// `limit_ns` of wall time.  A waiting warp then takes no issue slots from
// the warps doing the work, unlike a tight poll loop.  The wall clock is
// read only once the first suspended poll has returned without the phase,
// so the common case is a single poll.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait_suspend(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs,
                                                  uint32_t hint_ns = 1000000u) {
  if (mbar_try_wait_hint(bar, parity, hint_ns)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_hint(bar, parity, hint_ns)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// 1-D bulk copy global -> shared (this CTA), completion counted on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// L2 policy for data read once per pass (the weight stream): its lines are the
// first to be evicted, so the small operands re-read on the latency-bound path
// (activations, accumulators, vectors, recurrent state) stay in L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 policy for small operands re-read every token on the latency-bound path
// (the adapter second stages of the decode kernel, ~1.6 MB per 2.9B layer):
// kept in L2 across tokens, so their loads do not queue behind the HBM stream.
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_g2s with an L2 cache policy (l2_evict_first).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// ---------------------------------------------------- cp.async (16B)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Wait until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copy `bytes` (multiple of 16, both pointers 16-byte aligned) with all threads.
__device__ __forceinline__ void cp_async_block(void* dst, const void* src, uint32_t bytes) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  for (uint32_t o = threadIdx.x * 16u; o < bytes; o += blockDim.x * 16u) cp_async16(d + o, s + o);
}

// ------------------------------------------------ vector staging
__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// dst4[i] = f(i) for i < n4 with all threads, eight independent loads in
// flight per thread (one memory round trip for vectors up to 8 KB per 256
// threads); ends with __syncthreads().
template <class F>
__device__ __forceinline__ void stage4(float* dst, int n4, F f) {
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int base = threadIdx.x; base < n4; base += 8 * blockDim.x) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * blockDim.x;
      if (i < n4) v[u] = f(i);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * blockDim.x;
      if (i < n4) d4[i] = v[u];
    }
  }
  __syncthreads();
}

// ======================================================= ring-streamed GEMV
// One CTA computes rows [row0, row1) of an SG8 W [rows, K] (row-aligned
// groups, gpr = K/group even, payload and metadata 16-byte aligned).
// Its rows stream through `nst` shared-memory slots of `rs` rows each
// (codes + scales as two bulk copies per slot).  Each warp owns one K segment
// (kseg = K / nseg) and keeps the input values of its lane's 16-wide chunks
// in registers (CPL chunks per lane); per row and segment a warp reduces
//   sum_chunks d_g * sum(q * x) + min_g * sum(x)      (lut2_gather.c:344-381)
// and the per-segment partials are summed in fixed order.
struct RingPlan {
  int row0, row1;  // this CTA's rows
  int K, gpr, lg;  // row length, groups per row, log2(group)
  int nseg, kseg;  // K segments
  int rs;          // rows per slot
  int nst;         // slots
  uint32_t slot_bytes;
};

struct RingSmem {
  uint8_t* slots;   // nst * slot_bytes
  uint64_t* bars;   // nst mbarriers
  float* part;      // 2 * rs * nseg partials
};

__device__ __forceinline__ void ring_issue(const PackedView& W, const RingPlan& P, const RingSmem& S, int stage) {
  const int r = P.row0 + stage * P.rs;
  const int nr = min(P.rs, P.row1 - r);
  const int slot = stage % P.nst;
  uint8_t* dst = S.slots + (size_t)slot * P.slot_bytes;
  const uint32_t qb = (uint32_t)nr * (uint32_t)P.K;
  const uint32_t sb = (uint32_t)nr * (uint32_t)P.gpr * 8u;
  mbar_expect_tx(&S.bars[slot], qb + sb);
  bulk_g2s(dst, W.payload + (size_t)r * P.K, qb, &S.bars[slot]);
  bulk_g2s(dst + (size_t)P.rs * P.K, W.meta + (size_t)r * P.gpr * 8, sb, &S.bars[slot]);
}

// Prologue: barrier init + first slots in flight.  Call with all threads,
// BEFORE pdl_wait() (weights never depend on the previous kernel).
__device__ __forceinline__ void ring_start(const PackedView& W, const RingPlan& P, const RingSmem& S) {
  const int nstage = (P.row1 - P.row0 + P.rs - 1) / P.rs;
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.nst; ++i) mbar_init(&S.bars[i], 1);
    fence_mbar_init();
    for (int t = 0; t < min(P.nst, nstage); ++t) ring_issue(W, P, S, t);
  }
  __syncthreads();
}

// Consume every stage.  xin4(i) gives input elements i..i+3 of the row (i a
// multiple of 4; called after pdl_wait).  epi(row, value) receives each row.
// Returns false (and sets err) if a bounded wait gave up.
template <int CPL, class XIn, class Epi>
__device__ __forceinline__ bool ring_run(const PackedView& W, const RingPlan& P, const RingSmem& S, XIn xin4,
                                         Epi epi, int* err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int seg = warp % P.nseg, wsub = warp / P.nseg, wper = nw / P.nseg;
  const int nchunk = P.kseg >> 4;
  const int gshift = P.lg - 4;
  // input values of this lane's chunks (16-wide, 16-byte loads issued together), and their sums
  float xr[CPL][16];
  float xs[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = lane + 32 * j;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 v = c < nchunk ? xin4(seg * P.kseg + c * 16 + 4 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
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
  const int nstage = (P.row1 - P.row0 + P.rs - 1) / P.rs;
  bool ok = true;
  int t = 0;
  for (; t < nstage; ++t) {
    const int slot = t % P.nst;
    // every thread polls (bounded); the CTA then agrees on the outcome
    const bool got = mbar_wait_bounded(&S.bars[slot], (uint32_t)((t / P.nst) & 1));
    if (!__syncthreads_and(got)) {
      ok = false;
      if (threadIdx.x == 0) atomicOr(err, kErrTimeout);
      break;
    }
    const int r0 = P.row0 + t * P.rs;
    const int nr = min(P.rs, P.row1 - r0);
    const uint8_t* sq = S.slots + (size_t)slot * P.slot_bytes;
    const float2* ss = reinterpret_cast<const float2*>(sq + (size_t)P.rs * P.K);
    float* part = S.part + (t & 1) * P.rs * P.nseg;
    // two rows per warp pass: independent dependency chains for more ILP
    for (int ri = wsub; ri < nr; ri += 2 * wper) {
      const int rj = ri + wper;
      const bool two = rj < nr;
      const uint8_t* q0 = sq + (size_t)ri * P.K + seg * P.kseg;
      const uint8_t* q1 = sq + (size_t)(two ? rj : ri) * P.K + seg * P.kseg;
      const float2* sc0 = ss + ri * P.gpr + ((seg * P.kseg) >> P.lg);
      const float2* sc1 = ss + (two ? rj : ri) * P.gpr + ((seg * P.kseg) >> P.lg);
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunk) {
          const uint4 qa = *reinterpret_cast<const uint4*>(q0 + c * 16);
          const uint4 qb = *reinterpret_cast<const uint4*>(q1 + c * 16);
          const float2 sa = sc0[c >> gshift];
          const float2 sb = sc1[c >> gshift];
          const float4 x0 = make_float4(xr[j][0], xr[j][1], xr[j][2], xr[j][3]);
          const float4 x1 = make_float4(xr[j][4], xr[j][5], xr[j][6], xr[j][7]);
          const float4 x2 = make_float4(xr[j][8], xr[j][9], xr[j][10], xr[j][11]);
          const float4 x3 = make_float4(xr[j][12], xr[j][13], xr[j][14], xr[j][15]);
          float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
          a = dot4_u8(qa.x, x0, a);
          b = dot4_u8(qb.x, x0, b);
          a = dot4_u8(qa.y, x1, a);
          b = dot4_u8(qb.y, x1, b);
          a = dot4_u8(qa.z, x2, a);
          b = dot4_u8(qb.z, x2, b);
          a = dot4_u8(qa.w, x3, a);
          b = dot4_u8(qb.w, x3, b);
          acc0 = fmaf((sa.y - sa.x) * kInv255, a.x + a.y, fmaf(sa.x, xs[j], acc0));
          acc1 = fmaf((sb.y - sb.x) * kInv255, b.x + b.y, fmaf(sb.x, xs[j], acc1));
        }
      }
      acc0 = warp_sum(acc0);
      acc1 = warp_sum(acc1);
      if (lane == 0) {
        part[ri * P.nseg + seg] = acc0;
        if (two) part[rj * P.nseg + seg] = acc1;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && t + P.nst < nstage) ring_issue(W, P, S, t + P.nst);
    if ((int)threadIdx.x < nr) {
      float v = 0.f;
      for (int s = 0; s < P.nseg; ++s) v += part[threadIdx.x * P.nseg + s];
      epi(r0 + (int)threadIdx.x, v);
    }
  }
  if (!ok) {
    // let this CTA's outstanding copies land before it exits (bounded)
    if (threadIdx.x == 0) {
      const int issued = min(nstage, t + P.nst);
      for (int u = t; u < issued; ++u) mbar_wait_bounded(&S.bars[u % P.nst], (uint32_t)((u / P.nst) & 1), 1u << 16);
    }
    __syncthreads();
  }
  return ok;
}

// Host-side planning for a CTA count `ctas` over W's rows.  Returns false when
// W does not have the ring layout (callers then use the direct-load path).
__host__ inline bool ring_plan(const PackedView& W, int ctas, int slot_budget, int nst, int* cpl_out,
                               RingPlan* base) {
  if (W.kind != RWKVB_KIND_SG8 || W.lg < 4 || (W.cols % W.group) != 0) return false;
  const int K = W.cols, gpr = K / (int)W.group;
  if (gpr % 2 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(W.payload) & 15u) || (reinterpret_cast<uintptr_t>(W.meta) & 15u)) return false;
  int nseg = 1;
  while (nseg <= 8) {
    const int kseg = K / nseg;
    const bool fits = (K % nseg == 0) && (kseg % (int)W.group == 0) && (kseg % 16 == 0);
    const int cpl = (kseg / 16 + 31) / 32;
    if (fits && cpl <= 5) break;
    nseg *= 2;
  }
  if (nseg > 8) return false;
  const int kseg = K / nseg;
  const int row_bytes = K + gpr * 8;
  const int wper = 8 / nseg;
  // two rows per warp pass: slots hold a multiple of 2 * wper rows
  int rs = 2 * wper;
  while ((rs + 2 * wper) * row_bytes <= slot_budget) rs += 2 * wper;
  const int rpc = (W.rows + ctas - 1) / ctas;
  if (rs > rpc) rs = ((rpc + wper - 1) / wper) * wper;
  if (rs > 256) rs = 256;
  base->K = K;
  base->gpr = gpr;
  base->lg = W.lg;
  base->nseg = nseg;
  base->kseg = kseg;
  base->rs = rs;
  base->nst = nst;
  base->slot_bytes = (uint32_t)(rs * row_bytes);
  base->row0 = 0;
  base->row1 = rpc;  // rows per CTA (row0/row1 resolved per CTA on the device)
  *cpl_out = (kseg / 16 + 31) / 32;
  return true;
}

}  // namespace rwkvb
