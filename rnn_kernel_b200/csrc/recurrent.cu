// Persistent GRU time-loop kernels for B200 (sm_100a).
//
// Design (replaces the reference's grid-cooperative sm_80 kernels
// `..._row4_k1_shmem_gate_cache_kernel` and `..._split6_..._unroll8_kernel`,
// src/rnn_kernel/a100/prod/kernels/a100_gru_h256_kernels.cu:656-779 and
// :782-933):
//
// * The batch is split over independent thread-block clusters.  A cluster of
//   C = ceil(H/32) CTAs holds the whole W_hh on chip, in registers: CTA c owns
//   hidden units j in [c*Hc, c*Hc + Hc) and thus the three W_hh rows
//   (r_j, z_j, n_j).  Clusters never talk to each other, so there is no grid
//   barrier and no co-residency requirement on the batch size.
// * Forward, per step: every CTA multiplies its 3*Hc rows with the full
//   h_{t-1} of its cluster's batch rows (held in its own shared memory), does
//   the gate math for its units, and pushes the new h slice into the next
//   h buffer of every CTA of the cluster with `st.async` remote stores that
//   complete bytes on the receiver's mbarrier.  The receiver waits on its own
//   mbarrier only: there is no per-step cluster barrier and no fence that
//   would wait for the step's global stores.  h is double-buffered.
// * Backward, per step: every CTA computes the pointwise backward for its
//   units, then its share of dh_{t-1} = dG_hh . W_hh over all k, and
//   reduce-scatters that partial into the owning CTAs' shared memory the same
//   way (double-buffered partials, one mbarrier per buffer).
// * The recurrent products use packed FP32 FMA (FFMA2) on pairs of
//   independent partial sums.
// * Per-step inputs (input gates; dout and the stash) are prefetched `pd`
//   steps ahead into a shared-memory ring with cp.async.
// * Every wait is bounded (about 2 s of %globaltimer); on expiry the kernel
//   records GRU_STATUS_WAIT_TIMEOUT in the device status word
//   (gru_device_status()), leaves its time loop and exits through the final
//   cluster barrier.
//
// Gate math follows custom_gru.py:117-122 / a100_gru_h256_kernels.cu:758-775
// (forward) and :852-866 (backward).

#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace cg = cooperative_groups;

namespace gru {

__device__ int g_device_status = 0;

#ifdef GRU_TIMELINE
// Step timeline, compiled only into instrumented builds (-DGRU_TIMELINE):
// clock64() at marked points of iterations [kTlIt0, kTlIt0 + kTlSteps) of
// every launch, for threads 0 and blockDim-1 of every CTA, kept in shared
// memory during the loop (so the markers add no global stores to the
// measured stretches) and copied out for the first two CTAs of cluster 0 at
// the end of the launch (the last launch of each direction wins).
constexpr int kTlIt0 = 100, kTlSteps = 8, kTlPts = 12;
__device__ long long g_tl[2][4][kTlSteps][kTlPts];
#define GRU_TL_INIT                                                                      \
  __shared__ long long tl_s[2][kTlSteps][kTlPts];                                        \
  if (threadIdx.x == 0 || threadIdx.x == blockDim.x - 1)                                 \
    for (int q = 0; q < kTlSteps * kTlPts; ++q) (&tl_s[threadIdx.x != 0][0][0])[q] = 0;
#define GRU_TL(dir, k)                                                                                \
  do {                                                                                                \
    if ((threadIdx.x == 0 || threadIdx.x == blockDim.x - 1) && it >= kTlIt0 && it < kTlIt0 + kTlSteps) \
      tl_s[threadIdx.x != 0][it - kTlIt0][k] = clock64();                                             \
  } while (0)
#define GRU_TL_FLUSH(dir)                                                               \
  do {                                                                                  \
    if (blockIdx.x < 2 && (threadIdx.x == 0 || threadIdx.x == blockDim.x - 1))          \
      for (int q = 0; q < kTlSteps * kTlPts; ++q)                                       \
        (&g_tl[dir][blockIdx.x * 2 + (threadIdx.x != 0)][0][0])[q] =                    \
            (&tl_s[threadIdx.x != 0][0][0])[q];                                         \
  } while (0)
#else
#define GRU_TL_INIT
#define GRU_TL(dir, k) \
  do {                 \
  } while (0)
#define GRU_TL_FLUSH(dir) \
  do {                    \
  } while (0)
#endif

namespace {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t mapa_u32(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: false (and the timeout recorded) if the phase did not
// complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                               unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) {
      atomicOr(&g_device_status, GRU_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void st_async_f32(uint32_t remote_addr, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(remote_addr),
               "r"(__float_as_uint(v)), "r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async16(float* smem_dst, const float* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
  if (n >= 6) cp_async_wait<6>();
  else if (n == 5) cp_async_wait<5>();
  else if (n == 4) cp_async_wait<4>();
  else if (n == 3) cp_async_wait<3>();
  else if (n == 2) cp_async_wait<2>();
  else if (n == 1) cp_async_wait<1>();
  else cp_async_wait<0>();
}

// Store v as the pair (tf32(v), tf32(v - tf32(v))), both round to nearest.
__device__ __forceinline__ void split_store(float* hi, float* lo, float v) {
  uint32_t h, l;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
  const float r = v - __uint_as_float(h);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(r));
  *hi = __uint_as_float(h);
  *lo = __uint_as_float(l);
}

// 1/(1+e^-v).  The reciprocal is the hardware approximation (rcp.approx,
// at most 1 ulp off) refined by one Newton-Raphson step y += y (1 - d y),
// which leaves it within about 1 ulp of the exact quotient at a fraction of
// the latency of the correctly rounded reciprocal on the step's critical
// path.  v is clamped so that d stays finite (d = inf would give 0 * inf in
// the refinement); sigmoid(-80) = 1.8e-35 is already 0 at the tolerance of
// any use.
__device__ __forceinline__ float sigmoidf_acc(float v) {
  const float d = 1.0f + expf(-fmaxf(v, -80.0f));
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
  return fmaf(y, fmaf(-d, y, 1.0f), y);
}

// Parity of the mbarrier phase that carries the data consumed at iteration
// `it` (>= 1) from a buffer used every other iteration: one buffer is first
// consumed at it = 1, the other at it = 2, then each every second iteration.
constexpr int kMaxPrefetch = 8;  // deepest per-step input ring (steps)
// most per-step prefetch items (a row's inputs for 1 or 4 units) a thread
// keeps planned in registers
constexpr int kPlanItems = 2;

__device__ __forceinline__ uint32_t phase_parity(int it) { return (uint32_t)((((it + 1) >> 1) - 1) & 1); }

struct FwdArgs {
  const float* G;     // [B,T,3H] input gates (x.W_ih^T + b_ih), row stride 3H rounded up to 4
  const float* h0;    // [B,H]
  const float* w_hh;  // [3H,H]
  const float* b_hh;  // [3H]
  float* out;         // [B,T,H]
  float* hn;          // [B,H]
  float* stash;       // [B,T,5H] or null
  // Steps [t0, t0 + nt) of the sequence: h0 is the state before step t0 and
  // hn receives the state after step t0 + nt - 1 (a time chunk of a longer
  // sequence when nt < T; every row index still uses the full T).
  int t0, nt;
};

// R = batch rows per GEMV sub-chunk (= rows per cluster when that is <= 8).
template <int R>
__global__ void __launch_bounds__(256, 1)
gru_fwd_recurrent_kernel(FwdArgs a, RecGeom g) {
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int cid = blockIdx.x / g.C;
  const int b_begin = cid * g.bc;
  const int nb = min(g.bc, g.B - b_begin);
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int H = g.H, T = g.T, Hc = g.Hc, Kp = g.nw * 32, bcp = g.bcp, pd = g.pd;
  const int ldg = (3 * H + 3) & ~3;  // row stride of G
  const int t0 = a.t0, nT = a.nt;  // this launch's steps
  const int j0 = c * Hc;
  const int hcnt = max(1, min(Hc, H - j0));
  // first pointwise item of this thread (row, unit) in a sub-chunk
  const int my_s = tid / hcnt, my_jl = tid - my_s * hcnt;

  extern __shared__ __align__(16) float smem[];
  __shared__ __align__(8) unsigned long long mbar[2];
  float* hbuf = smem;                          // [2][bcp][Kp]
  float* part = smem + g.off1;                 // [R][3][2 halves][32 units][4 warp slots]
  float* ring = smem + g.off2;                 // [pd][bcp][3][Hc]
  float* bsl = smem + g.off3;                  // [3][Hc] this CTA's slice of b_hh
  GRU_TL_INIT
  const int ring_stride = bcp * 3 * Hc;
  const int slot_stride = bcp * Kp;

  // W_hh rows (r, z, n) of unit j0+lane, columns [32*warp, 32*warp+32), as
  // pairs of consecutive columns for FFMA2.
  float2 wr[16], wz[16], wn[16];
  if (H % 4 == 0 && (reinterpret_cast<uintptr_t>(a.w_hh) & 15) == 0) {
    // The 32 columns of a row this thread holds are contiguous: 8 16-byte
    // loads per gate (the scalar loads below, lanes on 32 different rows,
    // made this prologue ~16 us, a cost paid by every launch).
    const int jg = j0 + lane;
    const bool jv = lane < hcnt && jg < H;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int k = warp * 32 + 4 * q;
      const bool v = jv && k < H;  // H % 4 == 0: a 16-byte piece is wholly inside or outside
      const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 r = v ? *reinterpret_cast<const float4*>(a.w_hh + (size_t)jg * H + k) : zero;
      const float4 z = v ? *reinterpret_cast<const float4*>(a.w_hh + (size_t)(H + jg) * H + k) : zero;
      const float4 n = v ? *reinterpret_cast<const float4*>(a.w_hh + (size_t)(2 * H + jg) * H + k) : zero;
      wr[2 * q] = make_float2(r.x, r.y), wr[2 * q + 1] = make_float2(r.z, r.w);
      wz[2 * q] = make_float2(z.x, z.y), wz[2 * q + 1] = make_float2(z.z, z.w);
      wn[2 * q] = make_float2(n.x, n.y), wn[2 * q + 1] = make_float2(n.z, n.w);
    }
  } else {
    const int jg = j0 + lane;
    const bool jv = lane < hcnt && jg < H;
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      const int k = warp * 32 + 2 * kk;
      const bool v0 = jv && k < H, v1 = jv && k + 1 < H;
      wr[kk] = make_float2(v0 ? a.w_hh[(size_t)jg * H + k] : 0.f, v1 ? a.w_hh[(size_t)jg * H + k + 1] : 0.f);
      wz[kk] = make_float2(v0 ? a.w_hh[(size_t)(H + jg) * H + k] : 0.f,
                           v1 ? a.w_hh[(size_t)(H + jg) * H + k + 1] : 0.f);
      wn[kk] = make_float2(v0 ? a.w_hh[(size_t)(2 * H + jg) * H + k] : 0.f,
                           v1 ? a.w_hh[(size_t)(2 * H + jg) * H + k + 1] : 0.f);
    }
  }

  for (int e = tid; e < 2 * slot_stride; e += nthr) hbuf[e] = 0.0f;
  for (int e = tid; e < R * 3 * 32 * 8; e += nthr) part[e] = 0.0f;  // slots of absent warps stay 0
  for (int e = tid; e < 3 * Hc; e += nthr) {
    const int q = e / Hc, jl = e - q * Hc;
    bsl[e] = jl < hcnt ? a.b_hh[q * H + j0 + jl] : 0.0f;
  }
  __syncthreads();
  for (int e = tid; e < nb * H; e += nthr) {
    const int b = e / H, k = e - b * H;
    hbuf[b * Kp + k] = a.h0[(size_t)(b_begin + b) * H + k];
  }
  const uint32_t bar0 = smem_u32(&mbar[0]);
  const uint32_t bytes_per_step = (uint32_t)(nb * H * 4);
  if (tid == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    fence_mbar_init();
    if (nT > 1) mbar_expect_tx(bar0 + 8, bytes_per_step);  // slot 1 <- step 1
  }

  // Prefetch of step s's input gates into ring slot s % pd by the threads
  // first, first + stride, ...: 16-byte copies when the rows are 16-byte
  // aligned (H and Hc multiples of 4), else 4-byte copies.  No commit.
  const bool vec4 = g.vec4 != 0;
  auto issue = [&](int s, int first, int stride) {
    float* dst = ring + (s % pd) * ring_stride;
    const float* src = a.G + ((size_t)b_begin * T + t0 + s) * ldg + j0;
    const size_t bstride = (size_t)T * ldg;
    if (vec4) {
      const int h4 = hcnt >> 2, n = nb * 3 * h4;
      for (int e = first; e < n; e += stride) {
        const int r = e / h4, jl = 4 * (e - r * h4);
        const int b = r / 3, gi = r - 3 * b;
        cp_async16(dst + r * Hc + jl, src + b * bstride + gi * H + jl);
      }
    } else {
      const int n = nb * 3 * hcnt;
      for (int e = first; e < n; e += stride) {
        const int r = e / hcnt, jl = e - r * hcnt;
        const int b = r / 3, gi = r - 3 * b;
        cp_async4(dst + r * Hc + jl, src + b * bstride + gi * H + jl);
      }
    }
  };
  for (int s = 0; s < pd - 1; ++s) {
    if (s < nT) issue(s, tid, nthr);
    cp_async_commit();
  }
  // In the time loop the same threads issue the same copies every step (the
  // threads idle in the last sub-chunk's pointwise, else all threads after
  // the sends): plan them once, so that a step's prefetch is address adds and
  // copies only (no index divisions competing for issue slots with the GEMV).
  const int ns_last = nb - ((nb - 1) / R) * R;
  const int nact_last = ns_last * hcnt;
  const bool idle_issue = nact_last < nthr;
  const int pfirst = idle_issue ? tid - nact_last : tid, pstride = idle_issue ? nthr - nact_last : nthr;
  // Entry k of the plan: gates gi0 .. gi0 + cpe - 1 of row b, units
  // jl .. jl + w - 1 of this CTA, to ring offsets plan_dst[k] + gi * Hc from
  // G_c + s * 3H + plan_off[k] + gi * H (G_c = this cluster's rows, this CTA's
  // units).  cpe (copies per entry, 1 or 3) is the smallest that keeps every
  // thread at kPlanItems entries or fewer.
  int plan_n = 0, cpe = 1;
  int plan_dst[kPlanItems], plan_off[kPlanItems];
  const float* const G_c = a.G + (size_t)b_begin * T * ldg + j0;
  {
    const int w = vec4 ? 4 : 1;
    const int hw = hcnt / w;
#pragma unroll
    for (int k = 0; k < kPlanItems; ++k) plan_dst[k] = plan_off[k] = 0;
    if (pstride > 0 && nb * 3 * hw > kPlanItems * pstride) cpe = 3;
    const int n = nb * (3 / cpe) * hw;
    // more than kPlanItems entries per issuing thread, or offsets beyond 32
    // bits: no plan.  The decision must be the same for every thread of the
    // CTA (a planned and an unplanned thread index the items differently).
    if (kPlanItems * pstride < n || (size_t)nb * T * ldg >= (1ull << 31)) plan_n = -1;
    if (pfirst >= 0 && plan_n == 0) {
#pragma unroll
      for (int k = 0; k < kPlanItems; ++k) {
        const int e = pfirst + k * pstride;
        if (e < n) {
          const int r = e / hw, jl = w * (e - r * hw);
          const int b = cpe == 3 ? r : r / 3, gi0 = cpe == 3 ? 0 : r - 3 * b;
          plan_dst[k] = (b * 3 + gi0) * Hc + jl;
          plan_off[k] = b * T * ldg + gi0 * H + jl;
          plan_n = k + 1;
        }
      }
    }
  }
  auto issue_step = [&](int s) {
    if (plan_n < 0) {
      issue(s, pfirst, pstride);
      return;
    }
    float* dst = ring + (s % pd) * ring_stride;
    const float* src = G_c + (size_t)(t0 + s) * ldg;
#pragma unroll
    for (int k = 0; k < kPlanItems; ++k) {
      if (k < plan_n) {
        float* d = dst + plan_dst[k];
        const float* g = src + plan_off[k];
        for (int gi = 0; gi < cpe; ++gi) {
          if (vec4)
            cp_async16(d + gi * Hc, g + gi * H);
          else
            cp_async4(d + gi * Hc, g + gi * H);
        }
      }
    }
  };

  const uint32_t hbuf_u32 = smem_u32(hbuf);
  cluster.sync();  // buffers and mbarriers of every CTA initialised

  bool ok = true;
  for (int it = 0; it < nT; ++it) {
    const int t = t0 + it;  // absolute step (row index); `it` counts this launch's steps
    const int cur = it & 1, nxt = cur ^ 1;
    const float* hcur = hbuf + cur * slot_stride;
    const float* rg = ring + (it % pd) * ring_stride;
    GRU_TL(0, 0);
    // After an expired wait (recorded in the status word) this thread stops
    // waiting but still runs every remaining barrier, so no thread of the CTA
    // or cluster is left behind at one; the results are then invalid.
    if (it > 0 && ok) ok = mbar_wait_bounded(bar0 + 8 * cur, phase_parity(it));
    GRU_TL(0, 1);

    for (int b0 = 0; b0 < nb; b0 += R) {
      float2 acc[R][3];
#pragma unroll
      for (int s = 0; s < R; ++s) acc[s][0] = acc[s][1] = acc[s][2] = make_float2(0.f, 0.f);
      const float* hb = hcur + b0 * Kp + warp * 32;
#pragma unroll
      for (int kk = 0; kk < 32; kk += 4) {
#pragma unroll
        for (int s = 0; s < R; ++s) {
          const float4 hv = *reinterpret_cast<const float4*>(hb + s * Kp + kk);
          const float2 h01 = make_float2(hv.x, hv.y), h23 = make_float2(hv.z, hv.w);
          acc[s][0] = __ffma2_rn(wr[kk / 2], h01, acc[s][0]);
          acc[s][1] = __ffma2_rn(wz[kk / 2], h01, acc[s][1]);
          acc[s][2] = __ffma2_rn(wn[kk / 2], h01, acc[s][2]);
          acc[s][0] = __ffma2_rn(wr[kk / 2 + 1], h23, acc[s][0]);
          acc[s][1] = __ffma2_rn(wz[kk / 2 + 1], h23, acc[s][1]);
          acc[s][2] = __ffma2_rn(wn[kk / 2 + 1], h23, acc[s][2]);
        }
      }
      // Partial of warp w for (row s, gate q, unit lane) goes to slot
      // (w + lane/8) % 8 of that unit, stored as half slot/4, element slot%4:
      // the 32 lanes hit 32 distinct banks, and the pointwise thread reads its
      // unit's 8 partials with two float4 loads that are contiguous across
      // lanes (4 wavefronts each).
      if (b0 == 0) GRU_TL(0, 2);
      const int slot = (warp + (lane >> 3)) & 7;
      float* pw = part + ((slot >> 2) * 32 + lane) * 4 + (slot & 3);
#pragma unroll
      for (int s = 0; s < R; ++s) {
#pragma unroll
        for (int q = 0; q < 3; ++q) pw[(s * 3 + q) * 256] = acc[s][q].x + acc[s][q].y;
      }
      if (b0 == 0) cp_async_wait_dyn(pd - 2);
      __syncthreads();
      if (b0 == 0) GRU_TL(0, 3);
      // Every thread is past its wait on slot `cur`: re-arm it for step t+2.
      // (the last thread: it has no pointwise item when R * hcnt < nthr)
      if (b0 == 0 && tid == nthr - 1 && it + 2 < nT) mbar_expect_tx(bar0 + 8 * cur, bytes_per_step);

      const int ns = min(R, nb - b0);
      // Threads without a pointwise item in the last sub-chunk issue the
      // prefetch for step t+pd-1 meanwhile (it overwrites ring slot
      // (t-1) % pd: past this step's wait every thread of the cluster has
      // sent its step t-1 values, each of which depended on its reads of that
      // slot).
      const int nact = ns * hcnt;
      if (b0 + R >= nb && idle_issue && tid >= nact && it + pd - 1 < nT) issue_step(it + pd - 1);
      if (b0 + R >= nb) GRU_TL(0, 9);
      for (int e = tid; e < ns * hcnt; e += nthr) {
        const int s = e == tid ? my_s : e / hcnt, jl = e == tid ? my_jl : e - s * hcnt;
        const int b = b0 + s, j = j0 + jl;
        const float4* pp = reinterpret_cast<const float4*>(part + (s * 3) * 256 + jl * 4);
        const float4 r0 = pp[0], r1 = pp[32], z0 = pp[64], z1 = pp[96], n0 = pp[128], n1 = pp[160];
        const float ar = bsl[jl] + (((r0.x + r0.y) + (r0.z + r0.w)) + ((r1.x + r1.y) + (r1.z + r1.w)));
        const float az = bsl[Hc + jl] + (((z0.x + z0.y) + (z0.z + z0.w)) + ((z1.x + z1.y) + (z1.z + z1.w)));
        const float an = bsl[2 * Hc + jl] + (((n0.x + n0.y) + (n0.z + n0.w)) + ((n1.x + n1.y) + (n1.z + n1.w)));
        if (e == tid && b0 == 0) GRU_TL(0, 4);
        const float* gi = rg + (b * 3) * Hc + jl;
        const float r = sigmoidf_acc(gi[0] + ar);
        const float z = sigmoidf_acc(gi[Hc] + az);
        const float n = tanhf(gi[2 * Hc] + r * an);
        const float hp = hcur[b * Kp + j];
        const float hnew = n + z * (hp - n);
        if (e == tid && b0 == 0) GRU_TL(0, 5);
        if (it + 1 < nT) {
          const uint32_t la = hbuf_u32 + 4u * (uint32_t)(nxt * slot_stride + b * Kp + j);
          const uint32_t lb = bar0 + 8u * nxt;
          for (int q = 0; q < g.C; ++q) st_async_f32(mapa_u32(la, q), hnew, mapa_u32(lb, q));
        }
        if (e == tid && b0 == 0) GRU_TL(0, 6);
        const size_t row = (size_t)(b_begin + b) * T + t;
        a.out[row * H + j] = hnew;
        if (a.stash != nullptr) {
          float* st = a.stash + row * 5 * H + j;
          st[0] = r;
          st[H] = z;
          st[2 * H] = n;
          st[3 * H] = an;
          st[4 * H] = hp;
        }
        if (it == nT - 1) a.hn[(size_t)(b_begin + b) * H + j] = hnew;
        if (e == tid && b0 == 0) GRU_TL(0, 7);
      }
      if (b0 + R < nb) __syncthreads();  // `part` is reused by the next sub-chunk
    }
    // Every thread had a pointwise item: prefetch now, after the sends.
    if (!idle_issue && it + pd - 1 < nT) issue_step(it + pd - 1);
    cp_async_commit();
    GRU_TL(0, 8);
  }
  GRU_TL_FLUSH(0);
  cp_async_wait<0>();
  cluster.sync();  // no CTA leaves while a peer may still write into it
}

struct BwdArgs {
  const float* dout;   // [B,T,H] or null
  const float* dhn;    // [B,H] or null
  const float* w_hh;   // [3H,H]
  const float* stash;  // [B,T,5H]
  // dG_ih [B,T,3H] (row stride ldgi) and the n block of dG_hh [B,T,H] (row
  // stride ldgn; its r and z blocks equal dG_ih's and are not stored), each
  // written pre-split for the tensor-core products: hi = tf32(v),
  // lo = tf32(v - hi).
  float* dGi;
  float* dGi_lo;
  int ldgi;
  float* dGh;
  float* dGh_lo;
  int ldgn;
  float* dh0;          // [B,H]
  // Bias-gradient partial sums of this launch, one row of 4H per cluster
  // (cols [0, 3H): dG_ih's r, z, n columns; [3H, 4H): dG_hh's n block),
  // accumulated on chip in FP64 over every (b, t) of the cluster.
  double* dbpart;
  // Steps [t0, t0 + nt), walked backwards: dhn is the gradient flowing into
  // step t0 + nt - 1 and dh0 receives the gradient of the state before t0.
  int t0, nt;
};

template <int R>
__global__ void __launch_bounds__(256, 1)
gru_bwd_recurrent_kernel(BwdArgs a, RecGeom g) {
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int cid = blockIdx.x / g.C;
  const int b_begin = cid * g.bc;
  const int nb = min(g.bc, g.B - b_begin);
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int H = g.H, T = g.T, Hc = g.Hc, bcp = g.bcp, pd = g.pd, C = g.C;
  const int j0 = c * Hc;
  const int hcnt = max(1, min(Hc, H - j0));
  // first pointwise item of this thread (row, unit) in a sub-chunk
  const int my_s = tid / hcnt, my_jl = tid - my_s * hcnt;
  // GEMV mapping: lane l of warp w owns the W_hh columns k0 = 32w + 2(l & 15)
  // and k0 + 1 for the half jh = l >> 4 of this CTA's units (16 each).
  const int jh = lane >> 4;
  const int k0 = warp * 32 + 2 * (lane & 15);
  const int ksend = k0 + jh;  // the column whose finished partial this lane sends

  extern __shared__ __align__(16) float smem[];
  __shared__ __align__(8) unsigned long long mbar[2];
  float* red = smem;                           // [2][C][bcp][Hc]
  float* gz = smem + g.off1;                   // [bcp][Hc]
  float* dgs = smem + g.off2;                  // [R][3][32]
  float* ring = smem + g.off3;                 // [pd][bcp][6][Hc]
  const int ring_stride = bcp * 6 * Hc;
  const int red_slot = C * bcp * Hc;
  GRU_TL_INIT

  // (W_hh[g*H + j][k0], W_hh[g*H + j][k0 + 1]) for the 16 units j of half jh,
  // as pairs over the two columns for FFMA2.
  float2 wr[16], wz[16], wn[16];
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const int jl = 16 * jh + jj;
    const bool vj = jl < hcnt && j0 + jl < H;
    const bool v0 = vj && k0 < H, v1 = vj && k0 + 1 < H;
    const size_t rr = (size_t)(j0 + jl) * H, rz = (size_t)(H + j0 + jl) * H, rn = (size_t)(2 * H + j0 + jl) * H;
    wr[jj] = make_float2(v0 ? a.w_hh[rr + k0] : 0.f, v1 ? a.w_hh[rr + k0 + 1] : 0.f);
    wz[jj] = make_float2(v0 ? a.w_hh[rz + k0] : 0.f, v1 ? a.w_hh[rz + k0 + 1] : 0.f);
    wn[jj] = make_float2(v0 ? a.w_hh[rn + k0] : 0.f, v1 ? a.w_hh[rn + k0 + 1] : 0.f);
  }

  for (int e = tid; e < 2 * red_slot; e += nthr) red[e] = 0.0f;
  for (int e = tid; e < bcp * Hc; e += nthr) gz[e] = 0.0f;
  for (int e = tid; e < R * 3 * 32; e += nthr) dgs[e] = 0.0f;
  // FP64 sums of dr, dz, dn_pre, dhn per (sub-chunk row s, unit): each is
  // owned by the one thread that computes that item in every step
  double* dbacc = reinterpret_cast<double*>(smem + g.off4);  // [R][4][Hc]
  for (int e = tid; e < R * 4 * Hc; e += nthr) dbacc[e] = 0.0;
  const uint32_t bar0 = smem_u32(&mbar[0]);
  const uint32_t bytes_per_step = (uint32_t)(C * nb * hcnt * 4);
  if (tid == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    fence_mbar_init();
    mbar_expect_tx(bar0, bytes_per_step);  // slot 0 <- partials of iteration 0
  }

  // Ring entry q: 0 dout, 1 r, 2 z, 3 n, 4 hn (= W_hn.h + b_hn), 5 h_prev.
  // Prefetch of iteration it's inputs into ring slot it % pd by the threads
  // first, first + stride, ...; 16-byte copies when rows are 16-byte aligned.
  // No commit.
  const bool vec4 = g.vec4 != 0;
  const int t0 = a.t0, nT = a.nt;
  auto issue = [&](int it, int first, int stride) {
    const int s = t0 + nT - 1 - it;
    float* dst = ring + (it % pd) * ring_stride;
    const int w = vec4 ? 4 : 1;
    const int hw = hcnt / w, n = nb * 6 * hw;
    for (int e = first; e < n; e += stride) {
      const int r = e / hw, jl = w * (e - r * hw);
      const int b = r / 6, q = r - 6 * b;
      const size_t row = (size_t)(b_begin + b) * T + s;
      float* d = dst + r * Hc + jl;
      const float* src = q == 0 ? (a.dout ? a.dout + row * H + j0 + jl : nullptr)
                                : a.stash + row * 5 * H + (q - 1) * H + j0 + jl;
      if (src == nullptr) {
        for (int v = 0; v < w; ++v) d[v] = 0.0f;
      } else if (vec4) {
        cp_async16(d, src);
      } else {
        cp_async4(d, src);
      }
    }
  };
  for (int it = 0; it < pd - 1; ++it) {
    if (it < nT) issue(it, tid, nthr);
    cp_async_commit();
  }
  // Per-thread plan of the time loop's prefetch copies (as in the forward).
  // Entry k: inputs q0 .. q0 + cpe - 1 of row b, units jl .. jl + w - 1, to
  // ring offsets plan_dst[k] + q * Hc; input 0 (dout) comes from
  // dout_c + s * H + plan_offd[k], input q >= 1 from
  // stash_c + s * 5H + plan_offs[k] + (q - 1) * H.  cpe is 1, 2, 3 or 6: the
  // smallest that keeps every thread at kPlanItems entries or fewer.
  const int ns_last = nb - ((nb - 1) / R) * R;
  const int nact_last = ns_last * hcnt;
  const bool idle_issue = nact_last < nthr;
  const int pfirst = idle_issue ? tid - nact_last : tid, pstride = idle_issue ? nthr - nact_last : nthr;
  int plan_n = 0, cpe = 1, plan_q0[kPlanItems];
  int plan_dst[kPlanItems], plan_offd[kPlanItems], plan_offs[kPlanItems];
  const float* const dout_c = a.dout ? a.dout + (size_t)b_begin * T * H + j0 : nullptr;
  const float* const stash_c = a.stash + (size_t)b_begin * T * 5 * H + j0;
  {
    const int w = vec4 ? 4 : 1;
    const int hw = hcnt / w;
#pragma unroll
    for (int k = 0; k < kPlanItems; ++k) plan_dst[k] = plan_offd[k] = plan_offs[k] = plan_q0[k] = 0;
    while (cpe < 6 && nb * (6 / cpe) * hw > kPlanItems * pstride) cpe = cpe == 1 ? 2 : (cpe == 2 ? 3 : 6);
    const int per = 6 / cpe, n = nb * per * hw;
    // same rule as the forward: a CTA-uniform decision
    if (a.dout == nullptr || kPlanItems * pstride < n || (size_t)nb * T * 5 * H >= (1ull << 31)) plan_n = -1;
    if (pfirst >= 0 && plan_n == 0) {
#pragma unroll
      for (int k = 0; k < kPlanItems; ++k) {
        const int e = pfirst + k * pstride;
        if (e < n) {
          const int r = e / hw, jl = w * (e - r * hw);
          const int b = r / per, q0 = (r - per * b) * cpe;
          plan_q0[k] = q0;
          plan_dst[k] = (b * 6 + q0) * Hc + jl;
          plan_offd[k] = b * T * H + jl;
          plan_offs[k] = b * T * 5 * H + jl;
          plan_n = k + 1;
        }
      }
    }
  }
  auto issue_step = [&](int it) {
    if (plan_n < 0) {
      issue(it, pfirst, pstride);
      return;
    }
    const int s = t0 + nT - 1 - it;
    float* dst = ring + (it % pd) * ring_stride;
    const float* src_d = dout_c + (size_t)s * H;
    const float* src_s = stash_c + (size_t)s * 5 * H;
#pragma unroll
    for (int k = 0; k < kPlanItems; ++k) {
      if (k < plan_n) {
        float* d = dst + plan_dst[k];
        for (int c = 0; c < cpe; ++c) {
          const int q = plan_q0[k] + c;
          const float* src = q == 0 ? src_d + plan_offd[k] : src_s + plan_offs[k] + (q - 1) * H;
          if (vec4)
            cp_async16(d + c * Hc, src);
          else
            cp_async4(d + c * Hc, src);
        }
      }
    }
  };

  const int kown = (ksend < H) ? ksend / Hc : 0;
  const int kl = (ksend < H) ? ksend - kown * Hc : 0;
  // This thread's partial for row b of slot s lands in red[s][c][b][kl] of
  // CTA kown and completes bytes on that CTA's mbarrier s.
  const uint32_t dst_base = mapa_u32(smem_u32(red) + 4u * (uint32_t)(c * bcp * Hc + kl), kown);
  const uint32_t dst_bar0 = mapa_u32(bar0, kown);
  cluster.sync();

  bool ok = true;
  for (int it = 0; it < nT; ++it) {
    const int t = t0 + nT - 1 - it;
    const float* rg = ring + (it % pd) * ring_stride;
    const int rslot = (it + 1) & 1;  // partials written at iteration it-1
    const float* rin = red + rslot * red_slot;
    const int wslot = it & 1;
    GRU_TL(1, 0);
    // This thread's ring copies for iteration it (visible to all after the
    // barrier below); waited for before the partials, whose wait absorbs it.
    cp_async_wait_dyn(pd - 2);
    GRU_TL(1, 1);
    // After an expired wait (recorded in the status word) this thread stops
    // waiting but still runs every remaining barrier; results are then invalid.
    if (it > 0 && ok) ok = mbar_wait_bounded(bar0 + 8 * rslot, phase_parity(it));
    GRU_TL(1, 2);

    for (int b0 = 0; b0 < nb; b0 += R) {
      __syncthreads();
      if (b0 == 0) GRU_TL(1, 3);
      const int ns = min(R, nb - b0);
      // Threads without a pointwise item in the last sub-chunk issue the
      // prefetch for iteration it+pd-1 meanwhile (it overwrites ring slot
      // (it-1) % pd: past this iteration's wait every CTA has sent its
      // iteration it-1 partials, which follow (barrier) its reads of the slot).
      const int nact = ns * hcnt;
      if (b0 + R >= nb && idle_issue && tid >= nact && it + pd - 1 < nT) issue_step(it + pd - 1);
      for (int e = tid; e < ns * hcnt; e += nthr) {
        const int s = e == tid ? my_s : e / hcnt, jl = e == tid ? my_jl : e - s * hcnt;
        const int b = b0 + s, j = j0 + jl;
        float dh;
        if (it == 0) {
          dh = (a.dhn != nullptr) ? a.dhn[(size_t)(b_begin + b) * H + j] : 0.0f;
        } else {
          float pp[kMaxCluster];
#pragma unroll
          for (int q = 0; q < kMaxCluster; ++q) pp[q] = q < C ? rin[(q * bcp + b) * Hc + jl] : 0.0f;
          dh = gz[b * Hc + jl];
#pragma unroll
          for (int q = 0; q < kMaxCluster; ++q) dh += pp[q];
        }
        if (e == tid && b0 == 0) GRU_TL(1, 4);
        const float* v = rg + (b * 6) * Hc + jl;
        const float gg = dh + v[0];
        const float r = v[Hc], z = v[2 * Hc], n = v[3 * Hc], hn = v[4 * Hc], hp = v[5 * Hc];
        const float dz = gg * (hp - n);
        const float dn = gg * (1.0f - z);
        const float dn_pre = dn * (1.0f - n * n);
        const float dr = dn_pre * hn;
        const float dhn_gate = dn_pre * r;
        const float dr_pre = dr * r * (1.0f - r);
        const float dz_pre = dz * z * (1.0f - z);
        dgs[(s * 3 + 0) * 32 + jl] = dr_pre;
        dgs[(s * 3 + 1) * 32 + jl] = dz_pre;
        dgs[(s * 3 + 2) * 32 + jl] = dhn_gate;
        gz[b * Hc + jl] = gg * z;
        if (e == tid && b0 == 0) GRU_TL(1, 5);
        const size_t row = (size_t)(b_begin + b) * T + t;
        const size_t o = row * a.ldgi + j, on = row * a.ldgn + j;
        split_store(a.dGi + o, a.dGi_lo + o, dr_pre);
        split_store(a.dGi + o + H, a.dGi_lo + o + H, dz_pre);
        split_store(a.dGi + o + 2 * H, a.dGi_lo + o + 2 * H, dn_pre);
        split_store(a.dGh + on, a.dGh_lo + on, dhn_gate);
        if (e == tid && b0 == 0) GRU_TL(1, 6);
        double* acc = dbacc + (s * 4) * Hc + jl;
        acc[0] += (double)dr_pre;
        acc[Hc] += (double)dz_pre;
        acc[2 * Hc] += (double)dn_pre;
        acc[3 * Hc] += (double)dhn_gate;
        if (e == tid && b0 == 0) GRU_TL(1, 7);
      }
      __syncthreads();
      if (b0 == 0) GRU_TL(1, 8);
      // Every thread has consumed slot `rslot`: re-arm it for iteration it+2
      // (iteration T is the final dh0 read below).
      if (b0 == 0 && tid == 0 && it > 0 && it + 2 <= nT) mbar_expect_tx(bar0 + 8 * rslot, bytes_per_step);
      if (b0 == 0 && tid == 0 && it == 0 && nT >= 2) mbar_expect_tx(bar0 + 8, bytes_per_step);

      {
        const uint32_t dst = dst_base + 4u * (uint32_t)(wslot * red_slot + b0 * Hc);
        const uint32_t dbar = dst_bar0 + 8u * wslot;
        float2 acc[R][3];  // (column k0, column k0 + 1) partials per gate
#pragma unroll
        for (int s = 0; s < R; ++s) acc[s][0] = acc[s][1] = acc[s][2] = make_float2(0.f, 0.f);
#pragma unroll
        for (int jj = 0; jj < 16; jj += 4) {
#pragma unroll
          for (int s = 0; s < R; ++s) {
            const float* d = dgs + s * 3 * 32 + 16 * jh + jj;
            const float4 vr = *reinterpret_cast<const float4*>(d);
            const float4 vz = *reinterpret_cast<const float4*>(d + 32);
            const float4 vn = *reinterpret_cast<const float4*>(d + 64);
            acc[s][0] = __ffma2_rn(make_float2(vr.x, vr.x), wr[jj], acc[s][0]);
            acc[s][1] = __ffma2_rn(make_float2(vz.x, vz.x), wz[jj], acc[s][1]);
            acc[s][2] = __ffma2_rn(make_float2(vn.x, vn.x), wn[jj], acc[s][2]);
            acc[s][0] = __ffma2_rn(make_float2(vr.y, vr.y), wr[jj + 1], acc[s][0]);
            acc[s][1] = __ffma2_rn(make_float2(vz.y, vz.y), wz[jj + 1], acc[s][1]);
            acc[s][2] = __ffma2_rn(make_float2(vn.y, vn.y), wn[jj + 1], acc[s][2]);
            acc[s][0] = __ffma2_rn(make_float2(vr.z, vr.z), wr[jj + 2], acc[s][0]);
            acc[s][1] = __ffma2_rn(make_float2(vz.z, vz.z), wz[jj + 2], acc[s][1]);
            acc[s][2] = __ffma2_rn(make_float2(vn.z, vn.z), wn[jj + 2], acc[s][2]);
            acc[s][0] = __ffma2_rn(make_float2(vr.w, vr.w), wr[jj + 3], acc[s][0]);
            acc[s][1] = __ffma2_rn(make_float2(vz.w, vz.w), wz[jj + 3], acc[s][1]);
            acc[s][2] = __ffma2_rn(make_float2(vn.w, vn.w), wn[jj + 3], acc[s][2]);
          }
        }
        if (b0 == 0) GRU_TL(1, 9);
#pragma unroll
        for (int s = 0; s < R; ++s) {
          // this half's sums for columns k0 and k0+1; the other half (lane ^ 16)
          // holds the rest of the same two columns
          const float c0 = acc[s][0].x + acc[s][1].x + acc[s][2].x;
          const float c1 = acc[s][0].y + acc[s][1].y + acc[s][2].y;
          const float o0 = __shfl_xor_sync(0xffffffffu, c0, 16);
          const float o1 = __shfl_xor_sync(0xffffffffu, c1, 16);
          const float v = jh == 0 ? c0 + o0 : o1 + c1;  // column ksend = k0 + jh
          if (s < ns && ksend < H) st_async_f32(dst + 4u * (uint32_t)(s * Hc), v, dbar);
        }
        if (b0 == 0) GRU_TL(1, 10);
      }
    }
    // Every thread had a pointwise item: prefetch now, after the sends.
    if (!idle_issue && it + pd - 1 < nT) issue_step(it + pd - 1);
    cp_async_commit();
    GRU_TL(1, 11);
  }
  GRU_TL_FLUSH(1);

  // dh0 = g*z of the last iteration (t = t0) plus every CTA's partial product of
  // that iteration, which arrive in slot (nt+1)&1.
  if (ok && nT > 0) {
    const int rslot = (nT + 1) & 1;
    ok = mbar_wait_bounded(bar0 + 8 * rslot, phase_parity(nT));
    if (ok) {
      const float* rin = red + rslot * red_slot;
      for (int e = tid; e < nb * hcnt; e += nthr) {
        const int b = e / hcnt, jl = e - b * hcnt;
        float dh = gz[b * Hc + jl];
        for (int q = 0; q < C; ++q) dh += rin[(q * bcp + b) * Hc + jl];
        a.dh0[(size_t)(b_begin + b) * H + j0 + jl] = dh;
      }
    }
  }
  // This cluster's bias-gradient partials: the sub-chunk rows' sums added in
  // a fixed order (deterministic), this CTA's units of the four blocks.
  __syncthreads();
  for (int e = tid; e < 4 * hcnt; e += nthr) {
    const int q = e / hcnt, jl = e - q * hcnt;
    double sum = 0.0;
    for (int s = 0; s < R; ++s) sum += dbacc[(s * 4 + q) * Hc + jl];
    a.dbpart[(size_t)cid * 4 * H + q * H + j0 + jl] = sum;
  }
  cp_async_wait<0>();
  cluster.sync();
}

// ---------------------------------------------------------------------------
// Small hidden sizes (H <= 96): one CTA per group of up to NR batch rows, no
// cluster.  With H <= 96 the whole W_hh (3H x H <= 27,648 floats) fits in the
// registers of one CTA of 32 * ceil(H/8) threads, so a step needs no
// distributed shared memory exchange and no mbarrier: h (forward) or the
// dh partials (backward) pass through this CTA's shared memory and one
// __syncthreads per step.  The cluster kernels above keep a 32-unit slice of
// W_hh per CTA and pay a cross-CTA exchange and cross-warp partial sums every
// step, which at H <= 96 (one or two batch rows per cluster) left them
// latency-bound at ~1,700 cycles per step whatever the work.
//
// Mapping: warp w owns units j in [8w, 8w + 8); lane l = 8 ks + u works on
// unit j = 8w + u and on the K slice [ks KS, ks KS + KS) (4 slices cover
// K <= 4 KS), holding W_hh[g H + j][slice] for the three gates g (3 KS floats).
// Forward: the lane's partial dot products for every batch row are summed
// over the four slices with two xor shuffles (8, 16), so every lane of unit j
// has the complete r/z/n sums; lane ks then does the gate math of batch row
// ks.  Backward: lane (ks, u) computes dG for (row ks, unit j); each lane
// gets dG of its unit for every row by shuffles, forms dG . W_hh over its
// K slice, the warp reduce-scatters that over its 8 units (xor 4, 2, 1: lane
// u keeps KS/8 columns), and the warps' partial rows meet in shared memory.
// Per-step inputs (the input gates; dout and the stash) are loaded by the
// lane that uses them, two steps ahead, into registers (the time loop is
// unrolled by two so the two register sets have fixed names): a load is
// issued once its register set has been consumed and is waited for two
// steps later.  A step timeline (clock64 markers, H = 64) showed the earlier
// prefetch with 4-byte cp.async into a shared ring costing 250-400 cycles of
// issue per step wherever it was placed and however few instructions it
// took, and bulk copies (cp.async.bulk) issued by an extra I/O warp through
// mbarriers costing more (150-200 cycles per copy to issue, plus the proxy
// fence and hand-off); the register loads cut the step from 1,250 to 950
// cycles (forward) and from 1,700 to 1,220 (backward).
//
// Measured at T = 256, B = 64 (one launch each, CUDA events): forward
// 0.107 / 0.130 / 0.168 ms at H = 32 / 64 / 96 against the cluster kernel's
// 0.234 / 0.199 / 0.216 ms; backward 0.128 / 0.169 ms at H = 32 / 64 against
// 0.267 / 0.208 ms, but 0.252 against 0.230 ms at H = 96 (the dh partial
// rows of 12 warps and the 24-column reduce-scatter), so the backward uses
// these kernels for H <= 64 only.
// ---------------------------------------------------------------------------
constexpr int kSmallMaxH = 96;     // forward
constexpr int kSmallMaxHBwd = 64;  // backward
constexpr int kSmallThreads = 32 * (kSmallMaxH / 8);  // 12 warps at H = 96

// Row pitch (floats) of the shared h / partial / ring rows: 4 KS padded by 8 so
// that the four row groups (lanes 8 ks .. 8 ks + 7) of a warp fall in
// different banks.
template <int KS>
constexpr int small_pitch() { return 4 * KS + 8; }

template <int KS, int NR>
__global__ void __launch_bounds__(kSmallThreads, 1)
gru_fwd_small_kernel(FwdArgs a, RecGeom g) {
  constexpr int KP = small_pitch<KS>();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ks = lane >> 3, u = lane & 7;
  const int H = g.H, T = g.T;
  const int j = warp * 8 + u;
  const bool jv = j < H;
  const int b_begin = blockIdx.x * g.bc;
  const int nb = min(g.bc, g.B - b_begin);
  const bool act = jv && ks < nb;  // this lane does the gate math of (row ks, unit j)
  const int ldg = (3 * H + 3) & ~3;
  const int t0 = a.t0, nT = a.nt;

  extern __shared__ __align__(16) float smem[];
  float* hs = smem;  // [2][NR][KP]
  GRU_TL_INIT

  float2 w[3][KS / 2];
#pragma unroll
  for (int q = 0; q < 3; ++q)
#pragma unroll
    for (int i = 0; i < KS / 2; ++i) {
      const int k = ks * KS + 2 * i;
      const float* row = a.w_hh + (size_t)(q * H + j) * H;
      w[q][i] = make_float2(jv && k < H ? row[k] : 0.f, jv && k + 1 < H ? row[k + 1] : 0.f);
    }
  float bh[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) bh[q] = jv ? a.b_hh[q * H + j] : 0.f;

  for (int e = tid; e < 2 * NR * KP; e += blockDim.x) {
    const int b = (e / KP) % NR, k = e % KP;
    hs[e] = (e < NR * KP && b < nb && k < H) ? a.h0[(size_t)(b_begin + b) * H + k] : 0.f;
  }
  // This lane's input gates of step s (launch-relative), loaded two steps
  // ahead into registers (the loop is unrolled by two so the two register
  // sets have fixed names).
  const float* gsrc = a.G + ((size_t)(b_begin + (act ? ks : 0)) * T + t0) * ldg + j;
  auto load = [&](float (&d)[3], int s) {
    if (act && s < nT) {
      const float* p = gsrc + (size_t)s * ldg;
      d[0] = p[0];
      d[1] = p[H];
      d[2] = p[2 * H];
    }
  };
  float ga[3] = {0.f, 0.f, 0.f}, gb[3] = {0.f, 0.f, 0.f};
  load(ga, 0);
  load(gb, 1);
  __syncthreads();

  auto step = [&](int it, const float (&gi)[3]) {
    const int t = t0 + it;
    const float* hc = hs + (it & 1) * NR * KP;
    float* hx = hs + ((it + 1) & 1) * NR * KP;
    GRU_TL(0, 0);
    float s3[NR][3];
#pragma unroll
    for (int b = 0; b < NR; ++b) {
      float2 acc[3] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float4* h4 = reinterpret_cast<const float4*>(hc + b * KP + ks * KS);
#pragma unroll
      for (int i = 0; i < KS / 4; ++i) {
        const float4 hv = h4[i];
        const float2 h01 = make_float2(hv.x, hv.y), h23 = make_float2(hv.z, hv.w);
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          acc[q] = __ffma2_rn(w[q][2 * i], h01, acc[q]);
          acc[q] = __ffma2_rn(w[q][2 * i + 1], h23, acc[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < 3; ++q) s3[b][q] = acc[q].x + acc[q].y;
    }
    GRU_TL(0, 2);
    // sum over the four K slices: every lane of unit j gets the full sums
#pragma unroll
    for (int b = 0; b < NR; ++b)
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        s3[b][q] += __shfl_xor_sync(0xffffffffu, s3[b][q], 8);
        s3[b][q] += __shfl_xor_sync(0xffffffffu, s3[b][q], 16);
      }
    GRU_TL(0, 4);
    if (act) {
      float sr = s3[0][0], sz = s3[0][1], sn = s3[0][2];
#pragma unroll
      for (int b = 1; b < NR; ++b)
        if (ks == b) sr = s3[b][0], sz = s3[b][1], sn = s3[b][2];
      const float ar = bh[0] + sr, az = bh[1] + sz, an = bh[2] + sn;
      const float r = sigmoidf_acc(gi[0] + ar);
      const float z = sigmoidf_acc(gi[1] + az);
      const float n = tanhf(gi[2] + r * an);
      const float hp = hc[ks * KP + j];
      const float hnew = n + z * (hp - n);
      GRU_TL(0, 5);
      hx[ks * KP + j] = hnew;
      const size_t row = (size_t)(b_begin + ks) * T + t;
      a.out[row * H + j] = hnew;
      if (a.stash != nullptr) {
        float* st = a.stash + row * 5 * H + j;
        st[0] = r;
        st[H] = z;
        st[2 * H] = n;
        st[3 * H] = an;
        st[4 * H] = hp;
      }
      if (it == nT - 1) a.hn[(size_t)(b_begin + ks) * H + j] = hnew;
      GRU_TL(0, 7);
    }
    __syncthreads();  // the new h is complete; the old one is no longer read
    GRU_TL(0, 3);
  };
  for (int it = 0; it < nT; it += 2) {
    step(it, ga);
    load(ga, it + 2);
    if (it + 1 < nT) {
      step(it + 1, gb);
      load(gb, it + 3);
    }
  }
  GRU_TL_FLUSH(0);
}

template <int KS, int NR>
__global__ void __launch_bounds__(kSmallThreads, 1)
gru_bwd_small_kernel(BwdArgs a, RecGeom g) {
  constexpr int KP = small_pitch<KS>();
  constexpr int KU = KS / 8;  // columns per lane after the reduce-scatter
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ks = lane >> 3, u = lane & 7;
  const int H = g.H, T = g.T, NW = g.nw;
  const int j = warp * 8 + u;
  const bool jv = j < H;
  const int cid = blockIdx.x;
  const int b_begin = cid * g.bc;
  const int nb = min(g.bc, g.B - b_begin);
  const bool act = jv && ks < nb;  // this lane does the pointwise of (row ks, unit j)
  const int t0 = a.t0, nT = a.nt;

  extern __shared__ __align__(16) float smem[];
  float* part = smem;  // [2][NW][NR][KP] per-warp partial rows of dh
  GRU_TL_INIT

  float2 w[3][KS / 2];
#pragma unroll
  for (int q = 0; q < 3; ++q)
#pragma unroll
    for (int i = 0; i < KS / 2; ++i) {
      const int k = ks * KS + 2 * i;
      const float* row = a.w_hh + (size_t)(q * H + j) * H;
      w[q][i] = make_float2(jv && k < H ? row[k] : 0.f, jv && k + 1 < H ? row[k + 1] : 0.f);
    }

  // This lane's inputs of iteration s (walking t0 + nT - 1 down to t0),
  // loaded two iterations ahead into registers: 0 dout, 1 r, 2 z, 3 n,
  // 4 hn (= W_hn.h + b_hn), 5 h_prev.
  const size_t row0 = (size_t)(b_begin + (act ? ks : 0)) * T;
  auto load = [&](float (&d)[6], int s) {
    if (act && s < nT) {
      const size_t row = row0 + t0 + nT - 1 - s;
      d[0] = a.dout != nullptr ? a.dout[row * H + j] : 0.f;
      const float* st = a.stash + row * 5 * H + j;
#pragma unroll
      for (int q = 0; q < 5; ++q) d[q + 1] = st[q * H];
    }
  };
  float va[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, vb[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  load(va, 0);
  load(vb, 1);
  __syncthreads();

  float gz = 0.f;  // g * z of the previous iteration for (row ks, unit j)
  double db0 = 0.0, db1 = 0.0, db2 = 0.0, db3 = 0.0;
  auto step = [&](int it, const float (&v)[6]) {
    const int t = t0 + nT - 1 - it;
    GRU_TL(1, 0);
    float e0 = 0.f, e1 = 0.f, e2 = 0.f;  // dr_pre, dz_pre, dhn_gate of (row ks, unit j)
    if (act) {
      float dh;
      if (it == 0) {
        dh = (a.dhn != nullptr) ? a.dhn[(size_t)(b_begin + ks) * H + j] : 0.f;
      } else {
        const float* pr = part + ((it - 1) & 1) * NW * NR * KP + ks * KP + j;
        dh = gz;
        for (int q = 0; q < NW; ++q) dh += pr[q * NR * KP];
      }
      GRU_TL(1, 4);
      const float gg = dh + v[0];
      const float r = v[1], z = v[2], n = v[3], hn = v[4], hp = v[5];
      const float dz = gg * (hp - n);
      const float dn = gg * (1.0f - z);
      const float dn_pre = dn * (1.0f - n * n);
      const float dr = dn_pre * hn;
      e2 = dn_pre * r;
      e0 = dr * r * (1.0f - r);
      e1 = dz * z * (1.0f - z);
      gz = gg * z;
      GRU_TL(1, 5);
      const size_t row = (size_t)(b_begin + ks) * T + t;
      const size_t o = row * a.ldgi + j, on = row * a.ldgn + j;
      split_store(a.dGi + o, a.dGi_lo + o, e0);
      split_store(a.dGi + o + H, a.dGi_lo + o + H, e1);
      split_store(a.dGi + o + 2 * H, a.dGi_lo + o + 2 * H, dn_pre);
      split_store(a.dGh + on, a.dGh_lo + on, e2);
      db0 += (double)e0;
      db1 += (double)e1;
      db2 += (double)dn_pre;
      db3 += (double)e2;
      GRU_TL(1, 7);
    }
    // dh_{t-1} partial of this warp's units: for every row b, the lane of
    // (row b, unit j) hands over its dG; this lane multiplies it into its K
    // slice and the warp reduce-scatters over its 8 units.
    float* pw = part + (it & 1) * NW * NR * KP + warp * NR * KP + ks * KS + u * KU;
#pragma unroll
    for (int b = 0; b < NR; ++b) {
      const int src = (b << 3) | u;
      const float f0 = __shfl_sync(0xffffffffu, e0, src);
      const float f1 = __shfl_sync(0xffffffffu, e1, src);
      const float f2 = __shfl_sync(0xffffffffu, e2, src);
      float c[KS];
#pragma unroll
      for (int i = 0; i < KS / 2; ++i) {
        float2 p = __fmul2_rn(make_float2(f2, f2), w[2][i]);
        p = __ffma2_rn(make_float2(f1, f1), w[1][i], p);
        p = __ffma2_rn(make_float2(f0, f0), w[0][i], p);
        c[2 * i] = p.x;
        c[2 * i + 1] = p.y;
      }
      // reduce-scatter over lanes u (xor 4, 2, 1): lane u keeps columns
      // [u KU, u KU + KU) of its slice
#pragma unroll
      for (int m = 4, half = KS / 2; m >= 1; m >>= 1, half >>= 1) {
        const bool up = (u & m) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = up ? c[i] : c[i + half];
          const float keep = up ? c[i + half] : c[i];
          c[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
      }
#pragma unroll
      for (int i = 0; i < KU; ++i) pw[b * KP + i] = c[i];
    }
    GRU_TL(1, 9);
    __syncthreads();  // this iteration's partial rows complete
    GRU_TL(1, 8);
  };
  for (int it = 0; it < nT; it += 2) {
    step(it, va);
    load(va, it + 2);
    if (it + 1 < nT) {
      step(it + 1, vb);
      load(vb, it + 3);
    }
  }
  GRU_TL_FLUSH(1);
  if (act && nT > 0) {
    const float* pr = part + ((nT - 1) & 1) * NW * NR * KP + ks * KP + j;
    float dh = gz;
    for (int q = 0; q < NW; ++q) dh += pr[q * NR * KP];
    a.dh0[(size_t)(b_begin + ks) * H + j] = dh;
  }
  // this CTA's bias-gradient partials: the rows' sums in a fixed order
#pragma unroll
  for (int m = 8; m <= 16; m <<= 1) {
    db0 += __shfl_xor_sync(0xffffffffu, db0, m);
    db1 += __shfl_xor_sync(0xffffffffu, db1, m);
    db2 += __shfl_xor_sync(0xffffffffu, db2, m);
    db3 += __shfl_xor_sync(0xffffffffu, db3, m);
  }
  if (ks == 0 && jv) {
    double* dp = a.dbpart + (size_t)cid * 4 * H + j;
    dp[0] = db0;
    dp[H] = db1;
    dp[2 * H] = db2;
    dp[3 * H] = db3;
  }
}

int base_geometry(int B, int T, int H, RecGeom* g) {
  g->B = B;
  g->T = T;
  g->H = H;
  g->C = ceil_div(H, 32);
  g->Hc = ceil_div(H, g->C);
  g->nw = g->C;
  g->vec4 = (H % 4 == 0 && g->Hc % 4 == 0) ? 1 : 0;
  return GRU_OK;
}

inline int round4(size_t v) { return (int)((v + 3) / 4 * 4); }

// Lay out the forward kernel's shared memory in g (offsets) and return its size.
size_t fwd_smem(RecGeom& g) {
  const int Kp = g.nw * 32;
  g.off1 = round4((size_t)2 * g.bcp * Kp);
  g.off2 = g.off1 + round4((size_t)g.R * 3 * 32 * 8);
  g.off3 = g.off2 + round4((size_t)g.pd * g.bcp * 3 * g.Hc);
  return sizeof(float) * (size_t)(g.off3 + round4((size_t)3 * g.Hc));
}
size_t bwd_smem(RecGeom& g) {
  g.off1 = round4((size_t)2 * g.C * g.bcp * g.Hc);
  g.off2 = g.off1 + round4((size_t)g.bcp * g.Hc);
  g.off3 = g.off2 + round4((size_t)g.R * 3 * 32);
  g.off4 = g.off3 + round4((size_t)g.pd * g.bcp * 6 * g.Hc);
  return sizeof(float) * (size_t)(g.off4 + (size_t)8 * g.R * g.Hc);  // + FP64 [R][4][Hc]
}

template <int R>
const void* fwd_kernel_ptr() { return (const void*)gru_fwd_recurrent_kernel<R>; }
template <int R>
const void* bwd_kernel_ptr() { return (const void*)gru_bwd_recurrent_kernel<R>; }

const void* kernel_for(bool fwd, int R) {
  switch (R) {
#define GRU_CASE(r) \
  case r: return fwd ? fwd_kernel_ptr<r>() : bwd_kernel_ptr<r>();
    GRU_CASE(1) GRU_CASE(2) GRU_CASE(3) GRU_CASE(4) GRU_CASE(5) GRU_CASE(6) GRU_CASE(7) GRU_CASE(8)
#undef GRU_CASE
    default: return nullptr;
  }
}

// Rows per sub-chunk for bc rows per cluster, hcnt units per CTA and nthr
// threads: at most kMaxRows, balanced across the sub-chunks (e.g. 5 + 4
// instead of 8 + 1 rows: every sub-chunk costs about one step's latency
// whatever its rows; I=H=256, B=128: both time loops 20 % faster) as long as
// the last sub-chunk leaves enough threads without a pointwise item: those
// threads issue the next steps' input prefetch, and too few of them made it
// the bottleneck (35 rows balanced as 5 x 7 at H=256: backward 14.5 ->
// 23.5 ms).  Enough = 64 for the forward (3 inputs per item), 128 for the
// backward (6 inputs; 18 rows as 3 x 6 with 64 idle: 4.2 -> 4.9 ms).
inline int rows_per_subchunk(int bc, int hcnt, int nthr, bool fwd) {
  if (bc <= kMaxRows) return bc;
  const int nsub = ceil_div(bc, kMaxRows);
  const int rb = ceil_div(bc, nsub);
  const int last = bc - (nsub - 1) * rb;
  return nthr - last * hcnt >= (fwd ? 64 : 128) ? rb : kMaxRows;
}

// Choose the batch rows per cluster: spread B over as many clusters as can be
// resident at once, subject to the shared-memory budget.
template <typename SmemFn>
int finish_geometry(RecGeom* g, int device, bool fwd, SmemFn smem_of) {
  static_assert(sizeof(float) == 4, "layout assumes 4-byte floats");
  int optin = 0;
  GRU_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  int max_smem = optin;  // dynamic budget = opt-in limit minus the kernel's static shared memory
  for (int r = 1; r <= kMaxRows; ++r) {
    cudaFuncAttributes fa{};
    GRU_CUDA_TRY(cudaFuncGetAttributes(&fa, kernel_for(fwd, r)));
    max_smem = std::min(max_smem, optin - (int)fa.sharedSizeBytes);
  }
  for (int r = 1; r <= kMaxRows; ++r)
    GRU_CUDA_TRY(cudaFuncSetAttribute(kernel_for(fwd, r), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      max_smem));

  // Cluster residency probe with a small configuration.
  g->pd = 3;
  g->R = kMaxRows;
  g->bc = kMaxRows;
  g->bcp = kMaxRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g->C, 1, 1);
  cfg.blockDim = dim3(32 * g->nw, 1, 1);
  cfg.dynamicSmemBytes = smem_of(*g);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = g->C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  GRU_CUDA_TRY(cudaOccupancyMaxActiveClusters(&max_clusters, kernel_for(fwd, kMaxRows), &cfg));
  if (max_clusters < 1) {
    set_error("no cluster of the recurrent kernel fits on this device");
    return GRU_ERR_UNSUPPORTED;
  }
  int bc = ceil_div(g->B, max_clusters);
  for (;;) {
    g->bc = bc;
    g->R = rows_per_subchunk(bc, g->Hc, 32 * g->nw, fwd);
    g->bcp = ceil_div(bc, g->R) * g->R;
    g->pd = kMaxPrefetch;  // prefetch issued at the end of step t for step t + pd - 1
    while (g->pd > 2 && smem_of(*g) > (size_t)max_smem) --g->pd;
    if (smem_of(*g) <= (size_t)max_smem) break;
    if (bc <= 1) {
      set_error("recurrent kernel shared memory does not fit");
      return GRU_ERR_UNSUPPORTED;
    }
    bc = bc > kMaxRows ? bc - kMaxRows : bc - 1;
  }
  g->nclusters = ceil_div(g->B, g->bc);
  if (g->nclusters > max_clusters) {
    // More than one wave: the last wave would be part-empty while every wave
    // costs as much as its widest cluster, so spread the rows evenly over
    // whole waves (narrower clusters, each step cheaper).
    const int waves = ceil_div(g->nclusters, max_clusters);
    g->bc = ceil_div(g->B, waves * max_clusters);
    g->R = rows_per_subchunk(g->bc, g->Hc, 32 * g->nw, fwd);
    g->bcp = ceil_div(g->bc, g->R) * g->R;
    g->pd = kMaxPrefetch;
    while (g->pd > 2 && smem_of(*g) > (size_t)max_smem) --g->pd;
    g->nclusters = ceil_div(g->B, g->bc);
  }
  g->smem = smem_of(*g);
  if ((g->off1 | g->off2 | g->off3 | g->off4) & 3) {
    set_error("internal: recurrent shared-memory region not 16-byte aligned");
    return GRU_ERR_INVALID;
  }
  g->max_clusters = max_clusters;
  return GRU_OK;
}

// Highest stream priority of the device (numerically smallest).  The time
// loops launch at this priority so that, when a tensor-core product on a side
// stream becomes ready at the same moment, the loop's clusters are placed
// first and the product takes the SMs they leave idle.
int top_priority() {
  static int prio = 1;
  if (prio == 1) {
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) {
      cudaGetLastError();
      greatest = 0;
    }
    prio = greatest;
  }
  return prio;
}

template <typename Args>
int launch_clusters(const void* kernel, const Args& a, const RecGeom& g, cudaStream_t stream, int kind) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.C * g.nclusters, 1, 1);
  cfg.blockDim = dim3(32 * g.nw, 1, 1);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = g.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributePriority;
  attr[1].val.priority = top_priority();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  Args args = a;
  RecGeom geom = g;
  void* params[2] = {&args, &geom};
  LaunchScope scope(kind, stream);
  GRU_CUDA_TRY(cudaLaunchKernelExC(&cfg, kernel, params));
  return GRU_OK;
}

}  // namespace

// Self-test of the bounded wait: one CTA waits on an mbarrier phase that
// nothing ever completes, with a limit of limit_ns, and must come back with
// the timeout recorded in the status word instead of hanging.
__global__ void wait_probe_kernel(unsigned long long limit_ns, int* result) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) mbar_init(b, 1);
  __syncthreads();
  const bool ok = mbar_wait_bounded(b, 0, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) *result = ok ? 1 : 0;
}

int wait_probe(unsigned long long limit_ns, int* result_dev, cudaStream_t stream) {
  LaunchScope scope(kKindFwdRecurrent, stream);
  wait_probe_kernel<<<1, 32, 0, stream>>>(limit_ns, result_dev);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

#ifdef GRU_TIMELINE
int read_timeline(long long* out) {
  GRU_CUDA_TRY(cudaDeviceSynchronize());
  GRU_CUDA_TRY(cudaMemcpyFromSymbol(out, g_tl, sizeof(g_tl)));
  return GRU_OK;
}
#endif

int read_device_status(int reset, int* status) {
  GRU_CUDA_TRY(cudaDeviceSynchronize());
  GRU_CUDA_TRY(cudaMemcpyFromSymbol(status, g_device_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    GRU_CUDA_TRY(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)));
  }
  return GRU_OK;
}

namespace {

template <int KS, int NR>
const void* small_ptr(bool fwd) {
  // the backward runs on these kernels for H <= 32 only (16-column K slices)
  // the backward runs on these kernels for H <= 64 only (16-column K slices)
  if constexpr (KS == 16) return fwd ? (const void*)gru_fwd_small_kernel<KS, NR> : (const void*)gru_bwd_small_kernel<KS, NR>;
  return fwd ? (const void*)gru_fwd_small_kernel<KS, NR> : nullptr;
}
const void* small_kernel_for(bool fwd, int H, int NR) {
  if (H <= 64) return NR == 1 ? small_ptr<16, 1>(fwd) : NR == 2 ? small_ptr<16, 2>(fwd) : small_ptr<16, 4>(fwd);
  return NR == 1 ? small_ptr<24, 1>(fwd) : NR == 2 ? small_ptr<24, 2>(fwd) : small_ptr<24, 4>(fwd);
}

// Dynamic shared memory of the small-H kernels (layouts in the kernels).
size_t small_smem(const RecGeom& g, bool fwd) {
  const size_t KP = g.H <= 64 ? 16 * 4 + 8 : 24 * 4 + 8;
  const size_t R = g.R;
  const size_t floats = fwd ? 2 * R * KP : 2 * g.nw * R * KP;
  return floats * sizeof(float);
}

// One CTA of 32 * ceil(H/8) threads per group of bc <= 4 batch rows: the
// rows spread over about one CTA per SM, then up to 4 rows per CTA.
int small_geometry(RecGeom* g, int device, bool fwd) {
  int sms = 0, optin = 0;
  GRU_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  GRU_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  g->small = 1;
  g->C = 1;
  g->Hc = g->H;
  g->nw = ceil_div(g->H, 8);
  g->vec4 = 0;
  const int bc = std::min(4, std::max(1, ceil_div(g->B, sms)));
  g->bc = bc;
  g->R = bc == 1 ? 1 : (bc == 2 ? 2 : 4);
  g->bcp = g->R;
  g->nclusters = ceil_div(g->B, bc);
  g->max_clusters = g->nclusters;
  g->off1 = g->off2 = g->off3 = g->off4 = 0;
  cudaFuncAttributes fa{};
  GRU_CUDA_TRY(cudaFuncGetAttributes(&fa, small_kernel_for(fwd, g->H, g->R)));
  const int budget = std::min(optin - (int)fa.sharedSizeBytes, 160 * 1024);
  g->pd = 2;  // inputs are loaded two steps ahead into registers
  g->smem = small_smem(*g, fwd);
  if (g->smem > (size_t)budget) {
    set_error("small-H time loop shared memory does not fit");
    return GRU_ERR_UNSUPPORTED;
  }
  GRU_CUDA_TRY(cudaFuncSetAttribute(small_kernel_for(fwd, g->H, g->R), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    budget));
  return GRU_OK;
}

std::atomic<int> g_small_loops{0};  // 0: automatic (H <= 96), 1: off

template <typename Args>
int launch_small(bool fwd, const Args& a, const RecGeom& g, cudaStream_t stream, int kind) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.nclusters, 1, 1);
  cfg.blockDim = dim3(32 * g.nw, 1, 1);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = top_priority();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Args args = a;
  RecGeom geom = g;
  void* params[2] = {&args, &geom};
  LaunchScope scope(kind, stream);
  GRU_CUDA_TRY(cudaLaunchKernelExC(&cfg, small_kernel_for(fwd, g.H, g.R), params));
  return GRU_OK;
}

}  // namespace

int set_small_loops(int mode) {
  if (mode < 0 || mode > 1) return -1;
  return g_small_loops.exchange(mode);
}
int small_loops_mode() { return g_small_loops.load(); }

int rec_forward_geometry(int B, int T, int H, int device, RecGeom* g) {
  base_geometry(B, T, H, g);
  if (H <= kSmallMaxH && g_small_loops.load() == 0) return small_geometry(g, device, true);
  return finish_geometry(g, device, true, fwd_smem);
}

int rec_backward_geometry(int B, int T, int H, int device, RecGeom* g) {
  base_geometry(B, T, H, g);
  if (H <= kSmallMaxHBwd && g_small_loops.load() == 0) return small_geometry(g, device, false);
  return finish_geometry(g, device, false, bwd_smem);
}

int launch_rec_forward(const float* G, int ldg, const float* h0, const float* w_hh, const float* b_hh,
                       float* out, float* hn, float* stash, const RecGeom& g,
                       cudaStream_t stream, int t0, int nt) {
  if (ldg != ((3 * g.H + 3) & ~3)) {
    set_error("internal: input-gate row stride must be 3H rounded up to 4");
    return GRU_ERR_INVALID;
  }
  if (nt < 0) nt = g.T;
  if (t0 < 0 || nt < 1 || t0 + nt > g.T) {
    set_error("internal: time window outside the sequence");
    return GRU_ERR_INVALID;
  }
  FwdArgs a{G, h0, w_hh, b_hh, out, hn, stash, t0, nt};
  RecGeom gg = g;
  if (reinterpret_cast<uintptr_t>(G) & 15) gg.vec4 = 0;  // 16-byte copies need an aligned base
  if (gg.small) return launch_small(true, a, gg, stream, kKindFwdRecurrent);
  return launch_clusters(kernel_for(true, gg.R), a, gg, stream, kKindFwdRecurrent);
}

int launch_rec_backward(const float* dout, const float* dhn, const float* w_hh,
                        const float* stash, float* dGi, float* dGi_lo, int ldgi, float* dGh, float* dGh_lo,
                        int ldgn, float* dh0, double* dbpart, const RecGeom& g, cudaStream_t stream, int t0,
                        int nt) {
  if (nt < 0) nt = g.T;
  if (t0 < 0 || nt < 1 || t0 + nt > g.T) {
    set_error("internal: time window outside the sequence");
    return GRU_ERR_INVALID;
  }
  BwdArgs a{dout, dhn, w_hh, stash, dGi, dGi_lo, ldgi, dGh, dGh_lo, ldgn, dh0, dbpart, t0, nt};
  RecGeom gg = g;
  if ((reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(stash)) & 15) gg.vec4 = 0;
  if (gg.small) return launch_small(false, a, gg, stream, kKindBwdRecurrent);
  return launch_clusters(kernel_for(false, gg.R), a, gg, stream, kKindBwdRecurrent);
}

}  // namespace gru

#ifdef GRU_TIMELINE
// Instrumented builds only: copies the step timeline (int64 clock64 values,
// [direction 2][CTA 0/1 x thread 0/last 4][step 8][point 12]) to out.
extern "C" int gru_timeline_read(long long* out) { return gru::read_timeline(out); }
#endif
