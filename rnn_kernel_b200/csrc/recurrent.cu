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
//   the gate math for its units, and writes the new h slice into the next
//   h buffer of every CTA of the cluster through distributed shared memory.
//   One cluster barrier per step; the h buffer is double-buffered.
// * Backward, per step: every CTA computes the pointwise backward for its
//   units, then its share of dh_{t-1} = dG_hh . W_hh over all k, and
//   reduce-scatters that partial into the owning CTAs' shared memory.  Again
//   one cluster barrier per step with double-buffered partials.
// * Per-step inputs (input gates; dout and the stash) are prefetched `pd`
//   steps ahead into a shared-memory ring with cp.async.
//
// Gate math follows custom_gru.py:117-122 / a100_gru_h256_kernels.cu:758-775
// (forward) and :852-866 (backward).

#include <cooperative_groups.h>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace cg = cooperative_groups;

namespace gru {

namespace {

__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gmem_src) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
  // n is 1 or 2 (prefetch depth - 1); wait_group needs an immediate.
  if (n >= 2) cp_async_wait<2>();
  else if (n == 1) cp_async_wait<1>();
  else cp_async_wait<0>();
}

__device__ __forceinline__ float sigmoidf_acc(float v) { return 1.0f / (1.0f + expf(-v)); }

struct FwdArgs {
  const float* G;     // [B,T,3H] input gates (x.W_ih^T + b_ih)
  const float* h0;    // [B,H]
  const float* w_hh;  // [3H,H]
  const float* b_hh;  // [3H]
  float* out;         // [B,T,H]
  float* hn;          // [B,H]
  float* stash;       // [B,T,5H] or null
};

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
  const int j0 = c * Hc;
  const int hcnt = max(0, min(Hc, H - j0));

  extern __shared__ __align__(16) float smem[];
  float* hbuf = smem;                              // [2][bcp][Kp]
  float* part = hbuf + 2 * bcp * Kp;               // [nw][kSub][3][32]
  float* ring = part + g.nw * kSub * 3 * 32;       // [pd][bcp][3][Hc]
  const int ring_stride = bcp * 3 * Hc;

  // W_hh rows (r, z, n) of unit j0+lane, columns [32*warp, 32*warp+32).
  float wr[32], wz[32], wn[32];
  {
    const int jg = j0 + lane;
    const bool jv = lane < hcnt;
#pragma unroll
    for (int kk = 0; kk < 32; ++kk) {
      const int k = warp * 32 + kk;
      const bool v = jv && k < H;
      wr[kk] = v ? a.w_hh[(size_t)jg * H + k] : 0.0f;
      wz[kk] = v ? a.w_hh[(size_t)(H + jg) * H + k] : 0.0f;
      wn[kk] = v ? a.w_hh[(size_t)(2 * H + jg) * H + k] : 0.0f;
    }
  }

  for (int e = tid; e < 2 * bcp * Kp; e += nthr) hbuf[e] = 0.0f;
  __syncthreads();
  for (int e = tid; e < nb * H; e += nthr) {
    const int b = e / H, k = e - b * H;
    hbuf[b * Kp + k] = a.h0[(size_t)(b_begin + b) * H + k];
  }

  auto issue = [&](int s) {
    float* dst = ring + (s % pd) * ring_stride;
    const int n = nb * 3 * hcnt;
    for (int e = tid; e < n; e += nthr) {
      const int jl = e % hcnt;
      const int r = e / hcnt;
      const int gi = r % 3, b = r / 3;
      cp_async4(dst + (b * 3 + gi) * Hc + jl,
                a.G + ((size_t)(b_begin + b) * T + s) * 3 * H + gi * H + j0 + jl);
    }
    cp_async_commit();
  };
  for (int s = 0; s < pd - 1; ++s) {
    if (s < T) issue(s);
    else cp_async_commit();
  }

  cluster.sync();  // h buffers of every CTA initialised before any remote write

  for (int t = 0; t < T; ++t) {
    if (t + pd - 1 < T) issue(t + pd - 1);
    else cp_async_commit();
    const int cur = t & 1, nxt = cur ^ 1;
    const float* hcur = hbuf + cur * bcp * Kp;
    const float* rg = ring + (t % pd) * ring_stride;

    for (int b0 = 0; b0 < nb; b0 += kSub) {
      float acc[kSub][3];
#pragma unroll
      for (int s = 0; s < kSub; ++s) acc[s][0] = acc[s][1] = acc[s][2] = 0.0f;
      const float* hb = hcur + b0 * Kp + warp * 32;
#pragma unroll
      for (int kk = 0; kk < 32; kk += 4) {
#pragma unroll
        for (int s = 0; s < kSub; ++s) {
          const float4 hv = *reinterpret_cast<const float4*>(hb + s * Kp + kk);
          acc[s][0] = fmaf(wr[kk], hv.x, acc[s][0]);
          acc[s][1] = fmaf(wz[kk], hv.x, acc[s][1]);
          acc[s][2] = fmaf(wn[kk], hv.x, acc[s][2]);
          acc[s][0] = fmaf(wr[kk + 1], hv.y, acc[s][0]);
          acc[s][1] = fmaf(wz[kk + 1], hv.y, acc[s][1]);
          acc[s][2] = fmaf(wn[kk + 1], hv.y, acc[s][2]);
          acc[s][0] = fmaf(wr[kk + 2], hv.z, acc[s][0]);
          acc[s][1] = fmaf(wz[kk + 2], hv.z, acc[s][1]);
          acc[s][2] = fmaf(wn[kk + 2], hv.z, acc[s][2]);
          acc[s][0] = fmaf(wr[kk + 3], hv.w, acc[s][0]);
          acc[s][1] = fmaf(wz[kk + 3], hv.w, acc[s][1]);
          acc[s][2] = fmaf(wn[kk + 3], hv.w, acc[s][2]);
        }
      }
#pragma unroll
      for (int s = 0; s < kSub; ++s) {
#pragma unroll
        for (int q = 0; q < 3; ++q) part[((warp * kSub + s) * 3 + q) * 32 + lane] = acc[s][q];
      }
      if (b0 == 0) cp_async_wait_dyn(pd - 1);
      __syncthreads();

      const int ns = min(kSub, nb - b0);
      for (int e = tid; e < ns * hcnt; e += nthr) {
        const int s = e / hcnt, jl = e - s * hcnt;
        const int b = b0 + s, j = j0 + jl;
        float ar = 0.0f, az = 0.0f, an = 0.0f;
        for (int w = 0; w < g.nw; ++w) {
          const float* p = part + ((w * kSub + s) * 3) * 32 + jl;
          ar += p[0];
          az += p[32];
          an += p[64];
        }
        ar += a.b_hh[j];
        az += a.b_hh[H + j];
        an += a.b_hh[2 * H + j];
        const float* gi = rg + (b * 3) * Hc + jl;
        const float r = sigmoidf_acc(gi[0] + ar);
        const float z = sigmoidf_acc(gi[Hc] + az);
        const float n = tanhf(gi[2 * Hc] + r * an);
        const float hp = hcur[b * Kp + j];
        const float hnew = n + z * (hp - n);
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
        if (t == T - 1) a.hn[(size_t)(b_begin + b) * H + j] = hnew;
        float* dst = hbuf + nxt * bcp * Kp + b * Kp + j;
        for (int q = 0; q < g.C; ++q) *cluster.map_shared_rank(dst, q) = hnew;
      }
      __syncthreads();
    }
    cluster.sync();
  }
}

struct BwdArgs {
  const float* dout;   // [B,T,H] or null
  const float* dhn;    // [B,H] or null
  const float* w_hh;   // [3H,H]
  const float* stash;  // [B,T,5H]
  float* dGi;          // [B,T,3H]
  float* dGh;          // [B,T,3H]
  float* dh0;          // [B,H]
};

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
  const int hcnt = max(0, min(Hc, H - j0));
  const int k = warp * 32 + lane;  // W_hh column this thread owns in the GEMV

  extern __shared__ __align__(16) float smem[];
  float* red = smem;                           // [2][C][bcp][Hc]
  float* gz = red + 2 * C * bcp * Hc;          // [bcp][Hc]
  float* dgs = gz + bcp * Hc;                  // [kSub][3][32]
  float* ring = dgs + kSub * 3 * 32;           // [pd][bcp][6][Hc]
  const int ring_stride = bcp * 6 * Hc;
  const int red_slot = C * bcp * Hc;

  // W_hh[g*H + j0 + j][k] for j < Hc.
  float wr[32], wz[32], wn[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const bool v = j < hcnt && k < H;
    wr[j] = v ? a.w_hh[(size_t)(j0 + j) * H + k] : 0.0f;
    wz[j] = v ? a.w_hh[(size_t)(H + j0 + j) * H + k] : 0.0f;
    wn[j] = v ? a.w_hh[(size_t)(2 * H + j0 + j) * H + k] : 0.0f;
  }

  for (int e = tid; e < 2 * red_slot; e += nthr) red[e] = 0.0f;
  for (int e = tid; e < bcp * Hc; e += nthr) gz[e] = 0.0f;
  for (int e = tid; e < kSub * 3 * 32; e += nthr) dgs[e] = 0.0f;

  // Ring entry q: 0 dout, 1 r, 2 z, 3 n, 4 hn (= W_hn.h + b_hn), 5 h_prev.
  auto issue = [&](int it) {
    const int s = T - 1 - it;
    float* dst = ring + (it % pd) * ring_stride;
    const int n = nb * 6 * hcnt;
    for (int e = tid; e < n; e += nthr) {
      const int jl = e % hcnt;
      const int r = e / hcnt;
      const int q = r % 6, b = r / 6;
      const size_t row = (size_t)(b_begin + b) * T + s;
      float* d = dst + (b * 6 + q) * Hc + jl;
      if (q == 0) {
        if (a.dout != nullptr) cp_async4(d, a.dout + row * H + j0 + jl);
        else *d = 0.0f;
      } else {
        cp_async4(d, a.stash + row * 5 * H + (q - 1) * H + j0 + jl);
      }
    }
    cp_async_commit();
  };
  for (int it = 0; it < pd - 1; ++it) {
    if (it < T) issue(it);
    else cp_async_commit();
  }

  const int kown = (k < H) ? k / Hc : 0;
  const int kl = (k < H) ? k - kown * Hc : 0;
  cluster.sync();

  for (int it = 0; it < T; ++it) {
    const int t = T - 1 - it;
    if (it + pd - 1 < T) issue(it + pd - 1);
    else cp_async_commit();
    const float* rg = ring + (it % pd) * ring_stride;
    const float* rin = red + ((t + 1) & 1) * red_slot;  // partials written at step t+1
    const int wslot = t & 1;

    for (int b0 = 0; b0 < nb; b0 += kSub) {
      if (b0 == 0) cp_async_wait_dyn(pd - 1);
      __syncthreads();
      const int ns = min(kSub, nb - b0);
      for (int e = tid; e < ns * hcnt; e += nthr) {
        const int s = e / hcnt, jl = e - s * hcnt;
        const int b = b0 + s, j = j0 + jl;
        float dh;
        if (it == 0) {
          dh = (a.dhn != nullptr) ? a.dhn[(size_t)(b_begin + b) * H + j] : 0.0f;
        } else {
          dh = gz[b * Hc + jl];
          for (int q = 0; q < C; ++q) dh += rin[(q * bcp + b) * Hc + jl];
        }
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
        const size_t row = (size_t)(b_begin + b) * T + t;
        float* gi = a.dGi + row * 3 * H + j;
        float* gh = a.dGh + row * 3 * H + j;
        gi[0] = dr_pre;
        gi[H] = dz_pre;
        gi[2 * H] = dn_pre;
        gh[0] = dr_pre;
        gh[H] = dz_pre;
        gh[2 * H] = dhn_gate;
        dgs[(s * 3 + 0) * 32 + jl] = dr_pre;
        dgs[(s * 3 + 1) * 32 + jl] = dz_pre;
        dgs[(s * 3 + 2) * 32 + jl] = dhn_gate;
        gz[b * Hc + jl] = gg * z;
      }
      __syncthreads();

      if (k < H) {
        float* dst = cluster.map_shared_rank(red + wslot * red_slot + (c * bcp + b0) * Hc + kl, kown);
#pragma unroll 1
        for (int s = 0; s < ns; ++s) {
          const float* d = dgs + s * 3 * 32;
          float xr = 0.0f, xz = 0.0f, xn = 0.0f;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 vr = *reinterpret_cast<const float4*>(d + j);
            const float4 vz = *reinterpret_cast<const float4*>(d + 32 + j);
            const float4 vn = *reinterpret_cast<const float4*>(d + 64 + j);
            xr = fmaf(vr.x, wr[j], xr); xz = fmaf(vz.x, wz[j], xz); xn = fmaf(vn.x, wn[j], xn);
            xr = fmaf(vr.y, wr[j + 1], xr); xz = fmaf(vz.y, wz[j + 1], xz); xn = fmaf(vn.y, wn[j + 1], xn);
            xr = fmaf(vr.z, wr[j + 2], xr); xz = fmaf(vz.z, wz[j + 2], xz); xn = fmaf(vn.z, wn[j + 2], xn);
            xr = fmaf(vr.w, wr[j + 3], xr); xz = fmaf(vz.w, wz[j + 3], xz); xn = fmaf(vn.w, wn[j + 3], xn);
          }
          dst[s * Hc] = xr + xz + xn;
        }
      }
    }
    cluster.sync();
  }

  // dh0 = direct term of step 0 + every CTA's partial written at step 0.
  const float* rin = red;  // slot (0 & 1)
  for (int e = tid; e < nb * hcnt; e += nthr) {
    const int b = e / hcnt, jl = e - b * hcnt;
    float dh = gz[b * Hc + jl];
    for (int q = 0; q < C; ++q) dh += rin[(q * bcp + b) * Hc + jl];
    a.dh0[(size_t)(b_begin + b) * H + j0 + jl] = dh;
  }
}

int base_geometry(int B, int T, int H, RecGeom* g) {
  g->B = B;
  g->T = T;
  g->H = H;
  g->C = ceil_div(H, 32);
  g->Hc = ceil_div(H, g->C);
  g->nw = g->C;
  return GRU_OK;
}

size_t fwd_smem(const RecGeom& g) {
  const int Kp = g.nw * 32;
  return sizeof(float) * ((size_t)2 * g.bcp * Kp + (size_t)g.nw * kSub * 3 * 32 +
                          (size_t)g.pd * g.bcp * 3 * g.Hc);
}
size_t bwd_smem(const RecGeom& g) {
  return sizeof(float) * ((size_t)2 * g.C * g.bcp * g.Hc + (size_t)g.bcp * g.Hc +
                          (size_t)kSub * 3 * 32 + (size_t)g.pd * g.bcp * 6 * g.Hc);
}

// Choose the batch rows per cluster: spread B over as many clusters as can be
// resident at once, subject to the shared-memory budget.
template <typename SmemFn>
int finish_geometry(RecGeom* g, int device, const void* kernel, SmemFn smem_of) {
  int max_smem = 0;
  GRU_CUDA_TRY(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  GRU_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem));

  // Probe cluster residency with a small configuration.
  g->pd = 3;
  g->bc = kSub;
  g->bcp = kSub;
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
  GRU_CUDA_TRY(cudaOccupancyMaxActiveClusters(&max_clusters, kernel, &cfg));
  if (max_clusters < 1) {
    set_error("no cluster of the recurrent kernel fits on this device");
    return GRU_ERR_UNSUPPORTED;
  }
  int bc = ceil_div(g->B, max_clusters);
  for (;;) {
    g->bc = bc;
    g->bcp = ceil_div(bc, kSub) * kSub;
    g->pd = 3;
    if (smem_of(*g) > (size_t)max_smem) g->pd = 2;
    if (smem_of(*g) <= (size_t)max_smem) break;
    if (bc <= 1) {
      set_error("recurrent kernel shared memory does not fit");
      return GRU_ERR_UNSUPPORTED;
    }
    bc = bc > kSub ? bc - kSub : bc - 1;
  }
  g->nclusters = ceil_div(g->B, g->bc);
  g->smem = smem_of(*g);
  return GRU_OK;
}

template <typename Args>
int launch_clusters(void (*kernel)(Args, RecGeom), const Args& a, const RecGeom& g,
                    cudaStream_t stream, int kind) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.C * g.nclusters, 1, 1);
  cfg.blockDim = dim3(32 * g.nw, 1, 1);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = g.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LaunchScope scope(kind, stream);
  GRU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, a, g));
  return GRU_OK;
}

}  // namespace

int rec_forward_geometry(int B, int T, int H, int device, RecGeom* g) {
  base_geometry(B, T, H, g);
  return finish_geometry(g, device, (const void*)gru_fwd_recurrent_kernel, fwd_smem);
}

int rec_backward_geometry(int B, int T, int H, int device, RecGeom* g) {
  base_geometry(B, T, H, g);
  return finish_geometry(g, device, (const void*)gru_bwd_recurrent_kernel, bwd_smem);
}

int launch_rec_forward(const float* G, const float* h0, const float* w_hh, const float* b_hh,
                       float* out, float* hn, float* stash, const RecGeom& g,
                       cudaStream_t stream) {
  FwdArgs a{G, h0, w_hh, b_hh, out, hn, stash};
  return launch_clusters(gru_fwd_recurrent_kernel, a, g, stream, kKindFwdRecurrent);
}

int launch_rec_backward(const float* dout, const float* dhn, const float* w_hh,
                        const float* stash, float* dGi, float* dGh, float* dh0,
                        const RecGeom& g, cudaStream_t stream) {
  BwdArgs a{dout, dhn, w_hh, stash, dGi, dGh, dh0};
  return launch_clusters(gru_bwd_recurrent_kernel, a, g, stream, kKindBwdRecurrent);
}

}  // namespace gru
