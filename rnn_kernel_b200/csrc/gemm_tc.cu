// FP32-accurate dense products on the 5th-generation tensor cores (sm_100a).
//
//   C[m, n] = sum_k A[m, k] * B[n, k] (+ bias[n])      A: [M, K], B: [N, K], both K-major
//
// used for the input projection G = x . W_ih^T + b_ih (prod/gru.py:519-523)
// and dx = dG_ih . W_ih (prod/gru.py:575).
//
// Precision: "3xTF32".  Each FP32 operand a is split into a_hi = tf32(a) and
// a_lo = tf32(a - a_hi) (round to nearest); the product is accumulated in FP32
// in tensor memory as a_lo*b_hi + a_hi*b_lo + a_hi*b_hi, which keeps about 21
// bits of every product -- FP32-level accuracy for the short K of these two
// products (K = I or 3H).
//
// Structure of one CTA (one 128 x BN output tile, 256 threads):
//   warp 0      TMA producer: FP32 tiles of A and B (128-byte swizzle) into a
//               `S`-deep shared-memory ring;
//   warp 1      allocates the tensor-memory accumulator; lane 0 issues the
//               tcgen05.mma instructions (3 per 8-wide K step) and commits
//               each stage back to the producer;
//   warps 2-7   split every landed stage in place into hi (rounded) + lo
//               (separate buffer) and hand it to the MMA issuer;
//   warps 4-7   epilogue: tcgen05.ld of the accumulator, + bias, stores.
// Every mbarrier wait is bounded; on expiry the kernel records
// GRU_STATUS_WAIT_TIMEOUT and winds down.

#include <cuda.h>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

__device__ int g_gemm_status = 0;

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;           // fp32 elements per 128-byte swizzle row
constexpr int kThreads = 256;
constexpr int kTransformThreads = 192;  // warps 2..7
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_gemm_status, GRU_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ uint32_t to_tf32(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte rows,
// 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);        // start address
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::tf32, D = F32, A = B = TF32, both K-major.
__host__ __device__ constexpr uint32_t tf32_idesc(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

template <int BN, int S>
struct Smem {
  static constexpr int kATile = kBM * kBK * 4;   // bytes
  static constexpr int kBTile = BN * kBK * 4;
  static constexpr int kStage = 2 * kATile + 2 * kBTile;  // A hi, A lo, B hi, B lo
  static constexpr int kBarOff = S * kStage;
  static constexpr int kBytes = kBarOff + 256 + 1024;  // + barriers + alignment slack
};

// NACC tensor-memory accumulators of BN columns each: with NACC = 4 the
// hi*hi products and the two cross products go to separate accumulators,
// alternating between two of each by K stage, and the epilogue adds them in
// FP32 (the tensor cores' own accumulation is less precise than an FP32
// add, so fewer additions into any one accumulator keep the sum closer to
// FP32 accuracy).
template <int BN, int S, int NACC>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   float* __restrict__ C, long ldc, const float* __restrict__ bias, int M, int N, int K) {
  using L = Smem<BN, S>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kBarOff;
  // barriers: full[S], ready[S], empty[S], accum; then the TMEM address slot
  auto full = [&](int s) { return bars + 8u * s; };
  auto ready = [&](int s) { return bars + 8u * (S + s); };
  auto empty = [&](int s) { return bars + 8u * (2 * S + s); };
  const uint32_t accum = bars + 8u * (3 * S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBarOff + 8 * (3 * S + 1));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = (N + BN - 1) / BN;
  const int m0 = (blockIdx.x / tiles_n) * kBM;
  const int n0 = (blockIdx.x % tiles_n) * BN;
  const int nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(ready(s), kTransformThreads);
      mbar_init(empty(s), 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN * NACC)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(empty(s), ((i / S) - 1) & 1)) break;
        const uint32_t st = sbase + s * L::kStage;
        mbar_arrive_expect_tx(full(s), L::kATile + L::kBTile);
        tma_load_2d(st, &map_a, full(s), i * kBK, m0);
        tma_load_2d(st + 2 * L::kATile, &map_b, full(s), i * kBK, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tf32_idesc(kBM, BN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        if (!mbar_wait(ready(s), (i / S) & 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t st = sbase + s * L::kStage;
        const uint32_t a_hi = st, a_lo = st + L::kATile, b_hi = st + 2 * L::kATile, b_lo = b_hi + L::kBTile;
        // Accumulators: [0, NACC/2) hold hi*hi, [NACC/2, NACC) the cross terms.
        const int half = NACC / 2;
        const uint32_t d_big = tmem + (uint32_t)(BN * (i % half));
        const uint32_t d_small = tmem + (uint32_t)(BN * (half + i % half));
        const uint32_t fresh = (i < half) ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along the swizzled row
          const uint32_t acc = (fresh && kk == 0) ? 0u : 1u;
          mma_tf32(d_small, sw128_desc(a_lo + off), sw128_desc(b_hi + off), idesc, acc);
          mma_tf32(d_small, sw128_desc(a_hi + off), sw128_desc(b_lo + off), idesc, 1u);
          mma_tf32(d_big, sw128_desc(a_hi + off), sw128_desc(b_hi + off), idesc, acc);
        }
        mma_commit(empty(s));
      }
      mma_commit(accum);
    }
  } else {
    // Transform warps 2..7: split each landed stage into hi (in place) + lo.
    const int tt = threadIdx.x - 64;
    constexpr int kA4 = L::kATile / 16, kB4 = L::kBTile / 16;  // float4 count per tile
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(full(s), (i / S) & 1)) break;
      float4* a = reinterpret_cast<float4*>(smem + s * L::kStage);
      float4* alo = a + kA4;
      float4* b = alo + kA4;
      float4* blo = b + kB4;
      for (int e = tt; e < kA4 + kB4; e += kTransformThreads) {
        float4* src = e < kA4 ? a + e : b + (e - kA4);
        float4* dlo = e < kA4 ? alo + e : blo + (e - kA4);
        const float4 v = *src;
        uint4 hi, lo;
        hi.x = to_tf32(v.x); hi.y = to_tf32(v.y); hi.z = to_tf32(v.z); hi.w = to_tf32(v.w);
        lo.x = to_tf32(v.x - __uint_as_float(hi.x));
        lo.y = to_tf32(v.y - __uint_as_float(hi.y));
        lo.z = to_tf32(v.z - __uint_as_float(hi.z));
        lo.w = to_tf32(v.w - __uint_as_float(hi.w));
        *reinterpret_cast<uint4*>(src) = hi;
        *reinterpret_cast<uint4*>(dlo) = lo;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(ready(s));
    }
    if (warp >= 4) {
      // Epilogue: this warp owns accumulator lanes 32*(warp%4) .. +32.
      const bool ok = mbar_wait(accum, 0);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row = m0 + 32 * (warp & 3) + lane;
      const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
      const int used = nk < NACC / 2 ? nk : NACC / 2;  // accumulator pairs written
      for (int c0 = 0; c0 < BN && ok; c0 += 16) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.0f;
        // cross terms first (small), then the hi*hi sums
        for (int q = NACC - 1; q >= 0; --q) {
          if ((q % (NACC / 2)) >= used) continue;
          uint32_t r[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
              : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
              : "r"(taddr + (uint32_t)(q * BN + c0)));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += __uint_as_float(r[j]);
        }
        if (row < M) {
          float* crow = C + (long)row * ldc;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + c0 + j;
            if (n < N) crow[n] = v[j] + (bias ? bias[n] : 0.0f);
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN * NACC) : "memory");
  }
}


// cuTensorMapEncodeTiled reached through the runtime's driver entry point, so
// the library does not link libcuda directly (it still loads on machines
// without a driver, e.g. for the export checks).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    GRU_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || p == nullptr) {
      set_error("cuTensorMapEncodeTiled is not available from the driver");
      return GRU_ERR_CUDA;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return GRU_OK;
}

int make_map(CUtensorMap* map, const float* ptr, int rows, int k, long ld, int box_rows) {
  EncodeTiledFn enc = nullptr;
  int rc = encode_fn(&enc);
  if (rc) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return GRU_ERR_CUDA;
  }
  return GRU_OK;
}

}  // namespace

int read_gemm_status(int reset, int* status) {
  GRU_CUDA_TRY(cudaMemcpyFromSymbol(status, g_gemm_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    GRU_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int)));
  }
  return GRU_OK;
}

bool tc_gemm_supported(const TcGemmArgs& a) {
  return ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) == 0 && a.lda % 4 == 0 &&
         a.ldb % 4 == 0 && a.K >= 1;
}

int tc_gemm(const TcGemmArgs& a, cudaStream_t stream, int kind) {
  if (a.M <= 0 || a.N <= 0) return GRU_OK;
  if (!tc_gemm_supported(a)) {
    set_error("tc_gemm: operands must be 16-byte aligned with row strides a multiple of 4 floats");
    return GRU_ERR_INVALID;
  }
  constexpr int BN = 64, S = 4, NACC = 8;
  using L = Smem<BN, S>;
  static thread_local int configured_device = -1;
  int dev = 0;
  GRU_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_device != dev) {
    GRU_CUDA_TRY(cudaFuncSetAttribute(gemm_tf32x3_kernel<BN, S, NACC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      L::kBytes));
    configured_device = dev;
  }
  CUtensorMap ma, mb;
  int rc = make_map(&ma, a.A, a.M, a.K, a.lda, kBM);
  if (rc) return rc;
  if ((rc = make_map(&mb, a.B, a.N, a.K, a.ldb, BN))) return rc;
  const int tiles = ((a.M + kBM - 1) / kBM) * ((a.N + BN - 1) / BN);
  LaunchScope scope(kind, stream);
  gemm_tf32x3_kernel<BN, S, NACC><<<tiles, kThreads, L::kBytes, stream>>>(ma, mb, a.C, a.ldc, a.bias, a.M, a.N, a.K);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

}  // namespace gru
