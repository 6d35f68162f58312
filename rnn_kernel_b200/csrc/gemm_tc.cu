// FP32-accurate dense products on the 5th-generation tensor cores (sm_100a).
//
//   C[m, n] = sum_k A(m, k) * B(n, k) (+ bias[n])
//
// used for the input projection G = x . W_ih^T + b_ih (prod/gru.py:519-523),
// dx = dG_ih . W_ih (prod/gru.py:575) and the weight gradients
// dW_hh = dG_hh^T . h_prev, dW_ih = dG_ih^T . x (prod/gru.py:569-576).
//
// Precision: "3xTF32".  Every FP32 operand a arrives pre-split into
// a_hi = tf32(a) and a_lo = tf32(a - a_hi) (round to nearest; split_tf32()
// or the producing kernel writes both), and the product is formed as
// a_lo*b_hi + a_hi*b_lo + a_hi*b_hi, keeping about 21 bits of every product.
//
// Structure of one CTA (320 threads, persistent over output tiles):
//   warp 0      TMA producer: the four tiles (A hi/lo, B hi/lo; 128-byte
//               swizzle, unicast from this GPU's memory) of each K stage into
//               an S-deep shared-memory ring;
//   warp 1      allocates tensor memory; lane 0 issues the tcgen05.mma
//               instructions (3 per 8-wide K step) and commits each stage;
//   warps 2-9   drain every finished stage's accumulators into FP32 registers
//               (warp w: tensor-memory lane quarter w % 4, column half
//               (w - 2) / 4; two 32-column load batches per stage) and store
//               each finished tile.
// Every mbarrier wait is bounded; on expiry the kernel records
// GRU_STATUS_WAIT_TIMEOUT and winds down.

#include <cuda.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

__device__ int g_gemm_status = 0;

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;           // fp32 elements per 128-byte swizzle row
constexpr int kDrainWarps = 8;    // 2 per tensor-memory lane quarter
constexpr int kThreads = 64 + 32 * kDrainWarps;
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

// Every operand map is 3-D: (column, row within a period, period).  A plain
// matrix has one period; the rows of a time chunk of a [B*T, cols] matrix
// (rows b*T + t for t in a window of rin steps) have B periods of rin rows.
// Logical row r is (r % rin, r / rin); a box never straddles a period (rin is
// a multiple of the box's rows whenever there is more than one period).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int r,
                                            int rin) {
  const int y = r % rin, z = r / rin;
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
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

// Descriptor of an MN-major tf32 tile.  MN-major 32-bit operands use the
// "128-byte swizzle, 32-byte atom" layout: 32-element (128-byte) wide column
// blocks; within a block K rows of 128 bytes, swizzled in 32-byte granules
// with a 4-row period (4-row atoms of 512 bytes = stride byte offset); blocks
// along M/N are 4096 bytes apart (leading byte offset; one 32 x 32 TMA box
// each, written with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B).
__device__ __forceinline__ uint64_t sw128b32_desc_mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(4096 >> 4) << 16;               // leading byte offset: next 32-wide M/N block
  d |= (uint64_t)(512 >> 4) << 32;                // stride byte offset: next 4 K rows
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)1 << 61;                         // SWIZZLE_128B_BASE32B
  return d;
}

// Instruction descriptor: kind::tf32, D = F32, A = B = TF32; bit 15/16 select
// MN-major A/B.
__host__ __device__ constexpr uint32_t tf32_idesc(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
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
  // per drain warp a 32 x 16 epilogue staging block (row pitch 16 floats,
  // 16-byte chunks XOR-swizzled by row, see the epilogue)
  static constexpr int kEpiPitch = 16;
  static constexpr int kEpiOff = kBarOff + 256;
  static constexpr int kBytes = kEpiOff + kDrainWarps * 32 * kEpiPitch * 4 + 1024;  // + alignment slack
};

// Accumulation.  The tensor cores' FP32 accumulation truncates instead of
// rounding, which biases long sums toward zero (measured: -1.5e-7 relative
// on K = 256 with one accumulator; ~1e-6 after 32 stages).  So every K stage
// goes into a FRESH pair of tensor-memory accumulators (hi*hi products in one,
// the two cross products in the other), NPAIR pairs in rotation, and the
// epilogue warps drain each finished pair into FP32 registers with ordinary
// round-to-nearest adds while the tensor cores work on the next stages.
//
// A_MN / B_MN: the operand is stored MN-major (its K index is the row), as for
// the weight gradients dW = dG^T . X whose K is B*T.
//
// Persistent: the grid has at most one CTA per SM, and each CTA walks the
// work units u = blockIdx.x, blockIdx.x + gridDim.x, ... where a unit is one
// 128 x BN output tile of one K split (splits > 1 write FP32 partials to
// C + split * M * ldc, without bias, for a later FP64 reduce).  The stage
// ring, the accumulator pairs and their mbarrier phases continue across units,
// so loads of the next tile overlap the drain and stores of the previous one.
//
// Grouped launch: one kernel runs up to kMaxProblems products (the weight
// gradients of one backward) as one persistent grid; unit u belongs to the
// problem whose [unit_begin, unit_end) range holds it.
constexpr int kMaxProblems = 3;
struct GemmProblem {
  CUtensorMap ah, al, bh, bl;  // A hi/lo, B hi/lo tensor maps
  int a_rin, b_rin;             // rows per period of the A / B maps
  int c_rin;                    // C rows: logical row r is stored at row (r / c_rin) * c_rstride + r % c_rin
  long c_rstride;
  float* C;
  long ldc;
  const float* bias;
  int M, N, K, kchunk, splits, tiles_n, tiles, unit_end;  // unit_end: cumulative over the batch
};
struct GemmBatch {
  GemmProblem p[kMaxProblems];
  int np, units;
};

struct Unit {
  int m0, n0, kbeg, nk, split, pi;
};

template <int BN>
__device__ __forceinline__ Unit unit_of(const GemmBatch& bt, int u) {
  Unit w;
  int pi = 0;
  while (pi + 1 < bt.np && u >= bt.p[pi].unit_end) ++pi;
  const GemmProblem& P = bt.p[pi];
  const int v = u - (pi > 0 ? bt.p[pi - 1].unit_end : 0);
  const int tile = v % P.tiles;
  w.pi = pi;
  w.split = v / P.tiles;
  w.m0 = (tile / P.tiles_n) * kBM;
  w.n0 = (tile % P.tiles_n) * BN;
  w.kbeg = w.split * P.kchunk;
  const int kend = min(P.K, w.kbeg + P.kchunk);
  w.nk = kend > w.kbeg ? (kend - w.kbeg + kBK - 1) / kBK : 0;
  return w;
}

// 32 consecutive tensor-memory columns of this warp's lane quarter (one
// 32-bit value per lane and column) into r[0..31]; completes at the next
// tcgen05.wait::ld.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

template <int BN, int S, int NPAIR, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tf32x3_kernel(const __grid_constant__ GemmBatch bt) {
  using L = Smem<BN, S>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kBarOff;
  // barriers: full[S], (unused)[S], empty[S], filled[NPAIR], drained[NPAIR]; then the TMEM slot
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (2 * S + s); };
  auto filled = [&](int p) { return bars + 8u * (3 * S + p); };
  auto drained = [&](int p) { return bars + 8u * (3 * S + NPAIR + p); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBarOff + 8 * (3 * S + 2 * NPAIR));
  constexpr int kCols = 2 * NPAIR * BN;  // tensor-memory columns allocated

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = bt.units;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int p = 0; p < NPAIR; ++p) {
      mbar_init(filled(p), 1);
      mbar_init(drained(p), kDrainWarps);  // one arrival per drain warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    for (int pi = 0; pi < bt.np; ++pi) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bt.p[pi].ah)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bt.p[pi].al)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bt.p[pi].bh)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bt.p[pi].bl)) : "memory");
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int i = 0;  // global stage counter of this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = unit_of<BN>(bt, u);
        for (int ks = 0; ks < w.nk; ++ks, ++i) {
          const int s = i % S;
          if (i >= S && !mbar_wait(empty(s), ((i / S) - 1) & 1)) { ok = false; break; }
          const uint32_t st = sbase + s * L::kStage;
          mbar_arrive_expect_tx(full(s), 2 * (L::kATile + L::kBTile));
          const int k0 = w.kbeg + ks * kBK;
          const uint32_t a_hi = st, a_lo = st + L::kATile, b_hi = st + 2 * L::kATile, b_lo = b_hi + L::kBTile;
          const CUtensorMap* map_ah = &bt.p[w.pi].ah;
          const CUtensorMap* map_al = &bt.p[w.pi].al;
          const CUtensorMap* map_bh = &bt.p[w.pi].bh;
          const CUtensorMap* map_bl = &bt.p[w.pi].bl;
          const int arin = bt.p[w.pi].a_rin, brin = bt.p[w.pi].b_rin;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < kBM / 32; ++j) {
              tma_load_3d(a_hi + j * 4096, map_ah, full(s), w.m0 + 32 * j, k0, arin);
              tma_load_3d(a_lo + j * 4096, map_al, full(s), w.m0 + 32 * j, k0, arin);
            }
          } else {
            tma_load_3d(a_hi, map_ah, full(s), k0, w.m0, arin);
            tma_load_3d(a_lo, map_al, full(s), k0, w.m0, arin);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j) {
              tma_load_3d(b_hi + j * 4096, map_bh, full(s), w.n0 + 32 * j, k0, brin);
              tma_load_3d(b_lo + j * 4096, map_bl, full(s), w.n0 + 32 * j, k0, brin);
            }
          } else {
            tma_load_3d(b_hi, map_bh, full(s), k0, w.n0, brin);
            tma_load_3d(b_lo, map_bl, full(s), k0, w.n0, brin);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tf32_idesc(kBM, BN, A_MN, B_MN);
      // 8-wide K steps: 32 bytes along a K-major row, or 8 rows (1024 bytes)
      // of an MN-major block.
      auto da = [&](uint32_t base, int kk) {
        return A_MN ? sw128b32_desc_mn(base + kk * 1024) : sw128_desc(base + kk * 32);
      };
      auto db = [&](uint32_t base, int kk) {
        return B_MN ? sw128b32_desc_mn(base + kk * 1024) : sw128_desc(base + kk * 32);
      };
      int i = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = unit_of<BN>(bt, u);
        for (int ks = 0; ks < w.nk; ++ks, ++i) {
          const int s = i % S, p = i % NPAIR;
          if (!mbar_wait(full(s), (i / S) & 1)) { ok = false; break; }
          if (i >= NPAIR && !mbar_wait(drained(p), ((i / NPAIR) - 1) & 1)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = sbase + s * L::kStage;
          const uint32_t a_hi = st, a_lo = st + L::kATile, b_hi = st + 2 * L::kATile, b_lo = b_hi + L::kBTile;
          const uint32_t d_big = tmem + (uint32_t)(BN * (2 * p));
          const uint32_t d_small = tmem + (uint32_t)(BN * (2 * p + 1));
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint32_t acc = kk == 0 ? 0u : 1u;
            mma_tf32(d_small, da(a_lo, kk), db(b_hi, kk), idesc, acc);
            mma_tf32(d_small, da(a_hi, kk), db(b_lo, kk), idesc, 1u);
            mma_tf32(d_big, da(a_hi, kk), db(b_hi, kk), idesc, acc);
          }
          mma_commit(empty(s));
          mma_commit(filled(p));
        }
      }
    }
  } else {
    // Warps 2..9 drain each finished stage's accumulator pair into FP32
    // registers: warp w reads tensor-memory lanes 32 (w % 4) .. +31 (the only
    // quarter it may access) and the column half (w - 2) / 4, and stores that
    // part of each finished tile.
    constexpr int kCW = BN / 2;  // columns per drain warp
    const int quarter = warp & 3, chalf = (warp - 2) >> 2;
    const uint32_t taddr = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(kCW * chalf);
    float acc[kCW];
#pragma unroll
    for (int c = 0; c < kCW; ++c) acc[c] = 0.0f;
    bool ok = true;
    int d = 0;  // global stage counter of this CTA
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const Unit w = unit_of<BN>(bt, u);
      for (int ks = 0; ks < w.nk; ++ks, ++d) {
        const int p = d % NPAIR;
        // one lane polls (32 lanes polling one mbarrier serialise on its
        // bank), the warp then synchronises before the tensor-memory loads
        bool got = true;
        if (lane == 0) got = mbar_wait(filled(p), (d / NPAIR) & 1);
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        if (!got) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int c0 = 0; c0 < kCW; c0 += 32) {
          uint32_t rs[32], rb[32];
          tmem_ld32(taddr + (uint32_t)(BN * (2 * p + 1) + c0), rs);
          tmem_ld32(taddr + (uint32_t)(BN * (2 * p) + c0), rb);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) acc[c0 + jj] += __uint_as_float(rb[jj]) + __uint_as_float(rs[jj]);
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();  // every lane's tensor-memory loads of this pair are done
        if (lane == 0) mbar_arrive(drained(p));
      }
      if (!ok) break;
      // tile finished (units without K work produce a zero tile)
      const GemmProblem& P = bt.p[w.pi];
      const int M = P.M, N = P.N;
      const long ldc = P.ldc;
      const int crin = P.c_rin;
      const long crs = P.c_rstride;
      auto crow_of = [&](int r) -> long { return crin > 0 ? (long)(r / crin) * crs + r % crin : (long)r; };
      const int row = w.m0 + 32 * quarter + lane;
      const int n0 = w.n0 + kCW * chalf;
      float* Cu = P.splits > 1 ? P.C + (long)w.split * M * ldc : P.C;
      const float* bu = P.splits > 1 ? nullptr : P.bias;
      // Warp-uniform: 16-byte rows, whole 64-column block inside N.
      const bool vec = (ldc % 4 == 0) && n0 + kCW <= N && ((reinterpret_cast<uintptr_t>(Cu + n0) & 15) == 0);
      if (vec) {
        // Each lane holds one row; stage 16 columns at a time through this
        // warp's shared block and store them with 4 lanes per row (64
        // contiguous bytes, 8 rows per instruction) instead of one 16-byte
        // piece of 32 different rows per instruction.  Row r keeps its four
        // 16-byte chunks q at chunk slot q ^ ((r >> 1) & 3): the lane-per-row
        // float4 writes and the 4-lanes-per-row float4 reads then both touch
        // 8 distinct 16-byte bank groups per quarter warp (no conflicts).
        float* eb = reinterpret_cast<float*>(smem + L::kEpiOff) + (warp - 2) * (32 * L::kEpiPitch);
        const int rbase = w.m0 + 32 * quarter;
        const int wsw = (lane >> 1) & 3;
#pragma unroll
        for (int c0 = 0; c0 < kCW; c0 += 16) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int c = c0 + 4 * q;
            float4 v = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
            if (bu) {
              v.x += bu[n0 + c];
              v.y += bu[n0 + c + 1];
              v.z += bu[n0 + c + 2];
              v.w += bu[n0 + c + 3];
            }
            *reinterpret_cast<float4*>(eb + lane * L::kEpiPitch + 4 * (q ^ wsw)) = v;
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = i * 8 + (lane >> 2), q = lane & 3;
            if (rbase + r < M) {
              const float4 e = *reinterpret_cast<const float4*>(eb + r * L::kEpiPitch + 4 * (q ^ ((r >> 1) & 3)));
              *reinterpret_cast<float4*>(Cu + crow_of(rbase + r) * ldc + n0 + c0 + 4 * q) = e;
            }
          }
          __syncwarp();
        }
      } else if (row < M) {
        float* crow = Cu + crow_of(row) * ldc + n0;
        {
#pragma unroll
          for (int c = 0; c < kCW; ++c) {
            const int n = n0 + c;
            if (n < N) crow[c] = acc[c] + (bu ? bu[n] : 0.0f);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < kCW; ++c) acc[c] = 0.0f;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
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

// 3-D fp32 tensor map over the logical rows of a row-major matrix (row stride
// ld floats): `periods` blocks of `rin` consecutive rows, block p starting
// at row p * rstride (one block of rows rows for a plain matrix);
// box = box_cols (inner) x box_rows x 1, 128-byte swizzle.
int make_map(CUtensorMap* map, const float* ptr, long rows, long cols, long ld, int box_cols, int box_rows,
             bool mn_major, int rin = 0, long rstride = 0) {
  EncodeTiledFn enc = nullptr;
  int rc = encode_fn(&enc);
  if (rc) return rc;
  const long in = rin > 0 ? rin : rows;
  const long periods = rin > 0 ? rows / rin : 1;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)in, (cuuint64_t)periods};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(rin > 0 ? rstride : rows) * ld * 4};
  cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return GRU_ERR_CUDA;
  }
  return GRU_OK;
}

// Split-K sums of a batch: C_p[m, n] = sum_z part_p[z][m][n] in FP64, for
// every problem p with splits > 1 (deterministic order).
struct SplitSum {
  const float* part;
  float* C;
  long ldp, ldc;
  int S, M, N;
  long end;  // cumulative element count over the batch
};
struct SplitSumBatch {
  SplitSum q[kMaxProblems];
  int nq;
};

__global__ void splitk_sum_kernel(const __grid_constant__ SplitSumBatch sb) {
  const long total = sb.q[sb.nq - 1].end;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
    int qi = 0;
    while (qi + 1 < sb.nq && e >= sb.q[qi].end) ++qi;
    const SplitSum& Q = sb.q[qi];
    const long v = e - (qi > 0 ? sb.q[qi - 1].end : 0);
    const int m = (int)(v / Q.N), n = (int)(v - (long)m * Q.N);
    double acc = 0.0;
    for (int z = 0; z < Q.S; ++z) acc += Q.part[((long)z * Q.M + m) * Q.ldp + n];
    Q.C[(long)m * Q.ldc + n] = (float)acc;
  }
}

constexpr int kBN = 128, kS = 3, kNPAIR = 2;
constexpr int kMaxStagesPerSplit = 128;  // K stages (32 rows each) summed in FP32 by one split
using LDefault = Smem<kBN, kS>;

// One launch for problems a[0..n) (same operand majors); problem i writes
// to C[i] (row stride ldc[i]) with splits[i] K splits of kchunk[i].
template <bool A_MN, bool B_MN>
int launch_tc(const TcGemmArgs* a, int n, float* const* C, const long* ldc, const int* splits, const int* kchunk,
              cudaStream_t stream, int ctas) {
  auto kern = gemm_tf32x3_kernel<kBN, kS, kNPAIR, A_MN, B_MN>;
  static thread_local int configured_device = -1;
  int dev = 0;
  GRU_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_device != dev) {
    GRU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, LDefault::kBytes));
    configured_device = dev;
  }
  GemmBatch bt;
  memset(&bt, 0, sizeof(bt));
  bt.np = n;
  int units = 0;
  for (int i = 0; i < n; ++i) {
    GemmProblem& P = bt.p[i];
    int rc;
    // rin / rstride describe the rows of the [B*T]-row operands: A's rows (M
    // when K-major, K when MN-major), B's K rows when MN-major, and C's rows
    // when A is K-major (the input projection).
    const int rin = a[i].rin;
    const long rs = a[i].rstride;
    if (A_MN) {
      if ((rc = make_map(&P.ah, a[i].A, a[i].K, a[i].M, a[i].lda, 32, kBK, true, rin, rs))) return rc;
      if ((rc = make_map(&P.al, a[i].A_lo, a[i].K, a[i].M, a[i].lda, 32, kBK, true, rin, rs))) return rc;
      P.a_rin = rin > 0 ? rin : a[i].K;
    } else {
      if ((rc = make_map(&P.ah, a[i].A, a[i].M, a[i].K, a[i].lda, kBK, kBM, false, rin, rs))) return rc;
      if ((rc = make_map(&P.al, a[i].A_lo, a[i].M, a[i].K, a[i].lda, kBK, kBM, false, rin, rs))) return rc;
      P.a_rin = rin > 0 ? rin : a[i].M;
      P.c_rin = rin;
      P.c_rstride = rs;
    }
    if (B_MN) {
      if ((rc = make_map(&P.bh, a[i].B, a[i].K, a[i].N, a[i].ldb, 32, kBK, true, rin, rs))) return rc;
      if ((rc = make_map(&P.bl, a[i].B_lo, a[i].K, a[i].N, a[i].ldb, 32, kBK, true, rin, rs))) return rc;
      P.b_rin = rin > 0 ? rin : a[i].K;
    } else {
      if ((rc = make_map(&P.bh, a[i].B, a[i].N, a[i].K, a[i].ldb, kBK, kBN, false))) return rc;
      if ((rc = make_map(&P.bl, a[i].B_lo, a[i].N, a[i].K, a[i].ldb, kBK, kBN, false))) return rc;
      P.b_rin = a[i].N;
    }
    P.C = C[i];
    P.ldc = ldc[i];
    P.bias = splits[i] > 1 ? nullptr : a[i].bias;
    P.M = a[i].M;
    P.N = a[i].N;
    P.K = a[i].K;
    P.kchunk = kchunk[i];
    P.splits = splits[i];
    P.tiles_n = (a[i].N + kBN - 1) / kBN;
    P.tiles = ((a[i].M + kBM - 1) / kBM) * P.tiles_n;
    units += P.tiles * splits[i];
    P.unit_end = units;
  }
  bt.units = units;
  const int cap = ctas > 0 && ctas < sm_count(dev) ? ctas : sm_count(dev);
  const int grid = units < cap ? units : cap;
  kern<<<grid, kThreads, LDefault::kBytes, stream>>>(bt);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

__device__ __forceinline__ void split4(float4 v, float4& h, float4& l) {
  h = make_float4(__uint_as_float(to_tf32(v.x)), __uint_as_float(to_tf32(v.y)), __uint_as_float(to_tf32(v.z)),
                  __uint_as_float(to_tf32(v.w)));
  l = make_float4(__uint_as_float(to_tf32(v.x - h.x)), __uint_as_float(to_tf32(v.y - h.y)),
                  __uint_as_float(to_tf32(v.z - h.z)), __uint_as_float(to_tf32(v.w - h.w)));
}

// One split job: hi[r, c] = tf32(src[r, c]), lo[r, c] = tf32(src - hi) for
// c < cols, 0 for cols <= c < ldd.
struct SplitJob {
  const float* src;
  float* hi;
  float* lo;
  long rows, lds, row_end;  // row_end: cumulative rows over the launch
  int cols, ldd, vec;       // vec: float4 path allowed
  int rin;                  // periodic rows (0: plain)
  long rstride;
};
struct SplitJobs {
  SplitJob j[4];
  int n;
};

// One row per (blockIdx.x + k * gridDim.x) over the rows of all jobs,
// threads across the columns; float4 when the job's rows allow it.
__global__ void split_tf32_kernel(const __grid_constant__ SplitJobs js) {
  const long total = js.j[js.n - 1].row_end;
  for (long g = blockIdx.x; g < total; g += gridDim.x) {
    int ji = 0;
    while (ji + 1 < js.n && g >= js.j[ji].row_end) ++ji;
    const SplitJob& J = js.j[ji];
    const long rl = g - (ji > 0 ? js.j[ji - 1].row_end : 0);
    const long r = J.rin > 0 ? (rl / J.rin) * J.rstride + rl % J.rin : rl;
    const float* sr = J.src + r * J.lds;
    float* hr = J.hi + r * J.ldd;
    float* lr = J.lo + r * J.ldd;
    if (J.vec) {
      for (int c = 4 * threadIdx.x; c < J.ldd; c += 4 * blockDim.x) {
        const float4 v = c < J.cols ? *reinterpret_cast<const float4*>(sr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 h, l;
        split4(v, h, l);
        *reinterpret_cast<float4*>(hr + c) = h;
        *reinterpret_cast<float4*>(lr + c) = l;
      }
    } else {
      for (int c = threadIdx.x; c < J.ldd; c += blockDim.x) {
        const float v = c < J.cols ? sr[c] : 0.0f;
        const uint32_t h = to_tf32(v);
        hr[c] = __uint_as_float(h);
        lr[c] = __uint_as_float(to_tf32(v - __uint_as_float(h)));
      }
    }
  }
}

}  // namespace

int split_tf32_multi(const SplitArgs* a, int n, cudaStream_t stream) {
  if (n < 1 || n > 4) {
    set_error("split_tf32: 1 to 4 jobs per launch");
    return GRU_ERR_INVALID;
  }
  SplitJobs js;
  memset(&js, 0, sizeof(js));
  long rows = 0;
  int maxld = 0;
  for (int i = 0; i < n; ++i) {
    if (a[i].rows <= 0) continue;
    SplitJob& J = js.j[js.n++];
    J.src = a[i].src;
    J.hi = a[i].hi;
    J.lo = a[i].lo;
    J.rows = a[i].rows;
    J.lds = a[i].lds;
    J.cols = a[i].cols;
    J.ldd = a[i].ldd;
    J.rin = a[i].rin;
    J.rstride = a[i].rstride;
    J.vec = (a[i].cols % 4 == 0 && a[i].lds % 4 == 0 && a[i].ldd % 4 == 0 &&
             ((reinterpret_cast<uintptr_t>(a[i].src) | reinterpret_cast<uintptr_t>(a[i].hi) |
               reinterpret_cast<uintptr_t>(a[i].lo)) & 15) == 0) ? 1 : 0;
    rows += a[i].rows;
    J.row_end = rows;
    if (a[i].ldd > maxld) maxld = a[i].ldd;
  }
  if (js.n == 0) return GRU_OK;
  const int threads = maxld >= 1024 ? 256 : (maxld >= 256 ? 64 : 32);
  const long blocks = rows < 16384 ? rows : 16384;
  LaunchScope scope(kKindLayout, stream);
  split_tf32_kernel<<<(unsigned)blocks, threads, 0, stream>>>(js);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

int split_tf32(const float* src, long rows, int cols, long lds, float* hi, float* lo, int ldd, cudaStream_t stream) {
  const SplitArgs a{src, rows, cols, lds, hi, lo, ldd};
  return split_tf32_multi(&a, 1, stream);
}

int read_gemm_status(int reset, int* status) {
  GRU_CUDA_TRY(cudaMemcpyFromSymbol(status, g_gemm_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    GRU_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int)));
  }
  return GRU_OK;
}

// Periodic rows (a time chunk of [B*T]-row operands): the logical row count
// of every periodic operand (M for a K-major A, K for MN-major ones) must be
// whole periods, and a TMA box must not straddle two periods.
bool tc_rows_ok(const TcGemmArgs& a) {
  if (a.rin <= 0) return true;
  const bool ok_m = a.a_mn || (a.rin % kBM == 0 && a.M % a.rin == 0);
  const bool ok_k = !(a.a_mn || a.b_mn) || (a.rin % kBK == 0 && a.K % a.rin == 0);
  const bool ok_s = a.rstride >= a.rin && a.rstride % 4 == 0;
  if (!(ok_m && ok_k && ok_s)) {
    set_error("tc_gemm: periodic rows need whole periods of a multiple of the tile rows");
    return false;
  }
  return true;
}

bool tc_gemm_supported(const TcGemmArgs& a) {
  if (!a.A_lo || !a.B_lo) return false;
  return ((reinterpret_cast<uintptr_t>(a.A_lo) | reinterpret_cast<uintptr_t>(a.B_lo)) & 15) == 0 && ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) == 0 &&
         a.lda % 4 == 0 && a.ldb % 4 == 0 && a.K >= 1;
}

// K splits of the products of one launch: long K (the weight gradients,
// K = B*T) with few output tiles is split so that the whole batch covers the
// SMs about twice, each problem's share in proportion to its work, keeping
// >= 8 and (where that allows) <= kMaxStagesPerSplit K stages per split.
// Without a workspace nothing is split.
void tc_splits_ctas(const TcGemmArgs* a, int n, int ctas, int* out) {
  long work = 0;
  for (int i = 0; i < n; ++i)
    work += (long)((a[i].M + kBM - 1) / kBM) * ((a[i].N + kBN - 1) / kBN) * ((a[i].K + kBK - 1) / kBK);
  for (int i = 0; i < n; ++i) {
    const int tiles = ((a[i].M + kBM - 1) / kBM) * ((a[i].N + kBN - 1) / kBN);
    const int stages = (a[i].K + kBK - 1) / kBK;
    const double share = work > 0 ? (double)tiles * stages / (double)work : 1.0;
    int s = (int)(2.0 * ctas * share / tiles + 0.5);
    // Accuracy: each split's FP32 register sum covers at most
    // kMaxStagesPerSplit stages (long FP32 sums lose digits; the FP64
    // reduce of the splits does not).
    s = std::max(s, (stages + kMaxStagesPerSplit - 1) / kMaxStagesPerSplit);
    if (s > stages / 8) s = stages / 8;
    out[i] = s < 1 ? 1 : s;
  }
}

void tc_splits(const TcGemmArgs* a, int n, int device, int* out) { tc_splits_ctas(a, n, sm_count(device), out); }

size_t tc_gemm_ws_bytes(const TcGemmArgs* a, int n, int device) {
  int sp[kMaxProblems];
  tc_splits(a, n, device, sp);
  size_t total = 0;
  // partials [s][M][N rounded up to 4 floats]: 16-byte rows for the epilogue
  for (int i = 0; i < n; ++i)
    if (sp[i] > 1) total += align_up(sizeof(float) * (size_t)sp[i] * a[i].M * ((a[i].N + 3) / 4 * 4), 256);
  return total;
}

size_t tc_gemm_ws_bytes(const TcGemmArgs& a, int device) { return tc_gemm_ws_bytes(&a, 1, device); }

int tc_gemm_batch(const TcGemmArgs* a, int n, cudaStream_t stream, int kind, void* ws, size_t ws_bytes, int ctas) {
  if (n < 1 || n > kMaxProblems) {
    set_error("tc_gemm: 1 to 3 products per launch");
    return GRU_ERR_INVALID;
  }
  int dev = 0;
  GRU_CUDA_TRY(cudaGetDevice(&dev));
  int sp[kMaxProblems], kc[kMaxProblems];
  float* C[kMaxProblems];
  long ldc[kMaxProblems];
  if (ws) {
    tc_splits(a, n, dev, sp);
    if (ws_bytes < tc_gemm_ws_bytes(a, n, dev)) {
      set_error("tc_gemm: split-K workspace too small");
      return GRU_ERR_INVALID;
    }
  } else {
    for (int i = 0; i < n; ++i) sp[i] = 1;
  }
  SplitSumBatch sb;
  memset(&sb, 0, sizeof(sb));
  char* wp = static_cast<char*>(ws);
  long sum_elems = 0;
  int live = 0;  // problems with something to compute
  TcGemmArgs run[kMaxProblems];
  int rsp[kMaxProblems], rkc[kMaxProblems];
  float* rC[kMaxProblems];
  long rldc[kMaxProblems];
  for (int i = 0; i < n; ++i) {
    if (a[i].M <= 0 || a[i].N <= 0) continue;
    if (!tc_gemm_supported(a[i])) {
      set_error("tc_gemm: operands must be pre-split (hi and lo), 16-byte aligned, with row strides a multiple of 4 floats");
      return GRU_ERR_INVALID;
    }
    if (a[i].a_mn != a[0].a_mn || a[i].b_mn != a[0].b_mn) {
      set_error("tc_gemm: the products of one launch must share their operand majors");
      return GRU_ERR_INVALID;
    }
    if (!tc_rows_ok(a[i])) return GRU_ERR_INVALID;
    kc[i] = sp[i] > 1 ? ((a[i].K + sp[i] * kBK - 1) / (sp[i] * kBK)) * kBK : a[i].K;
    C[i] = a[i].C;
    ldc[i] = a[i].ldc;
    if (sp[i] > 1) {
      if (a[i].bias) {
        set_error("tc_gemm: bias with split-K is not supported");
        return GRU_ERR_INVALID;
      }
      C[i] = reinterpret_cast<float*>(wp);
      ldc[i] = (a[i].N + 3) / 4 * 4;
      wp += align_up(sizeof(float) * (size_t)sp[i] * a[i].M * ldc[i], 256);
      SplitSum& Q = sb.q[sb.nq++];
      Q.part = C[i];
      Q.C = a[i].C;
      Q.ldp = ldc[i];
      Q.ldc = a[i].ldc;
      Q.S = sp[i];
      Q.M = a[i].M;
      Q.N = a[i].N;
      sum_elems += (long)a[i].M * a[i].N;
      Q.end = sum_elems;
    }
    run[live] = a[i];
    rsp[live] = sp[i];
    rkc[live] = kc[i];
    rC[live] = C[i];
    rldc[live] = ldc[i];
    ++live;
  }
  if (live == 0) return GRU_OK;
  LaunchScope scope(kind, stream, sb.nq > 0 ? 2 : 1);
  int rc;
  if (run[0].a_mn && run[0].b_mn) rc = launch_tc<true, true>(run, live, rC, rldc, rsp, rkc, stream, ctas);
  else if (!run[0].a_mn && !run[0].b_mn) rc = launch_tc<false, false>(run, live, rC, rldc, rsp, rkc, stream, ctas);
  else {
    set_error("tc_gemm: mixed operand majors are not instantiated");
    return GRU_ERR_INVALID;
  }
  if (rc) return rc;
  if (sb.nq > 0) {
    splitk_sum_kernel<<<sm_count(dev) * 4, 256, 0, stream>>>(sb);
    GRU_CUDA_TRY(cudaGetLastError());
  }
  return GRU_OK;
}

int tc_gemm(const TcGemmArgs& a, cudaStream_t stream, int kind, void* ws, size_t ws_bytes, int ctas) {
  return tc_gemm_batch(&a, 1, stream, kind, ws, ws_bytes, ctas);
}

int tc_partial_splits(const TcGemmArgs* a, int n, int ctas, int* splits) {
  if (n < 1 || n > kMaxProblems) {
    set_error("tc_gemm: 1 to 3 products per launch");
    return GRU_ERR_INVALID;
  }
  tc_splits_ctas(a, n, ctas, splits);
  return GRU_OK;
}

int tc_gemm_partials(const TcGemmArgs* a, int n, cudaStream_t stream, int kind, int ctas, float* const* part,
                     const long* ldp, int* zoff) {
  int dev = 0;
  GRU_CUDA_TRY(cudaGetDevice(&dev));
  if (ctas <= 0 || ctas > sm_count(dev)) ctas = sm_count(dev);
  int sp[kMaxProblems], kc[kMaxProblems];
  if (int rc = tc_partial_splits(a, n, ctas, sp)) return rc;
  float* C[kMaxProblems];
  long ldc[kMaxProblems];
  for (int i = 0; i < n; ++i) {
    if (a[i].M <= 0 || a[i].N <= 0 || a[i].K <= 0 || !tc_gemm_supported(a[i]) || a[i].bias ||
        a[i].a_mn != a[0].a_mn || a[i].b_mn != a[0].b_mn || ldp[i] % 4 != 0 || ldp[i] < a[i].N) {
      set_error("tc_gemm_partials: unsupported product");
      return GRU_ERR_INVALID;
    }
    if (!tc_rows_ok(a[i])) return GRU_ERR_INVALID;
    kc[i] = ((a[i].K + sp[i] * kBK - 1) / (sp[i] * kBK)) * kBK;
    C[i] = part[i] + (long)zoff[i] * a[i].M * ldp[i];
    ldc[i] = ldp[i];
    zoff[i] += sp[i];
  }
  LaunchScope scope(kind, stream);
  if (a[0].a_mn && a[0].b_mn) return launch_tc<true, true>(a, n, C, ldc, sp, kc, stream, ctas);
  if (!a[0].a_mn && !a[0].b_mn) return launch_tc<false, false>(a, n, C, ldc, sp, kc, stream, ctas);
  set_error("tc_gemm: mixed operand majors are not instantiated");
  return GRU_ERR_INVALID;
}

int tc_gemm_sum(const TcGemmArgs* a, int n, const float* const* part, const long* ldp, const int* nslices,
                cudaStream_t stream, int kind) {
  if (n < 1 || n > kMaxProblems) {
    set_error("tc_gemm_sum: 1 to 3 products");
    return GRU_ERR_INVALID;
  }
  SplitSumBatch sb;
  memset(&sb, 0, sizeof(sb));
  long elems = 0;
  for (int i = 0; i < n; ++i) {
    if (a[i].M <= 0 || a[i].N <= 0) continue;
    SplitSum& Q = sb.q[sb.nq++];
    Q.part = part[i];
    Q.C = a[i].C;
    Q.ldp = ldp[i];
    Q.ldc = a[i].ldc;
    Q.S = nslices[i];
    Q.M = a[i].M;
    Q.N = a[i].N;
    elems += (long)a[i].M * a[i].N;
    Q.end = elems;
  }
  if (sb.nq == 0) return GRU_OK;
  int dev = 0;
  GRU_CUDA_TRY(cudaGetDevice(&dev));
  LaunchScope scope(kind, stream);
  splitk_sum_kernel<<<sm_count(dev) * 4, 256, 0, stream>>>(sb);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

}  // namespace gru
