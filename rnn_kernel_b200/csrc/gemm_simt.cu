// FP32 strided contraction with deterministic split-K, and FP64-accumulated
// column sums.  These implement the dense products around the GRU time loop:
// the input projection x.W_ih^T + b_ih (prod/gru.py:519-523) and the gradient
// contractions dW_hh, dx, dW_ih, db_* (prod/gru.py:569-578).

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

namespace {

constexpr int BM = 64, BN = 64, BK = 16;

// C tile (or split-K partial) = A(m, k) B(k, n) over k in [k0, k1).
// Acc = double: every FP32 x FP32 product is exact in FP64 and the sum is
// accumulated in FP64 (used for the weight-gradient contractions whose K is
// B*T); Acc = float: plain FP32 FMA (K = I or 3H).
template <typename Acc>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(GemmArgs a, int kchunk, Acc* partial) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int k0 = blockIdx.z * kchunk;
  const int k1 = min(a.K, k0 + kchunk);
  Acc acc[4][4] = {};
  const bool a_kfast = (a.sak == 1);
  const bool b_nfast = (a.sbn == 1);
  for (int kt = k0; kt < k1; kt += BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      int mm, kk;
      if (a_kfast) { mm = e / BK; kk = e % BK; }
      else { kk = e / BM; mm = e % BM; }
      const int m = m0 + mm, k = kt + kk;
      As[kk][mm] = (m < a.M && k < k1) ? a.A[(long)m * a.sam + (long)k * a.sak] : 0.0f;
      int nn, kb;
      if (b_nfast) { kb = e / BN; nn = e % BN; }
      else { nn = e / BK; kb = e % BK; }
      const int n = n0 + nn, k2 = kt + kb;
      Bs[kb][nn] = (n < a.N && k2 < k1) ? a.B[(long)k2 * a.sbk + (long)n * a.sbn] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      Acc av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= a.N) continue;
      if (partial != nullptr) {
        partial[((size_t)blockIdx.z * a.M + m) * a.N + n] = acc[i][j];
      } else {
        a.C[(long)m * a.ldc + n] = (float)(acc[i][j] + (a.bias ? (Acc)a.bias[n] : (Acc)0));
      }
    }
  }
}

template <typename Acc>
__global__ void splitk_reduce_kernel(const Acc* partial, int S, GemmArgs a) {
  const long MN = (long)a.M * a.N;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < MN; e += (long)gridDim.x * blockDim.x) {
    double s = 0.0;
    for (int z = 0; z < S; ++z) s += partial[z * MN + e];
    const int m = (int)(e / a.N), n = (int)(e % a.N);
    if (a.bias) s += a.bias[n];
    a.C[(long)m * a.ldc + n] = (float)s;
  }
}

int splits_for(int M, int N, int K, int device) {
  const int tiles = ceil_div(M, BM) * ceil_div(N, BN);
  const int sms = sm_count(device);
  int S = 1;
  while (tiles * S < 2 * sms && K / (S * 2) >= 256) S *= 2;
  return S;
}

// Bias gradients.  dG_ih = [dr, dz, dn_pre] and dG_hh = [dr, dz, dhn] share
// their r and z columns, so one pass sums the 3H columns of dG_ih and the n
// block of dG_hh (virtual columns 3H .. 4H): db_ih = cols [0, 3H),
// db_hh = [cols 0 .. 2H, cols 3H .. 4H).
__global__ void bias_grad_partial_kernel(const float* __restrict__ dgi, const float* __restrict__ dgh, long rows,
                                         int H, long ld, long rchunk, double* __restrict__ part) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= 4 * H) return;
  const float* X = col < 3 * H ? dgi + col : dgh + (col - H);  // dG_hh n block = its columns 2H .. 3H
  const long r0 = blockIdx.y * rchunk, r1 = min(rows, r0 + rchunk);
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
  long r = r0;
  for (; r + 4 <= r1; r += 4) {
    s0 += X[r * ld];
    s1 += X[(r + 1) * ld];
    s2 += X[(r + 2) * ld];
    s3 += X[(r + 3) * ld];
  }
  for (; r < r1; ++r) s0 += X[r * ld];
  part[(long)blockIdx.y * 4 * H + col] = (s0 + s1) + (s2 + s3);
}

__global__ void bias_grad_final_kernel(const double* __restrict__ part, int nchunks, int H, float* __restrict__ db_ih,
                                       float* __restrict__ db_hh) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= 4 * H) return;
  double s = 0.0;
  for (int z = 0; z < nchunks; ++z) s += part[(long)z * 4 * H + col];
  const float v = (float)s;
  if (col < 3 * H) db_ih[col] = v;
  if (col < 2 * H) db_hh[col] = v;
  else if (col >= 3 * H) db_hh[col - H] = v;
}

constexpr int kColChunks = 256;

__global__ void pad_rows_kernel(const float* src, long rows, int cols, float* dst, int ldd) {
  const long n = rows * ldd;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const long r = e / ldd;
    const int c = (int)(e - r * ldd);
    dst[e] = c < cols ? src[r * cols + c] : 0.0f;
  }
}

__global__ void transpose_kernel(const float* src, int rows, int cols, float* dst, int ldd) {
  __shared__ float tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? src[(long)r * cols + c] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;  // dst[c][r]
    if (c < cols && r < ldd) dst[(long)c * ldd + r] = r < rows ? tile[threadIdx.x][i] : 0.0f;
  }
}

}  // namespace

int pad_rows(const float* src, long rows, int cols, float* dst, int ldd, cudaStream_t stream) {
  if (rows <= 0) return GRU_OK;
  LaunchScope scope(kKindLayout, stream);
  pad_rows_kernel<<<1184, 256, 0, stream>>>(src, rows, cols, dst, ldd);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

int transpose(const float* src, int rows, int cols, float* dst, int ldd, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return GRU_OK;
  LaunchScope scope(kKindLayout, stream);
  dim3 grid(ceil_div(cols, 32), ceil_div(ldd, 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(src, rows, cols, dst, ldd);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

size_t gemm_ws_bytes(int M, int N, int K, int device) {
  const int S = splits_for(M, N, K, device);
  return S > 1 ? sizeof(double) * (size_t)S * M * N : 0;
}

template <typename Acc>
int gemm_impl(const GemmArgs& a, void* ws, size_t ws_bytes, int device, cudaStream_t stream, int kind) {
  const int S = (a.K > 0 && ws != nullptr) ? splits_for(a.M, a.N, a.K, device) : 1;
  const int kchunk = a.K > 0 ? ceil_div(ceil_div(a.K, S), BK) * BK : BK;
  dim3 grid(ceil_div(a.N, BN), ceil_div(a.M, BM), S);
  Acc* partial = nullptr;
  if (S > 1) {
    if (ws_bytes < gemm_ws_bytes(a.M, a.N, a.K, device)) {
      set_error("gemm: workspace too small");
      return GRU_ERR_INVALID;
    }
    partial = static_cast<Acc*>(ws);
  }
  LaunchScope scope(kind, stream, S > 1 ? 2 : 1);
  gemm_simt_kernel<Acc><<<grid, 256, 0, stream>>>(a, kchunk, partial);
  GRU_CUDA_TRY(cudaGetLastError());
  if (S > 1) {
    splitk_reduce_kernel<Acc><<<sm_count(device) * 4, 256, 0, stream>>>(partial, S, a);
    GRU_CUDA_TRY(cudaGetLastError());
  }
  return GRU_OK;
}

int gemm(const GemmArgs& a, void* ws, size_t ws_bytes, int device, cudaStream_t stream, int kind,
         bool exact) {
  if (a.M <= 0 || a.N <= 0) return GRU_OK;
  return exact ? gemm_impl<double>(a, ws, ws_bytes, device, stream, kind)
               : gemm_impl<float>(a, ws, ws_bytes, device, stream, kind);
}

size_t bias_grad_ws_bytes(int H) { return sizeof(double) * (size_t)kColChunks * 4 * H; }

int bias_grads(const float* dgi, const float* dgh, long rows, int H, long ld, float* db_ih, float* db_hh, void* ws,
               cudaStream_t stream) {
  if (H <= 0) return GRU_OK;
  const long rchunk = (rows + kColChunks - 1) / kColChunks;
  double* part = static_cast<double*>(ws);
  dim3 grid(ceil_div(4 * H, 128), kColChunks);
  LaunchScope scope(kKindColsum, stream, 2);
  bias_grad_partial_kernel<<<grid, 128, 0, stream>>>(dgi, dgh, rows, H, ld, rchunk > 0 ? rchunk : 1, part);
  GRU_CUDA_TRY(cudaGetLastError());
  bias_grad_final_kernel<<<ceil_div(4 * H, 128), 128, 0, stream>>>(part, kColChunks, H, db_ih, db_hh);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

}  // namespace gru
