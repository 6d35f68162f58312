// Bias gradients (FP64-accumulated column sums of dG, prod/gru.py:574/578)
// and the W_ih transpose that feeds the dx product.

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

namespace {

// Bias gradients.  dG_ih = [dr, dz, dn_pre] and dG_hh = [dr, dz, dhn] share
// their r and z columns, so one pass sums the 3H columns of dG_ih and the n
// block of dG_hh (its own buffer; virtual columns 3H .. 4H): db_ih = cols
// [0, 3H), db_hh = [cols 0 .. 2H, cols 3H .. 4H).
__global__ void bias_grad_partial_kernel(const float* __restrict__ dgi, const float* __restrict__ dgi_lo, long ld,
                                         const float* __restrict__ dgn, const float* __restrict__ dgn_lo, long ldn,
                                         long rows, int H, long rchunk, double* __restrict__ part) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= 4 * H) return;
  // values are hi + lo
  const bool ih = col < 3 * H;
  const float* X = ih ? dgi + col : dgn + (col - 3 * H);
  const float* Y = ih ? dgi_lo + col : dgn_lo + (col - 3 * H);
  if (!ih) ld = ldn;
  const long r0 = blockIdx.y * rchunk, r1 = min(rows, r0 + rchunk);
  // four rows per iteration: eight independent loads in flight per thread
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
  long r = r0;
  for (; r + 4 <= r1; r += 4) {
    const float x0 = X[r * ld], y0 = Y[r * ld], x1 = X[(r + 1) * ld], y1 = Y[(r + 1) * ld];
    const float x2 = X[(r + 2) * ld], y2 = Y[(r + 2) * ld], x3 = X[(r + 3) * ld], y3 = Y[(r + 3) * ld];
    s0 += (double)x0 + (double)y0;
    s1 += (double)x1 + (double)y1;
    s2 += (double)x2 + (double)y2;
    s3 += (double)x3 + (double)y3;
  }
  for (; r < r1; ++r) s0 += (double)X[r * ld] + (double)Y[r * ld];
  part[(long)blockIdx.y * 4 * H + col] = (s0 + s1) + (s2 + s3);
}

// One warp per column: lane l sums chunks l, l+32, ... then a fixed shuffle
// tree (deterministic).
__global__ void bias_grad_final_kernel(const double* __restrict__ part, int nchunks, int H, float* __restrict__ db_ih,
                                       float* __restrict__ db_hh) {
  const int col = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (col >= 4 * H) return;
  double s = 0.0;
  for (int z = lane; z < nchunks; z += 32) s += part[(long)z * 4 * H + col];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane != 0) return;
  const float v = (float)s;
  if (col < 3 * H) db_ih[col] = v;
  if (col < 2 * H) db_hh[col] = v;
  else if (col >= 3 * H) db_hh[col - H] = v;
}

constexpr int kColChunks = 256;

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

int transpose(const float* src, int rows, int cols, float* dst, int ldd, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return GRU_OK;
  LaunchScope scope(kKindLayout, stream);
  dim3 grid(ceil_div(cols, 32), ceil_div(ldd, 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(src, rows, cols, dst, ldd);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

size_t bias_grad_ws_bytes(int H) { return sizeof(double) * (size_t)kColChunks * 4 * H; }

int bias_grads(const float* dgi, const float* dgi_lo, long ld, const float* dgn, const float* dgn_lo, long ldn,
               long rows, int H, float* db_ih, float* db_hh, void* ws, cudaStream_t stream) {
  if (H <= 0) return GRU_OK;
  const long rchunk = (rows + kColChunks - 1) / kColChunks;
  double* part = static_cast<double*>(ws);
  dim3 grid(ceil_div(4 * H, 128), kColChunks);
  LaunchScope scope(kKindColsum, stream, 2);
  bias_grad_partial_kernel<<<grid, 128, 0, stream>>>(dgi, dgi_lo, ld, dgn, dgn_lo, ldn, rows, H,
                                                     rchunk > 0 ? rchunk : 1, part);
  GRU_CUDA_TRY(cudaGetLastError());
  bias_grad_final_kernel<<<ceil_div(4 * H, 8), 256, 0, stream>>>(part, kColChunks, H, db_ih, db_hh);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

}  // namespace gru
