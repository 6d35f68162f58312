// Bias gradients (final deterministic sum of the backward time loop's FP64
// per-cluster column sums of dG, prod/gru.py:574/578) and the W_ih transpose
// that feeds the dx product.

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

namespace {

// One warp per column: lane l sums partial rows l, l+32, ... then a fixed
// shuffle tree (deterministic).
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

int bias_grads_finish(const double* part, int nparts, int H, float* db_ih, float* db_hh, cudaStream_t stream) {
  if (H <= 0) return GRU_OK;
  LaunchScope scope(kKindColsum, stream);
  bias_grad_final_kernel<<<ceil_div(4 * H, 8), 256, 0, stream>>>(part, nparts, H, db_ih, db_hh);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

}  // namespace gru
