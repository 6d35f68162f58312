// Mean-squared-error loss of the time loop's output and its gradient, as the
// training harness uses it (F.mse_loss(pred, y): rnn_benchmark.py:636, :657,
// :680; tests/test_sequence_chunking.py:27-28).
//
// torch evaluates it in three passes over the [B, T, H] output (elementwise
// squares, a mean reduction, and the backward's elementwise gradient): about
// 50 us per step at B = 64, T = 512, H = 256.  Here:
//   forward   one pass reading out and target: each block sums (out - y)^2 in
//             FP64 and writes one partial; one single-block launch adds the
//             partials in a fixed order (deterministic) and writes the mean;
//   backward  one pass: dout = (2 / n) * (out - y) * g, with g the loss's
//             upstream gradient read from device memory (no host sync), in
//             torch's order of operations (norm * diff * g).
// HBM-bound: 8 bytes read per element (forward), 8 read + 4 written
// (backward).

#include <cuda_runtime.h>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {
namespace {

constexpr int kMseThreads = 256;

inline int mse_blocks(long n) {
  const long want = (n + 4L * kMseThreads * 8 - 1) / (4L * kMseThreads * 8);  // >= 8 float4 per thread
  const long cap = 4L * 148;
  return (int)(want < 1 ? 1 : (want > cap ? cap : want));
}

__global__ void __launch_bounds__(kMseThreads) mse_partial_kernel(const float* __restrict__ out,
                                                                  const float* __restrict__ tgt, long n, int vec,
                                                                  double* __restrict__ part) {
  double acc = 0.0;
  const long tid = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const long stride = (long)gridDim.x * blockDim.x;
  if (vec) {
    const float4* o4 = reinterpret_cast<const float4*>(out);
    const float4* t4 = reinterpret_cast<const float4*>(tgt);
    const long n4 = n / 4;
    for (long i = tid; i < n4; i += stride) {
      const float4 a = o4[i], b = t4[i];
      const float dx = a.x - b.x, dy = a.y - b.y, dz = a.z - b.z, dw = a.w - b.w;
      acc += (double)(dx * dx) + (double)(dy * dy) + ((double)(dz * dz) + (double)(dw * dw));
    }
  } else {
    for (long i = tid; i < n; i += stride) {
      const float d = out[i] - tgt[i];
      acc += (double)(d * d);
    }
  }
  // fixed-shape tree: warp shuffles, then the warps' sums in order
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  __shared__ double ws[kMseThreads / 32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kMseThreads / 32; ++w) s += ws[w];
    part[blockIdx.x] = s;
  }
}

__global__ void mse_final_kernel(const double* __restrict__ part, int nparts, long n, float* __restrict__ loss) {
  // one warp: lane l sums parts l, l + 32, ... then a fixed shuffle tree
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += 32) s += part[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if (threadIdx.x == 0) *loss = (float)(s / (double)n);
}

__global__ void __launch_bounds__(kMseThreads) mse_backward_kernel(const float* __restrict__ out,
                                                                   const float* __restrict__ tgt,
                                                                   const float* __restrict__ gloss, float norm,
                                                                   long n, int vec, float* __restrict__ dout) {
  const float g = *gloss;
  const long tid = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const long stride = (long)gridDim.x * blockDim.x;
  if (vec) {
    const float4* o4 = reinterpret_cast<const float4*>(out);
    const float4* t4 = reinterpret_cast<const float4*>(tgt);
    float4* d4 = reinterpret_cast<float4*>(dout);
    const long n4 = n / 4;
    for (long i = tid; i < n4; i += stride) {
      const float4 a = o4[i], b = t4[i];
      d4[i] = make_float4(norm * (a.x - b.x) * g, norm * (a.y - b.y) * g, norm * (a.z - b.z) * g,
                          norm * (a.w - b.w) * g);
    }
  } else {
    for (long i = tid; i < n; i += stride) dout[i] = norm * (out[i] - tgt[i]) * g;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace gru

using namespace gru;

extern "C" size_t gru_mse_workspace_bytes(long n) {
  if (n <= 0) return 0;
  return sizeof(double) * (size_t)mse_blocks(n);
}

extern "C" int gru_mse_loss(const float* out, const float* target, long n, float* loss, void* workspace,
                            size_t workspace_bytes, void* stream_) {
  clear_error();
  if (n <= 0 || !out || !target || !loss) {
    set_error("gru_mse_loss: need n >= 1 and non-null out, target, loss");
    return GRU_ERR_INVALID;
  }
  if (!workspace || workspace_bytes < gru_mse_workspace_bytes(n) || (reinterpret_cast<uintptr_t>(workspace) & 7)) {
    set_error("gru_mse_loss: workspace too small or not 8-byte aligned");
    return GRU_ERR_INVALID;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int nb = mse_blocks(n);
  const int vec = (n % 4 == 0 && aligned16(out) && aligned16(target)) ? 1 : 0;
  double* part = static_cast<double*>(workspace);
  LaunchScope scope(kKindLoss, stream, 2);
  mse_partial_kernel<<<nb, kMseThreads, 0, stream>>>(out, target, n, vec, part);
  GRU_CUDA_TRY(cudaGetLastError());
  mse_final_kernel<<<1, 32, 0, stream>>>(part, nb, n, loss);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}

extern "C" int gru_mse_loss_backward(const float* out, const float* target, const float* grad_loss, float* dout,
                                     long n, void* stream_) {
  clear_error();
  if (n <= 0 || !out || !target || !grad_loss || !dout) {
    set_error("gru_mse_loss_backward: need n >= 1 and non-null pointers");
    return GRU_ERR_INVALID;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int vec = (n % 4 == 0 && aligned16(out) && aligned16(target) && aligned16(dout)) ? 1 : 0;
  // torch: norm = 2 / numel as the tensor's type, grad = norm * (x - y) * g
  const float norm = (float)(2.0 / (double)n);
  LaunchScope scope(kKindLoss, stream);
  mse_backward_kernel<<<mse_blocks(n), kMseThreads, 0, stream>>>(out, target, grad_loss, norm, n, vec, dout);
  GRU_CUDA_TRY(cudaGetLastError());
  return GRU_OK;
}
