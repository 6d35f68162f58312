// gru_forward_inference_noalloc: the inference forward for callers that
// cannot allocate device memory.
//
// Some hosts of this library cannot hand it a workspace: plugins loaded into a
// process whose device memory is owned by someone else's allocator (calling
// cudaMalloc there would fragment or exceed a budget the host enforces), and
// code running where an allocation would stall or is not allowed.  For them
// this entry point runs the same forward as gru_forward(stash = NULL), but its
// scratch (always the input-gate buffer plus the TF32 hi/lo split copies of x
// and W_ih that feed the tensor-core projection) lives in one file-scope
// device array of GRU_NOALLOC_SCRATCH_BYTES that is part of the loaded module:
// every GPU that loads the library holds it until the process exits.  Nothing
// here calls cudaMalloc, cudaFree or an allocating library routine.
//
// The array's device address is looked up once per device ordinal and cached
// for the life of the process.  Resetting a device (cudaDeviceReset) or
// otherwise tearing down and recreating its primary context while the library
// stays loaded is not supported: the cached address would be stale.

#include <cuda_runtime.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {
namespace {

// Shared by every call on a device; keeps the last call's contents.  The
// forward overwrites every byte it reads from it before reading, so nothing
// needs clearing between calls.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GRU_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
std::map<int, void*> g_noalloc_ptr;  // device -> device address of g_noalloc_scratch

// The array's name in host code is only a host-side stand-in; the device
// address comes from cudaGetSymbolAddress, once per device with that device
// current.
int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_ptr.find(device);
  if (it != g_noalloc_ptr.end()) {
    *out = it->second;
    return GRU_OK;
  }
  void* p = nullptr;
  GRU_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  if (p == nullptr) {
    set_error("gru_forward_inference_noalloc: no device address for the static scratch");
    return GRU_ERR_CUDA;
  }
  g_noalloc_ptr[device] = p;
  *out = p;
  return GRU_OK;
}

}  // namespace
}  // namespace gru

using namespace gru;

extern "C" int gru_forward_inference_noalloc(const float* x, const float* h0, const float* w_ih,
                                             const float* w_hh, const float* b_ih, const float* b_hh,
                                             float* out, float* hn, int B, int T, int I, int H,
                                             void* stream) {
  clear_error();
  if (B < 0 || T < 0 || I < 1 || H < 1) {
    set_error("invalid shape: need B >= 0, T >= 0, I >= 1, H >= 1");
    return GRU_ERR_INVALID;
  }
  const size_t need = gru_forward_workspace_bytes(B, T, I, H);
  if (need > (size_t)GRU_NOALLOC_SCRATCH_BYTES) {
    set_error("gru_forward_inference_noalloc: this shape needs " + std::to_string(need) +
              " bytes of scratch, more than the static " + std::to_string((size_t)GRU_NOALLOC_SCRATCH_BYTES) +
              " (gru_forward_workspace_bytes(B, T, I, H) must fit); use gru_forward with a caller workspace");
    return GRU_ERR_UNSUPPORTED;
  }
  int dev = 0;
  GRU_CUDA_TRY(cudaGetDevice(&dev));
  void* scratch = nullptr;
  int rc = scratch_address(dev, &scratch);
  if (rc) return rc;
  return forward_impl(x, h0, w_ih, w_hh, b_ih, b_hh, out, hn, nullptr, scratch,
                      (size_t)GRU_NOALLOC_SCRATCH_BYTES, B, T, I, H, stream, false);
}
