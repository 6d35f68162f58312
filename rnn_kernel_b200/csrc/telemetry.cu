// Launch counting and opt-in CUDA-event timing per kernel kind (host code).

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

namespace {
std::atomic<unsigned long long> g_launches{0};
std::atomic<int> g_timing{0};
std::mutex g_tmu;
struct Rec {
  int kind;
  cudaEvent_t start, end;
};
std::vector<Rec> g_recs;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}
}  // namespace

LaunchScope::LaunchScope(int kind, cudaStream_t stream, int launches)
    : kind_(kind), stream_(stream), start_(nullptr) {
  g_launches.fetch_add(static_cast<unsigned long long>(launches));
  if (g_timing.load()) {
    std::lock_guard<std::mutex> lk(g_tmu);
    cudaEvent_t e = take_event();
    if (e && cudaEventRecord(e, stream) == cudaSuccess) start_ = e;
  }
}

LaunchScope::~LaunchScope() {
  if (!start_) return;
  std::lock_guard<std::mutex> lk(g_tmu);
  cudaEvent_t e = take_event();
  if (e && cudaEventRecord(e, stream_) == cudaSuccess) {
    g_recs.push_back(Rec{kind_, static_cast<cudaEvent_t>(start_), e});
  } else {
    g_pool.push_back(static_cast<cudaEvent_t>(start_));
    if (e) g_pool.push_back(e);
  }
}

}  // namespace gru

using namespace gru;

extern "C" {

unsigned long long gru_launch_count(void) { return g_launches.load(); }

int gru_timing_enable(int on) {
  g_timing.store(on ? 1 : 0);
  return GRU_OK;
}

int gru_timing_collect(double* total_ms, int* count, int n_kinds) {
  clear_error();
  std::lock_guard<std::mutex> lk(g_tmu);
  for (int k = 0; k < n_kinds; ++k) {
    if (total_ms) total_ms[k] = 0.0;
    if (count) count[k] = 0;
  }
  int rc = GRU_OK;
  for (const Rec& r : g_recs) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.end) != cudaSuccess ||
        cudaEventElapsedTime(&ms, r.start, r.end) != cudaSuccess) {
      set_error("gru_timing_collect: event query failed");
      cudaGetLastError();
      rc = GRU_ERR_CUDA;
    } else if (r.kind >= 0 && r.kind < n_kinds) {
      if (total_ms) total_ms[r.kind] += ms;
      if (count) count[r.kind] += 1;
    }
    g_pool.push_back(r.start);
    g_pool.push_back(r.end);
  }
  g_recs.clear();
  return rc;
}

}  // extern "C"
