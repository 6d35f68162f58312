// C ABI of the B200 GRU training path (declarations and contract in
// include/rnn_kernel_b200.h).

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "common.cuh"
#include "../../include/rnn_kernel_b200.h"

namespace gru {

namespace {
thread_local std::string g_last_error;
std::mutex g_mu;
std::map<std::tuple<int, int, int, int>, RecGeom> g_geom;  // (device, kind, B, H)
std::map<int, int> g_sms;

constexpr size_t kAlign = 256;

int geometry(int kind, int B, int T, int H, int device, RecGeom* out) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_geom.find(std::make_tuple(device, kind, B, H));
    if (it != g_geom.end()) {
      *out = it->second;
      out->T = T;
      return GRU_OK;
    }
  }
  RecGeom g{};
  const int rc = kind == 0 ? rec_forward_geometry(B, T, H, device, &g)
                           : rec_backward_geometry(B, T, H, device, &g);
  if (rc != GRU_OK) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  g_geom[std::make_tuple(device, kind, B, H)] = g;
  *out = g;
  return GRU_OK;
}

int check_shape(int B, int T, int I, int H) {
  if (B < 0 || T < 0 || I < 1 || H < 1) {
    set_error("invalid shape: need B >= 0, T >= 0, I >= 1, H >= 1");
    return GRU_ERR_INVALID;
  }
  if (H > 256) {
    set_error("hidden_size > 256 is not supported");
    return GRU_ERR_UNSUPPORTED;
  }
  return GRU_OK;
}

int current_device(int* dev) {
  GRU_CUDA_TRY(cudaGetDevice(dev));
  int major = 0;
  GRU_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev));
  if (major != 10) {
    set_error("rnn_kernel_b200 requires a compute capability 10.x (sm_100a) GPU");
    return GRU_ERR_UNSUPPORTED;
  }
  return GRU_OK;
}

inline int pad4(int v) { return (v + 3) / 4 * 4; }

struct FwdLayout {
  size_t g, xp, wp, total;
  bool pad;  // x / W_ih need a copy with a 16-byte row stride for TMA
};

FwdLayout fwd_layout(int B, int T, int I, int H) {
  const long BT = (long)B * T;
  FwdLayout l{};
  l.pad = (I % 4) != 0;
  size_t off = 0;
  l.g = off;
  off = align_up(off + sizeof(float) * BT * 3 * H, kAlign);
  // Room for 16-byte-stride copies of x and W_ih (I not a multiple of 4, or
  // caller buffers not 16-byte aligned).
  l.xp = off;
  off = align_up(off + sizeof(float) * BT * pad4(I), kAlign);
  l.wp = off;
  off = align_up(off + sizeof(float) * (size_t)3 * H * pad4(I), kAlign);
  l.total = off;
  return l;
}

struct BwdLayout {
  size_t dgi, dgh, wt, hp, xp, gemm, col, total;
  int ldgi;      // row stride of dG_ih / dG_hh (multiple of 4 floats for TMA)
  bool hp_copy;  // h_prev (stash stride 5H) needs a 16-byte-stride copy (H % 4 != 0)
  bool x_copy;   // x (stride I) needs a 16-byte-stride copy (I % 4 != 0)
};

BwdLayout bwd_layout(int B, int T, int I, int H, int device) {
  const long BT = (long)B * T;
  BwdLayout l{};
  l.ldgi = pad4(3 * H);
  size_t off = 0;
  l.dgi = off;
  off = align_up(off + sizeof(float) * BT * l.ldgi, kAlign);
  l.dgh = off;
  off = align_up(off + sizeof(float) * BT * l.ldgi, kAlign);
  l.wt = off;
  off = align_up(off + sizeof(float) * (size_t)I * l.ldgi, kAlign);
  l.hp_copy = H % 4 != 0;
  l.x_copy = I % 4 != 0;
  // Room for 16-byte-stride copies of h_prev and x, used when H or I is not a
  // multiple of 4 or the caller's buffers are not 16-byte aligned.
  l.hp = off;
  off = align_up(off + sizeof(float) * BT * pad4(H), kAlign);
  l.xp = off;
  off = align_up(off + sizeof(float) * BT * pad4(I), kAlign);
  l.gemm = off;
  // Split-K partials of the weight-gradient products.
  TcGemmArgs hh{nullptr, l.ldgi, nullptr, pad4(H), nullptr, H, nullptr, 3 * H, H, (int)BT, true, true};
  TcGemmArgs ih{nullptr, l.ldgi, nullptr, pad4(I), nullptr, I, nullptr, 3 * H, I, (int)BT, true, true};
  const size_t g = std::max(tc_gemm_ws_bytes(hh, device), tc_gemm_ws_bytes(ih, device));
  off = align_up(off + g, kAlign);
  l.col = off;
  off = align_up(off + bias_grad_ws_bytes(H), kAlign);
  l.total = off;
  return l;
}

}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

int sm_count(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_sms.find(device);
  if (it != g_sms.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) n = 148;
  g_sms[device] = n;
  return n;
}

}  // namespace gru

using namespace gru;

extern "C" {

const char* gru_last_error(void) { return g_last_error.c_str(); }

int gru_device_supported(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    cudaGetLastError();
    return 0;
  }
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return major == 10 ? 1 : 0;
}

int gru_device_status(int reset) {
  clear_error();
  int st = 0, st2 = 0;
  if (read_device_status(reset, &st) != GRU_OK) return -1;
  if (read_gemm_status(reset, &st2) != GRU_OK) return -1;
  return st | st2;
}

int gru_selftest_wait_timeout(int limit_ms, int* result, void* stream) {
  clear_error();
  if (limit_ms < 1 || limit_ms > 10000 || result == nullptr) {
    set_error("gru_selftest_wait_timeout: need 1 <= limit_ms <= 10000 and a result pointer");
    return GRU_ERR_INVALID;
  }
  return wait_probe((unsigned long long)limit_ms * 1000000ull, result, static_cast<cudaStream_t>(stream));
}

size_t gru_stash_bytes(int B, int T, int H) {
  if (B <= 0 || T <= 0 || H <= 0) return 0;
  return sizeof(float) * (size_t)B * T * 5 * H;
}

size_t gru_forward_workspace_bytes(int B, int T, int I, int H) {
  if (B <= 0 || T <= 0 || H <= 0 || I <= 0) return 0;
  return fwd_layout(B, T, I, H).total;
}

size_t gru_backward_workspace_bytes(int B, int T, int I, int H) {
  if (B <= 0 || T <= 0 || H <= 0 || I <= 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  return bwd_layout(B, T, I, H, dev).total;
}

int gru_forward(const float* x, const float* h0, const float* w_ih, const float* w_hh,
                const float* b_ih, const float* b_hh, float* out, float* hn, float* stash,
                void* workspace, size_t workspace_bytes, int B, int T, int I, int H,
                void* stream_) {
  clear_error();
  int rc = check_shape(B, T, I, H);
  if (rc) return rc;
  if (B == 0) return GRU_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!h0 || !hn || (T > 0 && (!x || !w_ih || !w_hh || !b_ih || !b_hh || !out))) {
    set_error("gru_forward: null tensor pointer");
    return GRU_ERR_INVALID;
  }
  int dev = 0;
  if ((rc = current_device(&dev))) return rc;
  if (T == 0) {
    GRU_CUDA_TRY(cudaMemcpyAsync(hn, h0, sizeof(float) * (size_t)B * H, cudaMemcpyDeviceToDevice, stream));
    return GRU_OK;
  }
  if (!workspace || workspace_bytes < gru_forward_workspace_bytes(B, T, I, H)) {
    set_error("gru_forward: workspace too small");
    return GRU_ERR_INVALID;
  }
  const FwdLayout l = fwd_layout(B, T, I, H);
  char* ws = static_cast<char*>(workspace);
  float* G = reinterpret_cast<float*>(ws + l.g);
  // G = x . W_ih^T + b_ih on the tensor cores (3xTF32).
  TcGemmArgs ga{x, I, w_ih, I, G, 3 * H, b_ih, B * T, 3 * H, I};
  if (l.pad || !tc_gemm_supported(ga)) {
    float* xp = reinterpret_cast<float*>(ws + l.xp);
    float* wp = reinterpret_cast<float*>(ws + l.wp);
    if ((rc = pad_rows(x, (long)B * T, I, I, xp, pad4(I), stream))) return rc;
    if ((rc = pad_rows(w_ih, 3L * H, I, I, wp, pad4(I), stream))) return rc;
    ga.A = xp;
    ga.lda = pad4(I);
    ga.B = wp;
    ga.ldb = pad4(I);
  }
  if ((rc = tc_gemm(ga, stream, kKindInputGemm))) return rc;
  RecGeom g{};
  if ((rc = geometry(0, B, T, H, dev, &g))) return rc;
  return launch_rec_forward(G, h0, w_hh, b_hh, out, hn, stash, g, stream);
}

int gru_backward(const float* dout, const float* dhn, const float* x, const float* w_ih,
                 const float* w_hh, const float* stash, float* dx, float* dh0, float* dw_ih,
                 float* dw_hh, float* db_ih, float* db_hh, void* workspace,
                 size_t workspace_bytes, int B, int T, int I, int H, void* stream_) {
  clear_error();
  int rc = check_shape(B, T, I, H);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!dw_ih || !dw_hh || !db_ih || !db_hh || (B > 0 && !dh0)) {
    set_error("gru_backward: null gradient pointer");
    return GRU_ERR_INVALID;
  }
  int dev = 0;
  if ((rc = current_device(&dev))) return rc;
  if (B == 0 || T == 0) {
    GRU_CUDA_TRY(cudaMemsetAsync(dw_ih, 0, sizeof(float) * 3 * H * (size_t)I, stream));
    GRU_CUDA_TRY(cudaMemsetAsync(dw_hh, 0, sizeof(float) * 3 * H * (size_t)H, stream));
    GRU_CUDA_TRY(cudaMemsetAsync(db_ih, 0, sizeof(float) * 3 * H, stream));
    GRU_CUDA_TRY(cudaMemsetAsync(db_hh, 0, sizeof(float) * 3 * H, stream));
    if (B > 0) {
      if (dhn) GRU_CUDA_TRY(cudaMemcpyAsync(dh0, dhn, sizeof(float) * (size_t)B * H, cudaMemcpyDeviceToDevice, stream));
      else GRU_CUDA_TRY(cudaMemsetAsync(dh0, 0, sizeof(float) * (size_t)B * H, stream));
    }
    return GRU_OK;
  }
  if (!x || !w_ih || !w_hh || !stash) {
    set_error("gru_backward: null input pointer");
    return GRU_ERR_INVALID;
  }
  const BwdLayout l = bwd_layout(B, T, I, H, dev);
  if (!workspace || workspace_bytes < l.total) {
    set_error("gru_backward: workspace too small");
    return GRU_ERR_INVALID;
  }
  char* ws = static_cast<char*>(workspace);
  float* dGi = reinterpret_cast<float*>(ws + l.dgi);
  float* dGh = reinterpret_cast<float*>(ws + l.dgh);
  void* gws = ws + l.gemm;
  const size_t gws_bytes = l.col - l.gemm;
  float* wt = reinterpret_cast<float*>(ws + l.wt);
  RecGeom g{};
  if ((rc = geometry(1, B, T, H, dev, &g))) return rc;
  if ((rc = launch_rec_backward(dout, dhn, w_hh, stash, dGi, l.ldgi, dGh, dh0, g, stream))) return rc;

  const int BT = B * T;
  const int H3 = 3 * H;
  // dW_hh = dG_hh^T . h_prev (h_prev = stash column block 4), dW_ih = dG_ih^T . x,
  // on the tensor cores; operands without a 16-byte row stride are first
  // copied into padded buffers.
  const float* hp = stash + 4 * H;
  long ldhp = 5L * H;
  if (l.hp_copy || (reinterpret_cast<uintptr_t>(hp) & 15)) {
    float* hpp = reinterpret_cast<float*>(ws + l.hp);
    if ((rc = pad_rows(hp, BT, H, 5L * H, hpp, pad4(H), stream))) return rc;
    hp = hpp;
    ldhp = pad4(H);
  }
  const float* xx = x;
  long ldx = I;
  if (l.x_copy || (reinterpret_cast<uintptr_t>(x) & 15)) {
    float* xpp = reinterpret_cast<float*>(ws + l.xp);
    if ((rc = pad_rows(x, BT, I, I, xpp, pad4(I), stream))) return rc;
    xx = xpp;
    ldx = pad4(I);
  }
  TcGemmArgs hh{dGh, l.ldgi, hp, ldhp, dw_hh, H, nullptr, H3, H, BT, true, true};
  TcGemmArgs ih{dGi, l.ldgi, xx, ldx, dw_ih, I, nullptr, H3, I, BT, true, true};
  if ((rc = tc_gemm(hh, stream, kKindGradGemm, gws, gws_bytes))) return rc;
  if ((rc = tc_gemm(ih, stream, kKindGradGemm, gws, gws_bytes))) return rc;
  if (dx) {
    // dx = dG_ih . W_ih on the tensor cores, with W_ih^T staged as [I, ldgi].
    if ((rc = transpose(w_ih, H3, I, wt, l.ldgi, stream))) return rc;
    TcGemmArgs a3{dGi, l.ldgi, wt, l.ldgi, dx, I, nullptr, BT, I, H3};
    if ((rc = tc_gemm(a3, stream, kKindGradGemm))) return rc;
  }
  if ((rc = bias_grads(dGi, dGh, BT, H, l.ldgi, db_ih, db_hh, ws + l.col, stream))) return rc;
  return GRU_OK;
}

}  // extern "C"
