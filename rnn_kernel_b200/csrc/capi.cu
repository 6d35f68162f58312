// C ABI of the B200 GRU training path (declarations and contract in
// include/rnn_kernel_b200.h).

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
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
std::map<std::tuple<int, int, int, int, int>, RecGeom> g_geom;  // (device, kind, B, H, small-loops mode)
std::map<int, int> g_sms;

constexpr size_t kAlign = 256;

// Time chunks.  The time loops occupy C * nclusters SMs (e.g. 104 of 148 at
// H = 256, B = 64), so while one chunk of the sequence runs, the tensor-core
// products of another chunk run on the idle SMs from a side stream: in the
// forward the input projection of chunk c+1 beside the loop over chunk c, in
// the backward the weight-gradient (and dx) products of chunk c beside the
// loop over chunk c-1.  A chunk is a multiple of 128 steps (whole M tiles of
// the projection per batch row).
constexpr int kMaxChunks = 4;
std::atomic<int> g_time_chunks{0};  // 0: automatic, 1: off, 2..kMaxChunks: that many when possible

// Automatic choice (two chunks or none) from a cost estimate: the chunked
// run saves the tensor-core time of one half of the products on the whole
// GPU, loses whatever the side half takes beyond the loop over the other
// half, and pays one more loop launch (measured ~15-30 us: prologue and
// pipeline fill).  Rates are conservative measurements at I = H = 256: the
// 3xTF32 products ~0.7 TFLOP/s (FP32-equivalent) per SM, a time-loop step
// ~1.6 us per GEMV sub-chunk of <= 8 rows.
constexpr double kGemmFlopsPerSm = 0.7e12;
constexpr double kStepSecondsPerSubchunk = 1.6e-6;
constexpr double kBoundarySeconds = 30e-6;

// side_flops: the FLOPs of the products that can move to the side stream,
// over the whole sequence.
int time_chunks(const RecGeom& g, int device, double side_flops) {
  const int knob = g_time_chunks.load();
  if (knob == 1 || g.small) return 1;  // the single-CTA loops of small H are too short to hide products
  const int sms = sm_count(device);
  const int free = sms - g.C * g.nclusters;
  if (g.nclusters > g.max_clusters || free < 1) return 1;
  if (knob >= 2) return (knob <= kMaxChunks && g.T % (128 * knob) == 0) ? knob : 1;
  if (g.T % 256 != 0) return 1;
  const double half = 0.5 * side_flops;
  const double on_all = half / (sms * kGemmFlopsPerSm);
  const double on_free = half / (free * kGemmFlopsPerSm);
  const double loop_half = 0.5 * g.T * (g.bcp / g.R) * kStepSecondsPerSubchunk;
  const double gain = on_all - std::max(0.0, on_free - loop_half) - kBoundarySeconds;
  return gain > 0.0 ? 2 : 1;
}

// One non-blocking side stream per host thread and device (default, i.e.
// lowest, priority) with a fork and a join event.  Created outside stream
// capture only: while the caller's stream is capturing and no side stream
// exists yet, the call runs without time chunks.
struct Side {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
thread_local std::map<int, Side> t_side;

int side_stream(int device, cudaStream_t main, Side** out) {
  *out = nullptr;
  auto it = t_side.find(device);
  if (it != t_side.end()) {
    *out = &it->second;
    return GRU_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  GRU_CUDA_TRY(cudaStreamIsCapturing(main, &cs));
  if (cs != cudaStreamCaptureStatusNone) return GRU_OK;
  Side sd;
  GRU_CUDA_TRY(cudaStreamCreateWithFlags(&sd.s, cudaStreamNonBlocking));
  GRU_CUDA_TRY(cudaEventCreateWithFlags(&sd.fork, cudaEventDisableTiming));
  GRU_CUDA_TRY(cudaEventCreateWithFlags(&sd.join, cudaEventDisableTiming));
  *out = &(t_side[device] = sd);
  return GRU_OK;
}
// `to` waits for everything issued so far on `from`.
int stream_after(cudaStream_t to, cudaStream_t from, cudaEvent_t ev) {
  GRU_CUDA_TRY(cudaEventRecord(ev, from));
  GRU_CUDA_TRY(cudaStreamWaitEvent(to, ev, 0));
  return GRU_OK;
}

int geometry(int kind, int B, int T, int H, int device, RecGeom* out) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_geom.find(std::make_tuple(device, kind, B, H, small_loops_mode()));
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
  g_geom[std::make_tuple(device, kind, B, H, small_loops_mode())] = g;
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

// Workspace layouts.  The tensor-core products take pre-split operands
// (hi = tf32(v), lo = tf32(v - hi)) with 16-byte row strides, so the
// workspaces hold split copies of x, W_ih and h_prev, and the backward time
// loop writes dG_ih / dG_hh already split.
struct FwdLayout {
  size_t g, xh, xl, wh, wl, total;
  int ldx;  // row stride of the split x / W_ih copies (I rounded up to 4)
  int ldg;  // row stride of the input gates G (3H rounded up to 4: 16-byte rows)
};

FwdLayout fwd_layout(int B, int T, int I, int H) {
  const long BT = (long)B * T;
  FwdLayout l{};
  l.ldx = pad4(I);
  l.ldg = pad4(3 * H);
  size_t off = 0;
  l.g = off;
  off = align_up(off + sizeof(float) * BT * l.ldg, kAlign);
  l.xh = off;
  off = align_up(off + sizeof(float) * BT * l.ldx, kAlign);
  l.xl = off;
  off = align_up(off + sizeof(float) * BT * l.ldx, kAlign);
  l.wh = off;
  off = align_up(off + sizeof(float) * (size_t)3 * H * l.ldx, kAlign);
  l.wl = off;
  off = align_up(off + sizeof(float) * (size_t)3 * H * l.ldx, kAlign);
  l.total = off;
  return l;
}

struct BwdLayout {
  size_t dgih, dgil, dghh, dghl, wt, wth, wtl, hph, hpl, xh, xl, gemm, col, total;
  int ldgi;  // row stride of dG_ih / W_ih^T (3H rounded up to 4)
  int ldh;   // row stride of the split h_prev copy and of dG_hh's n block (H rounded up to 4)
  int ldx;   // row stride of the split x copy (I rounded up to 4)
};

BwdLayout bwd_layout(int B, int T, int I, int H, int device) {
  const long BT = (long)B * T;
  BwdLayout l{};
  l.ldgi = pad4(3 * H);
  l.ldh = pad4(H);
  l.ldx = pad4(I);
  size_t off = 0;
  auto take = [&](size_t& at, size_t floats) {
    at = off;
    off = align_up(off + sizeof(float) * floats, kAlign);
  };
  take(l.dgih, (size_t)BT * l.ldgi);
  take(l.dgil, (size_t)BT * l.ldgi);
  // only dG_hh's n block: its r and z columns are dG_ih's
  take(l.dghh, (size_t)BT * l.ldh);
  take(l.dghl, (size_t)BT * l.ldh);
  take(l.wt, (size_t)I * l.ldgi);
  take(l.wth, (size_t)I * l.ldgi);
  take(l.wtl, (size_t)I * l.ldgi);
  take(l.hph, (size_t)BT * l.ldh);
  take(l.hpl, (size_t)BT * l.ldh);
  take(l.xh, (size_t)BT * l.ldx);
  take(l.xl, (size_t)BT * l.ldx);
  // Split-K partials of the weight-gradient products.
  // (the three products gru_backward runs: dW_hh r/z rows, dW_hh n rows, dW_ih)
  TcGemmArgs hrz{nullptr, l.ldgi, nullptr, l.ldh, nullptr, H, nullptr, 2 * H, H, (int)BT, true, true};
  TcGemmArgs hn{nullptr, l.ldh, nullptr, l.ldh, nullptr, H, nullptr, H, H, (int)BT, true, true};
  TcGemmArgs ih{nullptr, l.ldgi, nullptr, l.ldx, nullptr, I, nullptr, 3 * H, I, (int)BT, true, true};
  l.gemm = off;
  const TcGemmArgs grads[3] = {hrz, hn, ih};
  // With time chunks the three products are split per chunk (partial slices
  // of every chunk, summed at the end): room for the largest such plan.  The
  // split counts grow with the grid, so the full grid bounds them.
  size_t chunked = 0;
  for (int n = 2; n <= kMaxChunks; ++n) {
    if (T % (128 * n) != 0) continue;
    TcGemmArgs c[3] = {hrz, hn, ih};
    for (auto& x : c) x.K = (int)(BT / n);
    int sp[3];
    tc_partial_splits(c, 3, sm_count(device), sp);
    size_t bytes = 0;
    for (int i = 0; i < 3; ++i) bytes += align_up(sizeof(float) * (size_t)n * sp[i] * c[i].M * pad4(c[i].N), kAlign);
    chunked = std::max(chunked, bytes);
  }
  off = align_up(off + std::max(tc_gemm_ws_bytes(grads, 3, device), chunked), kAlign);
  // per-cluster FP64 bias-gradient partials written by the backward time loop
  // (one row set per time chunk), sized for B clusters per chunk (an upper
  // bound that needs no device query)
  l.col = off;
  off = align_up(off + sizeof(double) * (size_t)kMaxChunks * B * 4 * H, kAlign);
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

// The backward over time chunks (see time_chunks): the loop runs the chunks
// from the last to the first, the dh state passing between them through
// dh0; the weight-gradient products (and dx) of every chunk but the first
// run on the side stream beside the loop over the next earlier chunk, as
// partial slices that one final launch sums.
int backward_chunked(const float* dout, const float* dhn, const float* x, const float* w_ih, const float* w_hh,
                     const float* stash, float* dx, float* dh0, float* dw_ih, float* dw_hh, float* db_ih,
                     float* db_hh, char* ws, const BwdLayout& l, const RecGeom& g, int nch, const Side& sd, int B,
                     int T, int I, int H, int dev, cudaStream_t stream) {
  auto F = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  double* dbpart = reinterpret_cast<double*>(ws + l.col);
  const int Tc = T / nch, H3 = 3 * H;
  const int free = sm_count(dev) - g.C * g.nclusters;
  int rc;
  const SplitArgs sp[2] = {{stash + 4 * H, (long)B * T, H, 5L * H, F(l.hph), F(l.hpl), l.ldh},
                           {x, (long)B * T, I, I, F(l.xh), F(l.xl), l.ldx}};
  // Products of chunk c (rows b*T + t for t in [c*Tc, c*Tc + Tc)).
  TcGemmArgs full[3] = {
      {F(l.dgih), l.ldgi, F(l.hph), l.ldh, dw_hh, H, nullptr, 2 * H, H, B * T, true, true, F(l.dgil), F(l.hpl)},
      {F(l.dghh), l.ldh, F(l.hph), l.ldh, dw_hh + 2L * H * H, H, nullptr, H, H, B * T, true, true, F(l.dghl),
       F(l.hpl)},
      {F(l.dgih), l.ldgi, F(l.xh), l.ldx, dw_ih, I, nullptr, H3, I, B * T, true, true, F(l.dgil), F(l.xl)}};
  float* part[3];
  long ldp[3];
  int zoff[3] = {0, 0, 0};
  {
    char* p = ws + l.gemm;
    int spmax[3];
    TcGemmArgs c[3] = {full[0], full[1], full[2]};
    for (auto& a : c) a.K = B * Tc;
    tc_partial_splits(c, 3, sm_count(dev), spmax);
    for (int i = 0; i < 3; ++i) {
      part[i] = reinterpret_cast<float*>(p);
      ldp[i] = pad4(full[i].N);
      p += align_up(sizeof(float) * (size_t)nch * spmax[i] * full[i].M * ldp[i], kAlign);
    }
  }
  auto products = [&](int c, cudaStream_t s, int ctas) -> int {
    const size_t t0 = (size_t)c * Tc;
    TcGemmArgs a[3] = {full[0], full[1], full[2]};
    for (auto& q : a) {
      q.K = B * Tc;
      q.rin = Tc;
      q.rstride = T;
    }
    a[0].A = F(l.dgih) + t0 * l.ldgi, a[0].A_lo = F(l.dgil) + t0 * l.ldgi;
    a[0].B = F(l.hph) + t0 * l.ldh, a[0].B_lo = F(l.hpl) + t0 * l.ldh;
    a[1].A = F(l.dghh) + t0 * l.ldh, a[1].A_lo = F(l.dghl) + t0 * l.ldh;
    a[1].B = a[0].B, a[1].B_lo = a[0].B_lo;
    a[2].A = a[0].A, a[2].A_lo = a[0].A_lo;
    a[2].B = F(l.xh) + t0 * l.ldx, a[2].B_lo = F(l.xl) + t0 * l.ldx;
    if (int r = tc_gemm_partials(a, 3, s, kKindGradGemm, ctas, part, ldp, zoff)) return r;
    if (dx) {
      // dx rows of chunk c = dG_ih rows . W_ih, with W_ih^T staged as [I, ldgi]
      TcGemmArgs d{F(l.dgih) + t0 * l.ldgi, l.ldgi, F(l.wth), l.ldgi, dx + t0 * I, I, nullptr, B * Tc, I, H3,
                   false, false, F(l.dgil) + t0 * l.ldgi, F(l.wtl)};
      d.rin = Tc;
      d.rstride = T;
      if (int r = tc_gemm(d, s, kKindGradGemm, nullptr, 0, ctas)) return r;
    }
    return GRU_OK;
  };
  // Every loop is issued before the side work that runs beside it, so that
  // the loop's clusters are placed first; the side stream waits on the fork
  // event as recorded before that loop was issued.
  GRU_CUDA_TRY(cudaEventRecord(sd.fork, stream));
  for (int c = nch - 1; c >= 0; --c) {
    if ((rc = launch_rec_backward(dout, c == nch - 1 ? dhn : dh0, w_hh, stash, F(l.dgih), F(l.dgil), l.ldgi,
                                  F(l.dghh), F(l.dghl), l.ldh, dh0, dbpart + (size_t)(nch - 1 - c) * g.nclusters * 4 * H,
                                  g, stream, c * Tc, Tc)))
      return rc;
    GRU_CUDA_TRY(cudaStreamWaitEvent(sd.s, sd.fork, 0));
    if (c == nch - 1) {
      // the split copies of h_prev and x (and W_ih^T for dx) beside the first loop
      if ((rc = split_tf32_multi(sp, 2, sd.s))) return rc;
      if (dx) {
        if ((rc = transpose(w_ih, H3, I, F(l.wt), l.ldgi, sd.s))) return rc;
        if ((rc = split_tf32(F(l.wt), I, l.ldgi, l.ldgi, F(l.wth), F(l.wtl), l.ldgi, sd.s))) return rc;
      }
    } else {
      // chunk c+1's products beside the loop over chunk c
      if ((rc = products(c + 1, sd.s, free))) return rc;
    }
    GRU_CUDA_TRY(cudaEventRecord(sd.fork, stream));
  }
  if ((rc = stream_after(stream, sd.s, sd.join))) return rc;
  if ((rc = products(0, stream, 0))) return rc;
  int ns[3] = {zoff[0], zoff[1], zoff[2]};
  if ((rc = tc_gemm_sum(full, 3, part, ldp, ns, stream, kKindGradGemm))) return rc;
  return bias_grads_finish(dbpart, nch * g.nclusters, H, db_ih, db_hh, stream);
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

int gru_set_small_loops(int mode) { return set_small_loops(mode); }

int gru_set_time_chunks(int n) {
  if (n < 0 || n > kMaxChunks) return -1;
  return g_time_chunks.exchange(n);
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
  return gru::forward_impl(x, h0, w_ih, w_hh, b_ih, b_hh, out, hn, stash, workspace, workspace_bytes, B, T, I, H,
                           stream_, true);
}

}  // extern "C"

namespace gru {

int forward_impl(const float* x, const float* h0, const float* w_ih, const float* w_hh, const float* b_ih,
                 const float* b_hh, float* out, float* hn, float* stash, void* workspace, size_t workspace_bytes,
                 int B, int T, int I, int H, void* stream_, bool overlap) {
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
  float* xh = reinterpret_cast<float*>(ws + l.xh);
  float* xl = reinterpret_cast<float*>(ws + l.xl);
  float* wh = reinterpret_cast<float*>(ws + l.wh);
  float* wl = reinterpret_cast<float*>(ws + l.wl);
  // G = x . W_ih^T + b_ih on the tensor cores (3xTF32, pre-split operands).
  const SplitArgs sp[2] = {{x, (long)B * T, I, I, xh, xl, l.ldx}, {w_ih, 3L * H, I, I, wh, wl, l.ldx}};
  TcGemmArgs ga{xh, l.ldx, wh, l.ldx, G, l.ldg, b_ih, B * T, 3 * H, I, false, false, xl, wl};
  RecGeom g{};
  if ((rc = geometry(0, B, T, H, dev, &g))) return rc;
  const int nch = overlap ? time_chunks(g, dev, 2.0 * B * T * 3.0 * H * I) : 1;
  Side* sd = nullptr;
  if (nch > 1 && (rc = side_stream(dev, stream, &sd))) return rc;
  if (nch == 1 || sd == nullptr) {
    if ((rc = split_tf32_multi(sp, 2, stream))) return rc;
    if ((rc = tc_gemm(ga, stream, kKindInputGemm))) return rc;
    return launch_rec_forward(G, l.ldg, h0, w_hh, b_hh, out, hn, stash, g, stream);
  }
  // Time chunks: the projection of chunk 0 on the whole GPU, then the loop
  // over chunk c beside the projection of chunk c+1 (side stream, on the SMs
  // the loop leaves idle).  The state passes between chunks through hn.
  const int Tc = T / nch;
  const int free = sm_count(dev) - g.C * g.nclusters;
  auto chunk = [&](int c) {
    TcGemmArgs a = ga;
    a.A = xh + (size_t)c * Tc * l.ldx;
    a.A_lo = xl + (size_t)c * Tc * l.ldx;
    a.C = G + (size_t)c * Tc * l.ldg;
    a.M = B * Tc;
    a.rin = Tc;
    a.rstride = T;
    return a;
  };
  // The split copy of x is made per chunk too (chunk c's rows, periodic like
  // the projection's), chunk 0's with W_ih's before the first projection.
  auto split_x = [&](int c) {
    SplitArgs a = sp[0];
    a.src = x + (size_t)c * Tc * I;
    a.hi = xh + (size_t)c * Tc * l.ldx;
    a.lo = xl + (size_t)c * Tc * l.ldx;
    a.rows = (long)B * Tc;
    a.rin = Tc;
    a.rstride = T;
    return a;
  };
  const SplitArgs sp0[2] = {split_x(0), sp[1]};
  if ((rc = split_tf32_multi(sp0, 2, stream))) return rc;
  // Every loop is issued before the product that runs beside it, so that
  // the loop's clusters are placed first.
  if ((rc = tc_gemm(chunk(0), stream, kKindInputGemm))) return rc;
  GRU_CUDA_TRY(cudaEventRecord(sd->fork, stream));
  for (int c = 0; c < nch; ++c) {
    if ((rc = launch_rec_forward(G, l.ldg, c == 0 ? h0 : hn, w_hh, b_hh, out, hn, stash, g, stream, c * Tc, Tc)))
      return rc;
    if (c + 1 < nch) {
      if (c == 0) GRU_CUDA_TRY(cudaStreamWaitEvent(sd->s, sd->fork, 0));
      const SplitArgs spc = split_x(c + 1);
      if ((rc = split_tf32_multi(&spc, 1, sd->s))) return rc;
      if ((rc = tc_gemm(chunk(c + 1), sd->s, kKindInputGemm, nullptr, 0, free))) return rc;
      if ((rc = stream_after(stream, sd->s, sd->join))) return rc;  // the loop over chunk c+1 needs it
    }
  }
  return GRU_OK;
}

}  // namespace gru

extern "C" {

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
  RecGeom g{};
  if ((rc = geometry(1, B, T, H, dev, &g))) return rc;
  const BwdLayout l = bwd_layout(B, T, I, H, dev);
  if (!workspace || workspace_bytes < l.total) {
    set_error("gru_backward: workspace too small");
    return GRU_ERR_INVALID;
  }
  char* ws = static_cast<char*>(workspace);
  auto F = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  void* gws = ws + l.gemm;
  const size_t gws_bytes = l.col - l.gemm;
  double* dbpart = reinterpret_cast<double*>(ws + l.col);
  const int BT = B * T;
  const int H3 = 3 * H;
  const int nch = time_chunks(g, dev, 2.0 * B * T * 3.0 * H * (H + I + (dx ? I : 0)));
  Side* sd = nullptr;
  if (nch > 1 && (rc = side_stream(dev, stream, &sd))) return rc;
  if (nch > 1 && sd != nullptr)
    return backward_chunked(dout, dhn, x, w_ih, w_hh, stash, dx, dh0, dw_ih, dw_hh, db_ih, db_hh, ws, l, g, nch, *sd,
                            B, T, I, H, dev, stream);
  if ((rc = launch_rec_backward(dout, dhn, w_hh, stash, F(l.dgih), F(l.dgil), l.ldgi, F(l.dghh), F(l.dghl), l.ldh,
                                dh0, dbpart, g, stream)))
    return rc;

  // dW_hh = dG_hh^T . h_prev (h_prev = stash column block 4), dW_ih = dG_ih^T . x
  // on the tensor cores from pre-split copies.  dW_hh's r/z rows come from
  // dG_ih's r/z columns, its n rows from the separate n block.
  const SplitArgs sp[2] = {{stash + 4 * H, BT, H, 5L * H, F(l.hph), F(l.hpl), l.ldh},
                           {x, BT, I, I, F(l.xh), F(l.xl), l.ldx}};
  if ((rc = split_tf32_multi(sp, 2, stream))) return rc;
  TcGemmArgs hrz{F(l.dgih), l.ldgi, F(l.hph), l.ldh, dw_hh, H, nullptr, 2 * H, H, BT, true, true, F(l.dgil), F(l.hpl)};
  TcGemmArgs hn{F(l.dghh), l.ldh, F(l.hph), l.ldh, dw_hh + 2L * H * H, H, nullptr, H, H, BT, true, true, F(l.dghl),
                F(l.hpl)};
  TcGemmArgs ih{F(l.dgih), l.ldgi, F(l.xh), l.ldx, dw_ih, I, nullptr, H3, I, BT, true, true, F(l.dgil), F(l.xl)};
  const TcGemmArgs grads[3] = {hrz, hn, ih};
  if ((rc = tc_gemm_batch(grads, 3, stream, kKindGradGemm, gws, gws_bytes))) return rc;
  if (dx) {
    // dx = dG_ih . W_ih, with W_ih^T staged (and split) as [I, ldgi].
    if ((rc = transpose(w_ih, H3, I, F(l.wt), l.ldgi, stream))) return rc;
    if ((rc = split_tf32(F(l.wt), I, l.ldgi, l.ldgi, F(l.wth), F(l.wtl), l.ldgi, stream))) return rc;
    TcGemmArgs a3{F(l.dgih), l.ldgi, F(l.wth), l.ldgi, dx, I, nullptr, BT, I, H3, false, false, F(l.dgil), F(l.wtl)};
    if ((rc = tc_gemm(a3, stream, kKindGradGemm))) return rc;
  }
  if ((rc = bias_grads_finish(dbpart, g.nclusters, H, db_ih, db_hh, stream))) return rc;
  return GRU_OK;
}

}  // extern "C"
