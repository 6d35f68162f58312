// Shared helpers for the rnn_kernel_b200 CUDA sources (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include <string>

namespace gru {

// Per-thread last-error text behind gru_last_error().
void set_error(const std::string& msg);
void clear_error();

#define GRU_CUDA_TRY(expr)                                                          \
  do {                                                                              \
    cudaError_t err__ = (expr);                                                     \
    if (err__ != cudaSuccess) {                                                     \
      ::gru::set_error(std::string("CUDA error: ") + cudaGetErrorString(err__) +    \
                       " at " #expr);                                               \
      return GRU_ERR_CUDA;                                                          \
    }                                                                               \
  } while (0)

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// Recurrent-kernel geometry.  One GRU layer's time loop runs on independent
// thread-block clusters; every cluster owns `bc` batch rows and keeps the whole
// W_hh distributed over its C CTAs (CTA c owns hidden units [c*Hc, c*Hc+Hc),
// i.e. the rows r/z/n of those units).
// ---------------------------------------------------------------------------
struct RecGeom {
  int B, T, H;
  int C;    // CTAs per cluster (ceil(H/32), 1..8)
  int Hc;   // hidden units owned by one CTA (<= 32)
  int nw;   // warps per CTA = ceil(H/32): warp w covers k in [32w, 32w+32)
  int bc;   // batch rows per cluster
  int R;    // batch rows per GEMV sub-chunk (<= kMaxRows)
  int bcp;  // bc rounded up to a multiple of R
  int pd;   // prefetch depth of the per-step input ring (steps in flight)
  int nclusters;
  int max_clusters;  // clusters of this kernel resident at once on the device
  // Shared-memory layout, offsets in floats from the dynamic base; every
  // region starts on a 16-byte boundary (float4 accesses).
  int off1, off2, off3, off4;
  int vec4;  // per-step input rows are 16-byte aligned (H, Hc multiples of 4)
  int small;  // 1: the single-CTA kernels for H <= 96 (C = 1, nclusters = CTAs, R = rows per CTA)
  size_t smem;  // dynamic shared memory bytes per CTA
};

constexpr int kMaxRows = 8;     // largest GEMV sub-chunk (batch rows)
constexpr int kMaxCluster = 8;  // CTAs per cluster for H <= 256

int read_device_status(int reset, int* status);
int wait_probe(unsigned long long limit_ns, int* result_dev, cudaStream_t stream);
// Single-CTA time loops (forward H <= 96, backward H <= 64): 0 = on (default),
// 1 = the cluster kernels everywhere.  Process-wide; returns the previous mode, -1 if invalid.
int set_small_loops(int mode);
int small_loops_mode();
int rec_forward_geometry(int B, int T, int H, int device, RecGeom* g);
int rec_backward_geometry(int B, int T, int H, int device, RecGeom* g);

// G: input gates [B*T rows, 3H], row stride ldg floats.  Both time loops
// run the steps [t0, t0 + nt) (nt < 0: the whole sequence); the state enters
// through h0 / dhn and leaves through hn / dh0, so a sequence can be run as
// consecutive time chunks.
int launch_rec_forward(const float* G, int ldg, const float* h0, const float* w_hh, const float* b_hh,
                       float* out, float* hn, float* stash, const RecGeom& g,
                       cudaStream_t stream, int t0 = 0, int nt = -1);
// dG_ih [rows, 3H] (row stride ldgi) and the n block of dG_hh [rows, H] (row
// stride ldgn) are written pre-split (hi, lo).
int launch_rec_backward(const float* dout, const float* dhn, const float* w_hh,
                        const float* stash, float* dGi, float* dGi_lo, int ldgi, float* dGh, float* dGh_lo,
                        int ldgn, float* dh0, double* dbpart,
                        const RecGeom& g, cudaStream_t stream, int t0 = 0, int nt = -1);

// Tensor-core (tcgen05, 3xTF32) product C[m, n] = sum_k A(m, k) B(n, k) (+ bias).
// The operands come pre-split: A / A_lo hold tf32(a) and tf32(a - tf32(a))
// (round to nearest) with the same layout, likewise B / B_lo.
// K-major operand (a_mn = false): A [M, K] row-major, row stride lda.
// MN-major operand (a_mn = true): A stored [K, M] row-major (K is the row),
// row stride lda; same for B with N.  C [M, N], row stride ldc.  Operands
// must be 16-byte aligned and lda, ldb multiples of 4 floats (TMA);
// tc_gemm_supported() checks that.  With ws != null and a long K the product
// is split over K (partials in ws, FP64 reduce; bias must then be null).
struct TcGemmArgs {
  const float* A; long lda;
  const float* B; long ldb;
  float* C; long ldc;
  const float* bias;
  int M, N, K;
  bool a_mn = false, b_mn = false;
  const float* A_lo = nullptr;
  const float* B_lo = nullptr;
  // Periodic rows: the operands whose rows are the B*T (batch, step) rows --
  // A (its M rows when K-major, its K rows when MN-major), B when MN-major,
  // and C when A is K-major -- hold logical row r at physical row
  // (r / rin) * rstride + r % rin: with the pointers offset by t0 rows,
  // rin = steps of a time chunk and rstride = T select that chunk's rows of
  // every batch row.  rin = 0: plain rows.
  int rin = 0;
  long rstride = 0;
};
// hi[r, c] = tf32(src[r, c]), lo[r, c] = tf32(src - hi) for c < cols, 0 for
// cols <= c < ldd; src row stride lds, outputs row stride ldd.
int split_tf32(const float* src, long rows, int cols, long lds, float* hi, float* lo, int ldd, cudaStream_t stream);
// Several such splits in one launch (1 to 4).
struct SplitArgs {
  const float* src;
  long rows;
  int cols;
  long lds;
  float* hi;
  float* lo;
  int ldd;
  // Periodic rows (as TcGemmArgs::rin): logical row r of src and of hi / lo
  // is physical row (r / rin) * rstride + r % rin; rin = 0: plain rows.
  int rin = 0;
  long rstride = 0;
};
int split_tf32_multi(const SplitArgs* a, int n, cudaStream_t stream);
bool tc_gemm_supported(const TcGemmArgs& a);
size_t tc_gemm_ws_bytes(const TcGemmArgs& a, int device);
// ctas > 0 caps the persistent grid (the rest of the SMs stay free for work
// running concurrently on another stream).
int tc_gemm(const TcGemmArgs& a, cudaStream_t stream, int kind, void* ws = nullptr, size_t ws_bytes = 0,
            int ctas = 0);
// 1 to 3 products with the same operand majors in ONE launch (a persistent
// grid over all of their tiles and K splits) plus one launch summing all
// split-K partials; the workspace holds every product's partials.
size_t tc_gemm_ws_bytes(const TcGemmArgs* a, int n, int device);
int tc_gemm_batch(const TcGemmArgs* a, int n, cudaStream_t stream, int kind, void* ws, size_t ws_bytes,
                  int ctas = 0);
// Partial products without the final sum, for products summed over several
// launches (e.g. one per time chunk): problem i is split over K into
// splits[i] pieces (tc_partial_splits, for a grid of `ctas` CTAs) written as
// slices zoff[i], zoff[i] + 1, ... of part[i] ([slice][M][ldp[i]] floats);
// zoff[i] advances by the slices written.  tc_gemm_sum then writes
// C = sum of the first nslices[i] slices (FP64, fixed order).
int tc_partial_splits(const TcGemmArgs* a, int n, int ctas, int* splits);
int tc_gemm_partials(const TcGemmArgs* a, int n, cudaStream_t stream, int kind, int ctas, float* const* part,
                     const long* ldp, int* zoff);
int tc_gemm_sum(const TcGemmArgs* a, int n, const float* const* part, const long* ldp, const int* nslices,
                cudaStream_t stream, int kind);
bool tc_rows_ok(const TcGemmArgs& a);
int read_gemm_status(int reset, int* status);

// Transpose a [rows, cols] matrix into [cols, ldd] (columns rows .. ldd zeroed).
int transpose(const float* src, int rows, int cols, float* dst, int ldd, cudaStream_t stream);

// Bias gradients from the backward time loop's per-cluster FP64 partials
// part [nparts][4H] (cols [0, 3H): colsums of dG_ih; [3H, 4H): of dG_hh's n
// block; dG_hh's r/z columns are dG_ih's): db_ih = cols [0, 3H), db_hh =
// cols [0, 2H) and [3H, 4H); summed in a fixed order (deterministic).
int bias_grads_finish(const double* part, int nparts, int H, float* db_ih, float* db_hh, cudaStream_t stream);

int sm_count(int device);

// gru_forward's body; overlap = false keeps the whole forward on `stream`
// (no time chunks, no side stream), as the allocation-free entry point needs.
int forward_impl(const float* x, const float* h0, const float* w_ih, const float* w_hh, const float* b_ih,
                 const float* b_hh, float* out, float* hn, float* stash, void* workspace, size_t workspace_bytes,
                 int B, int T, int I, int H, void* stream, bool overlap);

// ---------------------------------------------------------------------------
// Launch accounting and optional per-kernel CUDA-event timing (host side).
// Every kernel launch of this library goes through a LaunchScope so that
// gru_launch_count() is exact and gru_timing_collect() can report per-kind
// device time.
// ---------------------------------------------------------------------------
enum KernelKind {
  kKindInputGemm = 0,   // x . W_ih^T + b_ih
  kKindFwdRecurrent = 1,
  kKindBwdRecurrent = 2,
  kKindGradGemm = 3,    // dW_hh, dW_ih, dx products (+ split-K reduce)
  kKindColsum = 4,      // db_ih / db_hh
  kKindLayout = 5,      // padding / transpose copies feeding the tensor-core products
  kKindLoss = 6,        // MSE loss and its gradient
  kKindCount = 7
};

class LaunchScope {
 public:
  LaunchScope(int kind, cudaStream_t stream, int launches = 1);
  ~LaunchScope();
 private:
  int kind_;
  cudaStream_t stream_;
  void* start_;
};

}  // namespace gru
