/*
 * rnn_kernel_b200 — C ABI of the B200 (sm_100a) FP32 GRU training path.
 *
 * Plain pointers and sizes only; every pointer is a device pointer unless
 * stated otherwise, every tensor is dense row-major float32, and every call is
 * stream-ordered on `stream` (a cudaStream_t, NULL = legacy default stream).
 * No call synchronises the stream, allocates device memory or throws; each
 * returns a status code (GRU_OK == 0) and on failure records a message that
 * gru_last_error() returns (per calling thread).
 *
 * Shapes: B batch, T seq_len, I input_size, H hidden_size (1 <= H <= 256).
 * Gate order is r, z, n and the weight layout is torch.nn.GRU's:
 * w_ih [3H, I], w_hh [3H, H], b_ih [3H], b_hh [3H]; x is batch_first [B, T, I].
 *
 * Reference interface replaced (paths inside HanXuxx/RNN_kernel):
 *   src/rnn_kernel/a100/prod/gru.py  — the Python ctypes / cuda-python
 *   launchers `_launch_forward` (:226-301), `_launch_forward_no_cache`
 *   (:304-376), `_launch_pack_hidden_prev` (:379-412),
 *   `_launch_backward_sequence` (:415-487) plus the torch GEMMs around them in
 *   `_A100GRUFunction.forward/backward` (:519-523, :569-578).
 */
#ifndef RNN_KERNEL_B200_H
#define RNN_KERNEL_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GRU_OK 0
#define GRU_ERR_INVALID 1     /* bad shape / null pointer / workspace too small */
#define GRU_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define GRU_ERR_UNSUPPORTED 3 /* device or shape outside the supported range */

/* Bits of the device status word (gru_device_status). */
#define GRU_STATUS_WAIT_TIMEOUT 1 /* a kernel's bounded inter-CTA wait expired */

/* Message for the last failing call on this thread ("" if none). Replaces the
 * RuntimeError text of `_check_cuda_error` (prod/gru.py:57-63). */
const char* gru_last_error(void);

/* 1 if `device` is a compute-capability 10.x (B200 class) GPU this library
 * was built for, else 0.  Replaces `is_a100_available` (prod/gru.py:109-117). */
int gru_device_supported(int device);

/* Bytes of the forward stash for one layer: per (b, t) the gates r, z, n, the
 * recurrent n pre-activation W_hn.h + b_hn and the step's input hidden state
 * h_prev, i.e. B*T*5H floats.  Replaces the gate cache of `_launch_forward`
 * (prod/gru.py:236-238) plus the packed h_prev (:379-412). */
size_t gru_stash_bytes(int B, int T, int H);

/* Device workspace `gru_forward` needs (input-gate buffer [B,T,3H]). */
size_t gru_forward_workspace_bytes(int B, int T, int I, int H);

/* One GRU layer forward.
 *   out [B,T,H], hn [B,H] are written.
 *   stash: gru_stash_bytes() bytes for a training forward, or NULL for the
 *   inference (no-stash) path.
 * Replaces `_A100GRUFunction.forward` (prod/gru.py:490-529) and
 * `_a100_gru_forward_inference` (:583-617). */
int gru_forward(const float* x, const float* h0, const float* w_ih, const float* w_hh,
                const float* b_ih, const float* b_hh, float* out, float* hn, float* stash,
                void* workspace, size_t workspace_bytes, int B, int T, int I, int H,
                void* stream);

/* Device workspace `gru_backward` needs. */
size_t gru_backward_workspace_bytes(int B, int T, int I, int H);

/* One GRU layer backward from the stash of a training `gru_forward`.
 *   dout [B,T,H] or NULL (treated as zeros), dhn [B,H] or NULL (zeros).
 *   Writes dh0 [B,H], dw_ih [3H,I], dw_hh [3H,H], db_ih [3H], db_hh [3H]
 *   (overwritten, not accumulated) and dx [B,T,I] unless dx is NULL.
 * Replaces `_A100GRUFunction.backward` (prod/gru.py:532-580). */
int gru_backward(const float* dout, const float* dhn, const float* x, const float* w_ih,
                 const float* w_hh, const float* stash, float* dx, float* dh0, float* dw_ih,
                 float* dw_hh, float* db_ih, float* db_hh, void* workspace,
                 size_t workspace_bytes, int B, int T, int I, int H, void* stream);

/* Size of the static device scratch behind gru_forward_inference_noalloc. */
#define GRU_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Inference forward (no stash) that allocates nothing and takes no workspace.
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory -- e.g. a plugin inside a host whose device memory is owned by the
 * host's own allocator, or code running where an allocation would stall or
 * is forbidden.  Same arguments and results as gru_forward(..., stash = NULL,
 * ...) minus the workspace: the scratch is a fixed
 * GRU_NOALLOC_SCRATCH_BYTES device array inside the library, held by every GPU
 * that loads it until the process exits.  Shapes whose forward workspace
 * (gru_forward_workspace_bytes) exceeds that size are rejected with
 * GRU_ERR_UNSUPPORTED and a message.  The first call on a device looks up the
 * array's device address (once per device, with that device current); make
 * that first call before any stream capture.  All calls on a device share the
 * one array, so calls that overlap on the GPU (different streams, no ordering
 * between them) race; serialise them.  The looked-up address is cached per
 * device ordinal for the process's life: resetting the device or recreating
 * its primary context while the library is loaded is not supported. */
int gru_forward_inference_noalloc(const float* x, const float* h0, const float* w_ih,
                                  const float* w_hh, const float* b_ih, const float* b_hh,
                                  float* out, float* hn, int B, int T, int I, int H, void* stream);

/* ---- MSE loss of the output (the training harness's F.mse_loss(pred, y):
 * rnn_benchmark.py:636, :657, :680; tests/test_sequence_chunking.py:27-28),
 * fused into one pass each way instead of torch's three. ---- */

/* Workspace of gru_mse_loss for n elements (FP64 block partials). */
size_t gru_mse_workspace_bytes(long n);

/* *loss = mean((out - target)^2) over n floats (device pointers; the sum in
 * FP64, deterministic). */
int gru_mse_loss(const float* out, const float* target, long n, float* loss, void* workspace,
                 size_t workspace_bytes, void* stream);

/* dout = (2 / n) * (out - target) * (*grad_loss), grad_loss a device scalar
 * (the loss's upstream gradient), in torch's order of operations. */
int gru_mse_loss_backward(const float* out, const float* target, const float* grad_loss, float* dout, long n,
                          void* stream);

/* Time chunks (no reference counterpart; a scheduling knob of this library).
 * When the time loops leave SMs idle (e.g. 104 of 148 at H = 256, B = 64),
 * gru_forward and gru_backward run the sequence as n consecutive chunks and
 * put the tensor-core products of one chunk on the idle SMs (an internal
 * side stream, joined before the call returns) beside the loop over another.
 * n = 0: automatic (2 chunks when T is a multiple of 256 and a cost
 * estimate says the overlap pays for the extra loop launch); 1: off; 2..4:
 * that many chunks whenever T is a multiple of 128 * n, the loop is one wave
 * and leaves an SM idle.  Results are the same up to the order of
 * the weight-gradient partial sums.  Process-wide; returns the previous
 * setting, or -1 for an invalid n. */
int gru_set_time_chunks(int n);

/* Time-loop kernels for small hidden sizes (no reference counterpart; a
 * kernel-selection knob of this library).  mode 0 (default): the forward
 * time loop for H <= 96 and the backward one for H <= 64 run one CTA per
 * group of up to 4 batch rows, which holds all of W_hh and runs a step with
 * one barrier; mode 1: the thread-block-cluster kernels used for larger H,
 * everywhere.  Both compute the same function (results agree to FP32
 * rounding).  Process-wide; returns the previous mode, or -1 for an invalid
 * mode. */
int gru_set_small_loops(int mode);

/* ---- Telemetry (no reference counterpart: the reference had no kernel
 * timers; its profiling scripts used torch.profiler / nsys, see
 * scripts/profile_a100_h256_step.py).  Kernel kinds: 0 input-projection GEMM,
 * 1 forward time loop, 2 backward time loop, 3 gradient products (dW, dx;
 * + split-K reduce), 4 bias-gradient column sums, 5 padding / transpose
 * copies, 6 MSE loss and its gradient. ---- */

/* Device status word of the current device: 0 when every kernel so far ran
 * to completion, else GRU_STATUS_* bits (a bounded wait inside a time-loop
 * kernel expired; results of that launch are invalid).  Synchronises the
 * device.  reset != 0 clears the word.  Returns -1 (and sets the error text)
 * if it cannot be read.  No reference counterpart: the reference's waits
 * were grid.sync() calls with no bound. */
int gru_device_status(int reset);

/* Failure-path self-test (no reference counterpart): launches one CTA that
 * waits, through the same bounded-wait routine the time loops use, on an
 * mbarrier phase that nothing completes, with a limit of limit_ms (1..10000).
 * It must return with *result (a device int) = 0 and GRU_STATUS_WAIT_TIMEOUT
 * set in the status word, leaving the context usable; no fault, no trap. */
int gru_selftest_wait_timeout(int limit_ms, int* result, void* stream);

/* Number of kernels this library has launched in this process. */
unsigned long long gru_launch_count(void);

/* Turn per-launch CUDA-event timing on (1) or off (0). */
int gru_timing_enable(int on);

/* Wait for the recorded events and return, per kernel kind, the summed device
 * time in ms and the number of timed launches; clears the record. */
int gru_timing_collect(double* total_ms, int* count, int n_kinds);

#ifdef __cplusplus
}
#endif

#endif /* RNN_KERNEL_B200_H */
