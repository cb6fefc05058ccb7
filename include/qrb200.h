/*
 * qrb200 -- batched Householder QR for NVIDIA B200 (sm_100a), C ABI.
 *
 * Drop-in boundary for the reference operator ``custom_kernel(data) -> (H, tau)``
 * (Raymondlol/qr-v2-b200-kernel ``submission.py:560-596``; contract of the harness that
 * calls it: ``harness/eval.py:189-211``, output checks ``harness/reference.py:175-204``).
 *
 * Layout (identical to torch.geqrf / LAPACK sgeqrf, row-major storage):
 *   A    : batch matrices, each n x n float32 row-major (row stride n), matrix b at
 *          A + b * a_batch_stride (a_batch_stride >= n*n elements). Read only.
 *   H    : batch x n x n float32 row-major, contiguous. R = triu(H); reflector j is
 *          v_j = (0,..,0, 1, H[j+1:, j]) with the unit diagonal implicit.
 *   tau  : batch x n float32, contiguous. Q = H_0 H_1 ... H_{n-1}, H_j = I - tau_j v_j v_j^T.
 * Sign convention: beta = -sign(alpha) * ||(alpha, x)||, tau = (beta - alpha)/beta,
 * tau = 0 when x == 0 (submission.py:91-107, LAPACK slarfg without rescaling).
 *
 * Execution: every call is asynchronous on ``stream`` (a cudaStream_t; NULL = legacy
 * default stream), makes no host synchronisation and allocates no memory: scratch comes
 * from the caller's ``workspace`` (size from qrb200_workspace_bytes, 256-byte aligned).
 * Two calls that share a workspace must be ordered on the same stream.
 *
 * Every entry point returns a status (QRB200_OK = 0). Device-side failures found by a
 * bounded wait are reported by qrb200_last_status() (no synchronisation) or
 * qrb200_device_status() once the work has executed.
 *
 * The first call on each device registers that device's failure word with a synchronous
 * symbol copy: make it before any stream capture on that device. The library does not
 * survive a cudaDeviceReset (its per-device set-up is not redone).
 */
#ifndef QRB200_H_
#define QRB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  QRB200_OK = 0,
  QRB200_ERR_ARG = 1,        /* bad shape, stride or null pointer                    */
  QRB200_ERR_WORKSPACE = 2,  /* workspace too small or not 256-byte aligned          */
  QRB200_ERR_CUDA = 3,       /* a CUDA runtime call or kernel launch failed          */
  QRB200_ERR_DEVICE = 4,     /* current device is not an sm_100 (B200-class) GPU     */
  QRB200_ERR_TIMEOUT = 5,    /* a device-side bounded wait expired (see device_status) */
  QRB200_ERR_SCRATCH_LIMIT = 6 /* qrb200_geqrf_f32_noalloc: problem needs more scratch than
                                  QRB200_NOALLOC_SCRATCH_BYTES                           */
};

/* Bytes of scratch that qrb200_geqrf_f32 needs for (batch, n).
 * Replaces the per-call temporaries the reference allocates through torch
 * (submission.py:177-185 H clone + tau, :453-480 V/G/M/W/Y). */
size_t qrb200_workspace_bytes(int64_t batch, int64_t n);

/* Batched QR: H, tau <- geqrf(A). Replaces custom_kernel (submission.py:560-596) and
 * its back-ends _fused_qr (:177-185), _factor_custom (:520-553) and torch.geqrf (:576, :583).
 * A is not modified (the reference clones it first, submission.py:179, :522). */
int qrb200_geqrf_f32(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                     int64_t a_batch_stride, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ---- using the factorisation: Q and Q^T (the reference's checker step, sorgqr/sormqr) ---- */

/* Bytes of scratch that qrb200_ormqr_f32 (nrhs columns) and qrb200_orgqr_f32 (nrhs = n) need. */
size_t qrb200_apply_workspace_bytes(int64_t batch, int64_t n, int64_t nrhs);

/* C <- Q^T C (transpose != 0) or Q C (transpose == 0), in place, for each matrix of the batch:
 * Q = H_0 H_1 ... H_{n-1} of (H, tau) in the layout qrb200_geqrf_f32 writes (H batch x n x n,
 * tau batch x n, contiguous), C batch x n x nrhs row-major contiguous. Left side only, as
 * torch.ormqr(H, tau, C, left=True, transpose=...). Blocked compact-WY on the tensor cores
 * (3xTF32). Needs n % 4 == 0, nrhs % 4 == 0, 1 <= n <= 4096, H and C 16-byte aligned
 * (QRB200_ERR_ARG otherwise). Replaces the LAPACK/cuSOLVER sormqr that a consumer of the
 * reference's (H, tau) output would call (README.md:42-50 of the reference: Q is implicit). */
int qrb200_ormqr_f32(const float* H, const float* tau, float* C, int64_t batch, int64_t n, int64_t nrhs,
                     int transpose, void* workspace, size_t workspace_bytes, void* stream);

/* Q (batch x n x n, row-major contiguous, written) = householder_product(H, tau) for square H:
 * replaces torch.linalg.householder_product, which the reference's checker calls on every
 * output (harness/reference.py:206). Same requirements as qrb200_ormqr_f32 (nrhs = n). */
int qrb200_orgqr_f32(const float* H, const float* tau, float* Q, int64_t batch, int64_t n, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Human-readable text for a status code (static storage). */
const char* qrb200_status_string(int status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int qrb200_version(void);

/* Device-side failures. Every wait inside a kernel is bounded; a kernel whose wait expires
 * records the failure, skips its outputs and returns (the results of that call are invalid).
 * The record lands in a device word and in a mapped pinned host word per device.
 *
 * qrb200_last_status: QRB200_ERR_TIMEOUT if a kernel on the current device has recorded a
 * failure since the last read, else QRB200_OK; the host word is cleared by the read. It makes
 * no CUDA call beyond cudaGetDevice and never waits, so it sees failures of work that has
 * already executed (read it after synchronising, or before the next call as the Python operator
 * does). *site_out (may be NULL) receives the wait site: 1 tensor-core mbarrier, 2 whole-matrix
 * hand-off, 3 cluster-panel exchange, 4 self-test. No counterpart in the reference (its only
 * failure mechanism is the exception fallback of submission.py:572-596). */
int qrb200_last_status(int* site_out);

/* Synchronous variant: reads (and clears) the device word of the current device with a symbol
 * copy (which waits for prior work on the legacy default stream) and clears the host word;
 * *status_out = QRB200_ERR_TIMEOUT or QRB200_OK. */
int qrb200_device_status(int* status_out);

/* Test hook: one warp waits `polls` times on a barrier that nothing completes, so the wait runs
 * out and reports site 4 through the same path as the factorisation kernels. Asynchronous on
 * `stream`; leaves the device usable. */
int qrb200_selftest_wait_timeout(uint32_t polls, void* stream);

/* ---- allocation-free entry (no counterpart in the reference) ------------------------- */

/* Size of the library's static device scratch used by qrb200_geqrf_f32_noalloc: 32 MiB.
 * It covers every call with qrb200_workspace_bytes(batch, n) <= this: up to 1 matrix of n = 4096,
 * 3 of n = 2048, 11 of n = 1024, 29 of n = 512 or 55 of n = 256 per call; n <= 128 needs no
 * scratch at any batch size. */
#define QRB200_NOALLOC_SCRATCH_BYTES (32u << 20)

/* Same result as qrb200_geqrf_f32 (bit for bit), but the scratch is a file-scope static
 * __device__ array of the library instead of a caller workspace, so neither the caller nor the
 * library allocates device memory. For callers that cannot or should not allocate: plain C or
 * FFI code with no device allocator at hand, loops that must not call cudaMalloc/cudaFree
 * (cudaFree waits for the whole device), and processes whose device memory is already fully
 * reserved by another allocator.
 *   - Limit: returns QRB200_ERR_SCRATCH_LIMIT, launching nothing, when
 *     qrb200_workspace_bytes(batch, n) > QRB200_NOALLOC_SCRATCH_BYTES; use qrb200_geqrf_f32
 *     with a workspace for larger problems. Other errors are those of qrb200_geqrf_f32.
 *   - Set-up: the first call on each device (the current device) looks up the array's device
 *     address with cudaGetSymbolAddress, which loads the library module that holds it there;
 *     make that first call before any stream capture on that device.
 *   - Nothing needs to start at zero: every scratch word is written before it is read within
 *     a call, so the array's contents between calls do not matter.
 *   - One array per device: calls on the same device whose executions overlap (different
 *     streams, or host threads, without ordering) race on it and give wrong results. Order
 *     them on one stream, or with events. */
int qrb200_geqrf_f32_noalloc(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                             int64_t a_batch_stride, void* stream);

/* ---- diagnostics (no counterpart in the reference; used by bench.py) ---------------- */

/* The three 3xTF32 tcgen05 GEMMs of the 128-wide trailing update on their own, for accuracy
 * tests: for each matrix of H (batch x n x n, contiguous, 129 <= n <= 1024, n % 4 == 0),
 * V = the unit lower trapezoid of H[:, 0:128] (entries above the diagonal of that block read as
 * zero, the diagonal as one), C = H[:, 128:n]; computes C <- C - V (Tt (V^T C)) with the
 * 128 x 128 matrix Tt given (batch x 128 x 128, row-major; the two-level schedule passes the
 * block factor T transposed), through W^T = C^T V (tc_vtc128), W'^T = W^T Tt^T (tc_tw128) and
 * C -= V W' (tc_upd128). The first 128 columns of H are left as they are. Workspace as for
 * qrb200_geqrf_f32(batch, n). */
int qrb200_diag_wide_update_f32(float* H, const float* Tt, int64_t batch, int64_t n, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Number of kernels this library has launched in the process so far (all threads). */
long long qrb200_launch_count(void);

/* Per-kernel-kind totals of one profiled call. */
typedef struct qrb200_kernel_stat {
  char name[32];        /* kernel kind, e.g. "panel_factor", "wy_upd"                 */
  int32_t launches;     /* launches of this kind in the call                          */
  int32_t tensor_bound; /* 1: compute (FLOP) bound contraction, 0: memory/latency     */
  double ms;            /* summed CUDA-event duration of those launches               */
  double flops;         /* algorithmic FLOPs of those launches                         */
  double bytes;         /* algorithmic HBM bytes of those launches                     */
} qrb200_kernel_stat;

/* Same computation as qrb200_geqrf_f32, with a CUDA event pair around every launch; waits
 * for the stream, then fills up to max_stats entries (one per kernel kind that ran). */
int qrb200_profile_geqrf_f32(const float* A, float* H, float* tau, int64_t batch, int64_t n,
                             int64_t a_batch_stride, void* workspace, size_t workspace_bytes,
                             void* stream, qrb200_kernel_stat* stats, int max_stats, int* n_stats);

#ifdef __cplusplus
}
#endif

#endif /* QRB200_H_ */
