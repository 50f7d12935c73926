/*
 * fastqr -- batched square Householder QR (geqrf) for NVIDIA B200 (sm_100a).
 *
 * C ABI of libfastqr.so.  Plain pointers and sizes only; every pointer below
 * is a CUDA device pointer unless stated otherwise, and `stream` is a
 * cudaStream_t passed as void*.  All calls are asynchronous on `stream`: they
 * validate arguments on the host, enqueue kernels and return.  The library
 * allocates no device memory on this path; scratch space is caller-owned
 * (see fqr_workspace_bytes).  Calls are thread-safe: the only global state is
 * per device -- up to three internal streams and their events, created on
 * first use, on which the blocked path runs parts of a batch of two or more
 * matrices (two parts, four for n >= 2048; always ordered with the caller's
 * stream: they wait for the caller's prior work and the caller's stream waits
 * for them).  Because every such call on a device forks onto the same side
 * streams, two callers on independent streams are serialised through them:
 * each caller's stream picks up an ordering dependency on the other's
 * blocked-path work.  Results stay correct; concurrency between such calls
 * is lost.  The single-launch paths (n <= 64, and the one-launch mid-size
 * kernel where the plan takes it) use only the caller's stream.
 *
 * Output layout (the contract of torch.geqrf, and of the reference's
 * `custom_kernel(data) -> (H, tau)`):
 *   H   : float32, column-major per matrix, element (i, j) of matrix b at
 *         H[b*n*n + j*n + i]  (strides (n*n, 1, n) in elements).  R is on and
 *         above the diagonal, the Householder vectors v_j (implicit unit
 *         diagonal) below it.
 *   tau : float32 [batch][n] contiguous.  tau[b][n-1] is always 0.
 * Reflector convention (LAPACK xLARFG): H_j = I - tau_j v_j v_j^T with
 * beta_j = -sign(alpha_j) * ||[alpha_j; x_j]||; tau_j = 0 when x_j == 0.
 */
#ifndef FASTQR_H
#define FASTQR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference reports failures by raising from its pybind
 * entry points (TORCH_CHECK / C10_CUDA_KERNEL_LAUNCH_CHECK,
 * submissions/candidate.py:111-125, :1333-1353); this ABI returns codes. */
enum {
    FQR_OK = 0,
    FQR_EINVAL = 1,        /* null pointer, negative size, bad stride */
    FQR_EUNSUPPORTED = 2,  /* n outside the dispatch table */
    FQR_ELAUNCH = 3,       /* a kernel launch failed */
    FQR_ETIMEOUT = 4,      /* a bounded device-side wait gave up */
    FQR_EWORKSPACE = 5,    /* workspace missing or too small */
    FQR_ECUDA = 6,         /* other CUDA runtime error (no device, ...) */
    FQR_ENOALLOC_LIMIT = 7 /* batch too large for fqr_geqrf_f32_noalloc's scratch */
};

/* Largest supported n. */
#define FQR_MAX_N 8192

/*
 * Batched QR of `batch` float32 n x n matrices.
 *
 * Replaces the reference's submission entry point
 *   custom_kernel(data) -> (H, tau)       submissions/candidate.py:8383-8415
 *                                         (contract: official/submission.py:5-6,
 *                                          official/task.py:4-5)
 * and the extension entries it dispatches to
 *   geqrf32(data, h, tau)                 submissions/candidate.py:111-125
 *   geqrf512_blocked(data, h, tau, ...)   submissions/candidate.py:1333-1353
 * with caller-allocated H / tau as there.
 *
 * A: element (i, j) of matrix b at A[b*a_bstride + i*a_rstride + j*a_cstride]
 *    (strides in elements; the reference passes row-major contiguous input,
 *    a_bstride = n*n, a_rstride = n, a_cstride = 1).  A is read only.
 * H, tau: outputs as described above; must not overlap A.
 * workspace: device scratch of at least fqr_workspace_bytes(batch, n) bytes,
 *    256-byte aligned (may be NULL when that size is 0).
 * Returns FQR_OK once the work is enqueued.
 */
int fqr_geqrf_f32(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                  int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                  void *workspace, size_t workspace_bytes, void *stream);

/* Scratch bytes fqr_geqrf_f32 needs for (batch, n); 0 for the small-n path.
 * Replaces the reference's cached workspace sizing
 * (submissions/candidate.py:3682-3851), which allocated inside the call. */
size_t fqr_workspace_bytes(int64_t batch, int64_t n);

/* Static string for a status code. */
const char *fqr_status_string(int status);

/* Writes a one-line description of the kernel plan chosen for (batch, n)
 * into buf (NUL-terminated, truncated to len).  Returns FQR_OK or
 * FQR_EUNSUPPORTED.  The plan depends only on (batch, n) and the device's SM
 * count -- never on matrix values (the reference's data-dependent routing,
 * submissions/candidate.py:7779-8381, is deliberately absent). */
int fqr_plan_describe(int64_t batch, int64_t n, char *buf, size_t len);

/* Number of kernel launches fqr_geqrf_f32 enqueues for (batch, n), counting
 * every part of a batch of two or more on the blocked path (n > 64). */
int fqr_launch_count(int64_t batch, int64_t n);

/* Largest batch fqr_geqrf_f32_noalloc accepts when n > 64 (its static
 * scratch holds this many 64 x 64 float S blocks: 16 MiB per device). */
#define FQR_NOALLOC_MAX_BATCH 1024

/*
 * Same computation and output as fqr_geqrf_f32, for callers that cannot
 * allocate device memory: no workspace argument, and the library allocates
 * nothing.  Scratch comes from a fixed 16 MiB __device__ array inside the
 * library, present on every GPU that loads it until the process exits.
 * Its address is looked up on the first call made in each CUDA context (that
 * device current) and again whenever the current context changes (e.g. after
 * cudaDeviceReset).  The first call with batch >= 2 on the split blocked path
 * of a device also creates that device's side streams and events (see the top
 * of this file).  Make the first call on each device before any stream
 * capture.
 * n > 64 allows at most FQR_NOALLOC_MAX_BATCH matrices per call, else
 * FQR_ENOALLOC_LIMIT is returned and nothing is enqueued; n <= 64 needs no
 * scratch and has no batch limit.  Every call on a device shares the array:
 * calls that may run concurrently on the GPU (unordered streams) race and give
 * wrong results, so issue them on one stream or order them.
 * A bounded device-side wait that gave up is recorded in the array's status
 * block; fqr_noalloc_check_status reports it.
 * No counterpart in the reference: its entry points always allocate their
 * outputs and workspace through PyTorch.
 */
int fqr_geqrf_f32_noalloc(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                          int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                          void *stream);

/* fqr_check_status for fqr_geqrf_f32_noalloc, which has no caller workspace:
 * synchronizes `stream`, then returns FQR_ETIMEOUT if the last no-alloc call
 * with n > 64 on the current device hit a bounded device-side wait that gave
 * up, else FQR_OK (also when no such call has been made on this device; calls
 * with n <= 64 use no scratch and leave the status block as it was).  Call it
 * on the stream of that call, before the next no-alloc call clears the
 * status block.  No counterpart in the reference. */
int fqr_noalloc_check_status(void *stream);

/*
 * Batched QR of matrices in HOST memory: the same result as fqr_geqrf_f32,
 * with A, H and tau host pointers (page-locked memory, from cudaHostAlloc or
 * cudaHostRegister, lets the copies overlap; pageable memory works, slower).
 * The batch is cut into chunks that are uploaded, factored and downloaded on
 * internal streams with separate device staging, so that copies in both
 * directions overlap the kernels.  Asynchronous on `stream` like
 * fqr_geqrf_f32: H and tau are complete, and A may be reused, once `stream`
 * has passed the call.
 * A: each matrix one dense n x n block, row-major (a_rstride = n,
 *    a_cstride = 1) or column-major (1, n); a_bstride >= n*n elements.
 * H, tau: host, layouts as for fqr_geqrf_f32.
 * workspace: DEVICE scratch of fqr_host_workspace_bytes(batch, n) bytes,
 *    256-byte aligned (staging for the chunks in flight).
 * Creates a few streams and events per device on its first call there.
 * The reference's entry point takes device tensors only
 * (submissions/candidate.py:8383-8415, official/eval.py:125-132); this is the
 * form a host-resident caller (a CPU library's ctypes/JNI binding) uses
 * instead of copying the batch itself around the device call.
 */
size_t fqr_host_workspace_bytes(int64_t batch, int64_t n);
int fqr_geqrf_f32_host(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                       int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                       void *workspace, size_t workspace_bytes, void *stream);
/* fqr_check_status for fqr_geqrf_f32_host: synchronizes `stream`, then
 * returns FQR_ETIMEOUT if any chunk's bounded device-side wait gave up. */
int fqr_host_check_status(const void *workspace, size_t workspace_bytes, int64_t batch, int64_t n,
                          void *stream);

/*
 * Q of a factorisation in compact form, Q = H_0 H_1 ... H_{n-1} with
 * H_j = I - tau_j v_j v_j^T (v_j read from below the diagonal of column j of
 * H, unit diagonal implied).  H and tau as fqr_geqrf_f32 returns them (device
 * pointers; H column-major per matrix, tau [batch][n]); Q: batch x n x n,
 * column-major like H.  workspace: fqr_orgqr_workspace_bytes(batch, n) bytes
 * (0 for n <= 512 with n % 4 != 0 or n < 128: those sizes take a
 * reflector-by-reflector kernel).  Larger n run panel by panel: on the tensor
 * cores when n % 4 == 0 and H and Q (C) are 16-byte aligned, else with an
 * FP32 SIMT update.
 * Replaces the reference's use of torch.linalg.householder_product in its
 * checker (official/reference.py:199).
 */
size_t fqr_orgqr_workspace_bytes(int64_t batch, int64_t n);
int fqr_orgqr_f32(const float *H, const float *tau, int64_t batch, int64_t n, float *Q,
                  void *workspace, size_t workspace_bytes, void *stream);

/*
 * C := Q^T C (transpose != 0) or C := Q C, in place, for the Q of (H, tau)
 * as in fqr_orgqr_f32.  C: batch x n x ncols, column-major per matrix
 * (element (i, j) of matrix b at C[b*n*ncols + j*n + i]), device pointer.
 * workspace: fqr_orgqr_workspace_bytes(batch, n) bytes.  Replaces the
 * reference's torch.ormqr calls (submissions/candidate.py:7224-7242), left
 * side.
 */
int fqr_ormqr_f32(const float *H, const float *tau, int64_t batch, int64_t n, float *C, int64_t ncols,
                  int transpose, void *workspace, size_t workspace_bytes, void *stream);

/*
 * C := C Q (transpose == 0) or C := C Q^T, in place, right side: torch.ormqr
 * with left=False, which the reference's tail projection uses
 * (submissions/candidate.py:7231).  C: batch x mrows x n, ROW-major per
 * matrix (element (r, j) of matrix b at C[b*mrows*n + r*n + j], torch's
 * default layout), device pointer; H, tau and workspace as for
 * fqr_ormqr_f32.  (C read column-major is C^T, and C Q = (Q^T C^T)^T.)
 */
int fqr_ormqr_right_f32(const float *H, const float *tau, int64_t batch, int64_t n, float *C, int64_t mrows,
                        int transpose, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Rectangular batched QR: torch.geqrf on [batch, m, n].  Replaces the
 * reference's tall-block geqrf, torch.geqrf(data[:, :, :cols]) in
 * _embedded_rectangular_geqrf (submissions/candidate.py:7204-7214).
 *   A:   any strides, element (b, i, j) at A[b*a_bstride + i*a_rstride + j*a_cstride]
 *   H:   m x n column-major per matrix, H[b*m*n + j*m + i] (strides (m*n, 1, m))
 *   tau: [batch][n]; a wide block (m < n) has min(m, n) = m reflectors,
 *        tau[b][0 .. m-1], and tau[b][m .. n-1] is set to 0 (torch.geqrf
 *        returns the first m)
 * m == n is exactly fqr_geqrf_f32.  A wide block is factored like LAPACK
 * xGEQRF: m reflectors from the first m columns, every trailing update also
 * applied to columns m .. n-1 (which end as R's right part).  Both m and n
 * are at most FQR_MAX_N.  The workspace is
 * fqr_geqrf_rect_workspace_bytes(batch, m, n) bytes, 256-byte aligned; the
 * status word for fqr_check_status sits in it as for fqr_geqrf_f32.
 */
size_t fqr_geqrf_rect_workspace_bytes(int64_t batch, int64_t m, int64_t n);
int fqr_geqrf_rect_f32(const float *A, int64_t batch, int64_t m, int64_t n, int64_t a_bstride,
                       int64_t a_rstride, int64_t a_cstride, float *H, float *tau, void *workspace,
                       size_t workspace_bytes, void *stream);

/*
 * Synchronizes `stream`, then reports whether the last fqr_geqrf_f32 that
 * used `workspace` (for `batch` matrices) hit a bounded device-side wait that
 * gave up: FQR_OK or FQR_ETIMEOUT.  The tensor-core kernels never spin
 * without a limit; on giving up they record it here and return.  No
 * counterpart in the reference, whose kernels have no device-side waits.
 */
int fqr_check_status(const void *workspace, size_t workspace_bytes, int64_t batch, void *stream);

/*
 * Test hook for the failure path.  enable != 0: in every later call, each CTA
 * of the rank-32 tensor-core trailing update (and of the one-launch mid-size
 * kernel) makes its first wait on a barrier that nothing completes, with a
 * 2 ms limit, so that the bounded-wait failure path runs (copies and MMAs in
 * flight drain, FQR_ETIMEOUT is recorded for fqr_check_status) without any
 * GPU fault.  enable == 0 restores normal
 * operation.  Process-wide; returns the previous setting.  No counterpart in
 * the reference, whose kernels have no device-side waits.
 */
int fqr_debug_force_timeout(int enable);

/*
 * Diagnostic plan override, process-wide; returns the previous mode.
 * mode 0: the static plan (default).  mode 1: square 128 <= n <= 256 with
 * n % 4 == 0 run the one-launch mid-size kernel (one CTA per matrix runs its
 * whole factorisation) instead of the blocked multi-launch path; that kernel
 * measured slower than the blocked path at every batch size tried, so the
 * static plan does not take it.  No counterpart in the reference.
 */
int fqr_debug_plan(int mode);

/* Kernel classes timed by fqr_geqrf_f32_profile. */
enum {
    FQR_STAGE_SMALL = 0,     /* warp-per-matrix kernel (n <= 64) */
    FQR_STAGE_COPY_IN = 1,   /* row-major A -> column-major H */
    FQR_STAGE_PANEL = 2,     /* panel factorisation + S = V^T V and tau */
    FQR_STAGE_TRAILING = 3,  /* trailing update C -= V T^T V^T C */
    FQR_STAGE_INBLOCK = 4,   /* rank-64 blocks: next-panel update and cross Gram block */
    FQR_STAGE_MID = 5,       /* one-launch mid-size kernel (whole factorisation) */
    FQR_NUM_STAGES = 6
};

/*
 * Diagnostic twin of fqr_geqrf_f32: identical launches, with a CUDA event
 * pair recorded on `stream` around every kernel; synchronizes `stream` before
 * returning and writes the summed device time per stage (milliseconds) into
 * stage_ms[FQR_NUM_STAGES].  Not for production use (it blocks the host).
 * No counterpart in the reference, which never times its kernels
 * individually.
 */
int fqr_geqrf_f32_profile(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                          int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                          void *workspace, size_t workspace_bytes, void *stream,
                          float *stage_ms);

/* Library version, e.g. 100 for 0.1.0. */
int fqr_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FASTQR_H */
