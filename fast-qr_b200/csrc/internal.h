// Host-side launchers shared between the fastqr translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fqr {

// Panel width of the blocked path (columns factored per panel kernel).
constexpr int kPanel = 32;

// Small-n path: one warp per matrix, n <= 64.
cudaError_t launch_small(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs,
                         float *H, float *tau, cudaStream_t st);

// Blocked path pieces (n > 64, or any m x n with m >= n).  H holds m x n
// column-major per matrix (column length m), tau n values per matrix.
// Also clears status[i] for every bit i set in clear_mask (the bounded-wait
// status words).
cudaError_t launch_copy_in(const float *A, int64_t batch, int m, int n, int64_t bs, int64_t rs, int64_t cs,
                           float *H, int *status, unsigned clear_mask, cudaStream_t st);
// Where a panel kernel stores its S = V^T V (strictly upper 32 x 32):
// S(l, c) at base + mat * stride + l * ls + c * cs.
struct SBlock {
    float *base;
    int64_t stride;
    int ls, cs;
};
cudaError_t launch_panel(float *H, float *tau, const SBlock &sb, int64_t batch, int m, int n, int k,
                         cudaStream_t st);
// SIMT fp32 trailing update (any m) of columns c_begin .. n-1 with the
// reflectors of columns k .. k+31 (tau of the others 0); S blocks (32 x 32,
// column-major) at Sws + mat * s_stride.
cudaError_t launch_trailing(float *H, const float *Sws, int64_t s_stride, const float *tau, int64_t batch, int m,
                            int n, int k, int c_begin, cudaStream_t st);

// Tensor-core (tcgen05, 3xTF32) trailing update; needs a row count m with
// m % 4 == 0, m >= 128 and a 16-byte aligned H.  Sets *status to nonzero if a bounded wait gave up.
// Its phase-A operands arrive by TMA through two tensor maps of H, encoded
// once per call by prepare_trailing_tc (they depend on H, n and batch only).
bool trailing_tc_supported(int m);
struct TrailingMaps {
    CUtensorMap c;  // 32 rows x 128 trailing columns, 128-byte swizzle
    CUtensorMap v;   // 32 rows x 32 panel columns, 128-byte swizzle
    CUtensorMap cq;  // 32 rows x 32 trailing columns, no swizzle (phase C)
    CUtensorMap v64;  // 32 rows x 64 panel columns, 128-byte swizzle (rank-64 update)
};
cudaError_t prepare_trailing_tc(float *H, int64_t batch, int m, int n, TrailingMaps *maps);
// 32 x 32 tiles (128-byte swizzle) of a batch of row-major rows x cols float
// matrices: element (i, j) of matrix b at A[b * bs + i * rs + j]; needs a
// 16-byte aligned A and rs, bs multiples of 4.
cudaError_t encode_rowmajor_tiles(const float *A, int64_t batch, int rows, int cols, int64_t bs, int64_t rs,
                                  CUtensorMap *map);
// Maps for applying the reflectors stored in H (n x n per matrix) to a
// target C (m x c_cols per matrix, column-major, batch stride m * c_cols);
// H is m x hcols (column length m).
cudaError_t prepare_apply_maps(const float *H, int m, int hcols, float *C, int64_t c_cols, int64_t batch,
                               TrailingMaps *maps);
// C[k:m, c_begin:c_end] := (I - V T^T V^T) C (apply_t) or (I - V T V^T) C,
// V = the unit-lower reflectors of columns k .. k+31 of H (fewer at the end;
// H is m x hcols, tau hcols values per matrix),
// T = D (I + S D)^-1 from S blocks at Sws + mat * s_stride (floats) and tau.
cudaError_t launch_apply_tc(const TrailingMaps &maps, const float *H, const float *Sws, int64_t s_stride,
                            const float *tau, int *status, int64_t batch, int m, int hcols, int k,
                            int c_begin, int c_end, bool apply_t, cudaStream_t st);
// batch_all: the whole call's batch (the launch covers `batch` of them); the
// static plan splits each tile's rows over a cluster of 2, 4 or 8 CTAs when
// the call's tiles fit one CTA per SM.
cudaError_t launch_trailing_tc(const TrailingMaps &maps, float *H, const float *Sws, int64_t s_stride,
                               const float *tau, int *status, int64_t batch, int64_t batch_all, int m, int n, int k,
                               cudaStream_t st);

// Rank-64 blocking (two 32-column panels per trailing update) for m x n
// matrices with n >= 2048 and m <= 4096 (m % 4 == 0, the tensor-core
// trailing update's condition): per 64 columns a panel, the in-block update
// of the next 32 columns, a second panel, the cross Gram block V1^T V2 and
// one rank-64 trailing update.  A static plan by (m, n).  The rank-64 update
// moves half the HBM bytes of two rank-32 updates (-42% trailing time at
// 16 x 4096^2), but the two in-block launches per block lengthen the
// per-block chain of latency-bound kernels: at n = 512 and 1024 the step
// was 5 to 7% slower, so smaller n keep rank-32 steps.
constexpr int kOuter = 64;
constexpr bool use_outer64(int64_t m, int64_t n) { return n >= 2048 && m >= n && m <= 4096 && m % 4 == 0; }

// Workspace layout: a 256-byte status block (one int status word per part of
// a split batch), then one S block per matrix: 32 x 32 floats (column-major)
// for rank-32 plans, 64 x 64 floats (row-major, S(l, c) at l * 64 + c) for
// rank-64 plans.  S = V^T V (strictly upper); the compact-WY T factor is
// T = D (I + S D)^-1, D = diag(tau).
constexpr size_t kWsAlign = 256;
constexpr int64_t s_block_floats(int64_t m, int64_t n)
{
    return use_outer64(m, n) ? kOuter * kOuter : kPanel * kPanel;
}
constexpr size_t ws_t_bytes(int64_t batch, int64_t m, int64_t n)
{
    return ((size_t)batch * (size_t)s_block_floats(m, n) * sizeof(float) + kWsAlign - 1) / kWsAlign * kWsAlign;
}
constexpr size_t ws_total_bytes(int64_t batch, int64_t m, int64_t n) { return kWsAlign + ws_t_bytes(batch, m, n); }

// In-block steps of a rank-64 block at columns k .. k+63 (S64: the
// matrices' 64 x 64 row-major S blocks, s_stride floats apart; the two
// panels store their S11 and S22 on its diagonal):
// gram == false: C2 := (I - V1 T1^T V1^T) C2 for C2 = H[k:m, k+32:k+64], V1
//   the reflectors of columns k .. k+31, T1 from S11 and tau;
// gram == true: the off-diagonal block S12 = V1^T V2 over rows k+32 .. m-1.
cudaError_t launch_inblock(float *H, const float *tau, float *S64, int64_t s_stride, int64_t batch, int m,
                           int n, int k, bool gram, cudaStream_t st);
// Rank-64 tensor-core trailing update of columns k+64 .. n-1 with the 64
// reflectors of columns k .. k+63 (S64 complete) and tau.  batch_all: the
// whole call's batch (the launch covers `batch` of them), which the static
// plan uses to decide how many CTAs (1, 2, 4 or 8) share each tile's rows.
cudaError_t launch_trailing64_tc(const TrailingMaps &maps, float *H, const float *S64, int64_t s_stride,
                                 const float *tau, int *status, int64_t batch, int64_t batch_all, int m, int n,
                                 int k, cudaStream_t st);

// Mid-size square QR in one launch (qr_mid.cu): one CTA per matrix runs
// the copy-in and every panel and trailing update of its matrix.  Taken for
// 128 <= n <= kMidMaxN with n % 4 == 0 and a 16-byte aligned H (the
// tensor-core update's conditions).  The launch first clears status_words
// status words at `status`; a bounded wait that gave up sets the first.
// flags: kMidFlagForceTimeout makes the first trailing update of every
// matrix wait on a barrier that nothing completes (2 ms limit), so the
// failure path runs without any fault (a test hook).
constexpr int kMidMaxN = 256;
constexpr int kMidFlagForceTimeout = 1;
// The process-wide test-hook flags (fqr_debug_force_timeout): the tensor-core
// kernels make their first wait on a barrier that nothing completes.
int debug_flags();
constexpr int kMidFlagTmaCopy = 2;  // internal: A is read by TMA tiles (row-major, aligned)
bool mid_supported(int64_t m, int64_t n, const void *H);
cudaError_t launch_mid(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs, float *H,
                       float *tau, int *status, int status_words, int flags, cudaStream_t st);

// Validates and enqueues one batched geqrf (the body of fqr_geqrf_f32);
// returns an FQR_* status.
int geqrf_enqueue(const float *A, int64_t batch, int64_t n, int64_t a_bstride, int64_t a_rstride,
                  int64_t a_cstride, float *H, float *tau, void *workspace, size_t workspace_bytes,
                  cudaStream_t st);
// The same with the bounded-wait status word at `status_word` instead of
// inside the workspace (the first kernel of the call clears it), in one part
// on `st`.  batch_in_flight: how many matrices of the caller's work run on
// the device at once (>= batch); the plan sizes its grids for that many, so a
// chunk that runs beside others does not split rows as if it were alone.
int geqrf_enqueue_status(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                         int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                         void *workspace, size_t workspace_bytes, int *status_word,
                         int64_t batch_in_flight, cudaStream_t st);

// Launch with programmatic dependent launch: the kernel may be scheduled
// while the previous kernel on `st` is still running (once every CTA of that
// kernel has executed griddepcontrol.launch_dependents or exited) and must
// execute griddepcontrol.wait (pdl_wait) before it touches memory the
// previous kernels write or read.  Used only for kernels that do.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             const cudaLaunchAttribute *extra, int n_extra, Args... args)
{
    cudaLaunchAttribute attr[4];
    int na = 0;
    for (int i = 0; i < n_extra && na < 3; ++i) attr[na++] = extra[i];
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = (unsigned)na;
    return cudaLaunchKernelEx(&cfg, kern, ((KArgs)args)...);
}

// Panel plan for m remaining rows: threads per CTA and cluster size.
struct PanelShape {
    int warps;
    int rows_per_thread_blocks;  // R: 32-row blocks per warp
    int cluster;                 // CTAs per matrix (1 = no cluster)
};
PanelShape panel_shape(int m);

}  // namespace fqr
