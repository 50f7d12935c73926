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
cudaError_t launch_panel(float *H, float *tau, float *Tws, int64_t batch, int m, int n, int k,
                         cudaStream_t st);
cudaError_t launch_trailing(float *H, const float *Sws, const float *tau, int64_t batch, int m, int n, int k,
                            cudaStream_t st);

// Tensor-core (tcgen05, 3xTF32) trailing update; needs a row count m with
// m % 4 == 0, m >= 128 and a 16-byte aligned H.  Sets *status to nonzero if a bounded wait gave up.
// Its phase-A operands arrive by TMA through two tensor maps of H, encoded
// once per call by prepare_trailing_tc (they depend on H, n and batch only).
bool trailing_tc_supported(int m);
struct TrailingMaps {
    CUtensorMap c;  // 32 rows x 128 trailing columns, 128-byte swizzle
    CUtensorMap v;   // 32 rows x 32 panel columns, 128-byte swizzle
    CUtensorMap cq;  // 128 rows x 32 trailing columns, no swizzle (phase C)
};
cudaError_t prepare_trailing_tc(float *H, int64_t batch, int m, int n, TrailingMaps *maps);
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
cudaError_t launch_trailing_tc(const TrailingMaps &maps, float *H, const float *Sws, const float *tau,
                               int *status, int64_t batch, int m, int n, int k, cudaStream_t st);

// Workspace layout: one 32 x 32 float block per matrix holding the panel's
// S = V^T V (strictly upper; the compact-WY T factor is T = D (I + S D)^-1,
// D = diag(tau)), then a 256-byte status block (int status word first).
constexpr size_t kWsAlign = 256;
constexpr size_t ws_t_bytes(int64_t batch)
{
    return ((size_t)batch * kPanel * kPanel * sizeof(float) + kWsAlign - 1) / kWsAlign * kWsAlign;
}
constexpr size_t ws_total_bytes(int64_t batch) { return ws_t_bytes(batch) + kWsAlign; }

// Validates and enqueues one batched geqrf (the body of fqr_geqrf_f32);
// returns an FQR_* status.
int geqrf_enqueue(const float *A, int64_t batch, int64_t n, int64_t a_bstride, int64_t a_rstride,
                  int64_t a_cstride, float *H, float *tau, void *workspace, size_t workspace_bytes,
                  cudaStream_t st);
// The same with the bounded-wait status word at `status_word` instead of
// inside the workspace (the first kernel of the call clears it).
int geqrf_enqueue_status(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                         int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                         void *workspace, size_t workspace_bytes, int *status_word,
                         cudaStream_t st);

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
