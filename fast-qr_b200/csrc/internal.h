// Host-side launchers shared between the fastqr translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fqr {

// Panel width of the blocked path (columns factored per panel kernel).
constexpr int kPanel = 32;

// Small-n path: one warp per matrix, n <= 64.
cudaError_t launch_small(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs,
                         float *H, float *tau, cudaStream_t st);

// Blocked path pieces (n > 64).
cudaError_t launch_copy_in(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs,
                           float *H, cudaStream_t st);
cudaError_t launch_panel(float *H, float *tau, float *Tws, int64_t batch, int n, int k,
                         cudaStream_t st);
cudaError_t launch_trailing(float *H, const float *Tws, int64_t batch, int n, int k,
                            cudaStream_t st);

// Validates and enqueues one batched geqrf (the body of fqr_geqrf_f32);
// returns an FQR_* status.
int geqrf_enqueue(const float *A, int64_t batch, int64_t n, int64_t a_bstride, int64_t a_rstride,
                  int64_t a_cstride, float *H, float *tau, void *workspace, size_t workspace_bytes,
                  cudaStream_t st);

// Panel plan for m remaining rows: threads per CTA and cluster size.
struct PanelShape {
    int warps;
    int rows_per_thread_blocks;  // R: 32-row blocks per warp
    int cluster;                 // CTAs per matrix (1 = no cluster)
};
PanelShape panel_shape(int m);

}  // namespace fqr
