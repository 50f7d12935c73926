// Panel factorisation of the blocked QR: 32 columns, m - k rows, one CTA per
// matrix (a thread-block cluster for panels taller than 1024 rows).
// The reference's panel_factor_kernel (submissions/candidate.py:2404-2505)
// works column by column on global memory with block-wide reductions and
// leaves T to every trailing CTA; the algorithm here is the blocked
// restatement in oracle/geqr2.c (oracle_geqrf_blocked_f64).
#include <cooperative_groups.h>

#include "common.cuh"
#include "internal.h"
#include "panel_body.cuh"

namespace cg = cooperative_groups;

namespace fqr {

// Panel kernel: one panel_body (panel_body.cuh) per matrix.
template <int NW, int R, bool CLUSTER>
__global__ void __launch_bounds__(NW * 32, 1)
panel_kernel(float *__restrict__ H, float *__restrict__ tau, float *__restrict__ Sb, int64_t s_stride, int s_ls,
             int s_cs, int ld, int n, int k)
{
    int ncl = 1;
    if constexpr (CLUSTER) ncl = (int)cg::this_cluster().num_blocks();
    extern __shared__ float4 panel_stage[];
    panel_body<NW, R, CLUSTER, true>(H, tau, Sb, s_stride, s_ls, s_cs, ld, n, k, blockIdx.x / ncl,
                                     reinterpret_cast<float *>(panel_stage));
}

static size_t panel_stage_bytes(int nw) { return (size_t)nw * 32 * kStagePitch * sizeof(float); }

PanelShape panel_shape(int m)
{
    // Fewer, fuller warps: per column every warp pays a fixed cost (shuffles,
    // partial reads, reflector), so 16 rows per thread beat 8.
    if (m <= 128) return {4, 1, 1};
    if (m <= 256) return {4, 2, 1};
    if (m <= 512) return {8, 2, 1};
    if (m <= 1024) return {16, 2, 1};
    // taller panels: a cluster of 8-warp CTAs (512 rows each; the 16-warp
    // shape is register-limited to 128 per thread and spills) up to the
    // portable cluster size of 8
    if (m <= 4096) return {8, 2, (m + 511) / 512};
    return {16, 2, (m + 1023) / 1024};
}

template <int NW, int R>
static cudaError_t launch_panel_t(float *H, float *tau, const SBlock &sb, int64_t batch, int ld, int n, int k,
                                  int cluster, cudaStream_t st)
{
    // the limit covers static + dynamic shared memory beyond 48 KB, so it is
    // raised for every shape rather than from the dynamic size alone
    const size_t dyn = panel_stage_bytes(NW);
    if (cluster <= 1) {
        cudaError_t e = cudaFuncSetAttribute(panel_kernel<NW, R, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
        if (e != cudaSuccess) return e;
        return launch_dependent(panel_kernel<NW, R, false>, dim3((unsigned)batch), dim3(NW * 32), dyn, st,
                                nullptr, 0, H, tau, sb.base, sb.stride, sb.ls, sb.cs, ld, n, k);
    }
    cudaError_t e = cudaFuncSetAttribute(panel_kernel<NW, R, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    return launch_dependent(panel_kernel<NW, R, true>, dim3((unsigned)(batch * cluster)), dim3(NW * 32), dyn,
                            st, attr, 1, H, tau, sb.base, sb.stride, sb.ls, sb.cs, ld, n, k);
}

cudaError_t launch_panel(float *H, float *tau, const SBlock &sb, int64_t batch, int ld, int n, int k,
                         cudaStream_t st)
{
    const PanelShape s = panel_shape(ld - k);
    if (s.cluster > 8) return cudaErrorInvalidValue;
    if (s.warps == 4 && s.rows_per_thread_blocks == 1)
        return launch_panel_t<4, 1>(H, tau, sb, batch, ld, n, k, 1, st);
    if (s.warps == 4) return launch_panel_t<4, 2>(H, tau, sb, batch, ld, n, k, 1, st);
    if (s.warps == 8) return launch_panel_t<8, 2>(H, tau, sb, batch, ld, n, k, s.cluster, st);
    return launch_panel_t<16, 2>(H, tau, sb, batch, ld, n, k, s.cluster, st);
}

}  // namespace fqr
