// Panel factorisation of the blocked QR: 32 columns, m - k rows, one CTA per
// matrix (a thread-block cluster for panels taller than 1024 rows).
// The reference's panel_factor_kernel (submissions/candidate.py:2404-2505)
// works column by column on global memory with block-wide reductions and
// leaves T to every trailing CTA; the algorithm here is the blocked
// restatement in oracle/geqr2.c (oracle_geqrf_blocked_f64).
#include <cooperative_groups.h>

#include "common.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace fqr {

namespace {
constexpr int kStagePitch = 36;  // floats per row of a warp's 32 x 32 staging block
}  // namespace

// ---------------------------------------------------------------------------
// Panel kernel.
//
// Thread layout: a warp covers blocks of 32 panel rows x 32 columns; lane =
// cg + 8*rg owns columns 4cg..4cg+3 of rows 8rg..8rg+7 of each block, in
// registers (4 columns per lane keep the unrolled per-column body small
// enough for the instruction cache).  Per column c:
//   * the x-values of the lane's rows are fetched from the lane of the same
//     row group that owns column c (one shuffle per row);
//   * the 4 unscaled partial dots d_j = x^T a_j are reduced over the warp's 4
//     row groups (3 shuffles; a reduce-scatter leaves column 4cg+rg in lane
//     (cg, rg)); column c's own slot is sum x*x = sigma.  The per-warp
//     results go to a shared buffer double-buffered by column parity;
//   * ONE CTA barrier; then every warp sums the per-warp partials itself (in
//     the same order, so all warps hold bitwise-identical values), forms the
//     reflector and tau * w_j with w_j = a(c, j) + scale * d_j -- no serial
//     single-warp section and no second barrier.  Panels taller than one CTA
//     are split over a thread-block cluster: warp 0 of each CTA also sends its
//     CTA's partials to every CTA of the cluster through distributed shared
//     memory and one cluster barrier replaces the CTA barrier's role;
//   * every thread applies the rank-1 update to its tile.
// Only the warp holding panel rows 0..31 needs row masks (rows <= c are R
// rows), but every warp runs the same masked code (the masks are all-true
// elsewhere): one copy of the unrolled column body instead of two keeps it in
// the instruction cache (measured: panel time -14% at m = 256).
// The compact-WY factor is stored as S(l, c) = v_l^T v_c (= w_l for l < c,
// a by-product of column c's reduction) plus tau; the trailing update uses
// them through Y = T^T W = (I + D S^T)^-1 D W, D = diag(tau).
// ---------------------------------------------------------------------------
template <int NW, int R, bool CLUSTER>
__global__ void __launch_bounds__(NW * 32, 1)
panel_kernel(float *__restrict__ H, float *__restrict__ tau, float *__restrict__ Sb, int64_t s_stride, int s_ls,
             int s_cs, int ld, int n, int k)
{
    constexpr int ROWS = NW * 32 * R;  // panel rows held by one CTA
    constexpr int NR = 8 * R;          // rows per thread
    constexpr int PS = 33;             // partial slots: 32 dots (slot c = sigma)
    constexpr int XS = 64;             // cluster slots: 32 dots + 32 row-c values
    __shared__ float part[2][NW][PS];
    __shared__ float rowc_s[2][32];
    __shared__ float red2[NW][32];
    __shared__ double sigd_part[NW];
    __shared__ float Ysm[32][33];
    __shared__ float tau_s[32];
    __shared__ float xch[CLUSTER ? 2 : 1][CLUSTER ? 8 : 1][XS];
    __shared__ float xrb[CLUSTER ? 8 : 1][32];
    __shared__ double xchd[CLUSTER ? 8 : 1];

    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int cgp = lane & 7, rg = lane >> 3;
    int crank = 0, ncl = 1;
    if constexpr (CLUSTER) {
        cg::cluster_group cl = cg::this_cluster();
        crank = (int)cl.block_rank();
        ncl = (int)cl.num_blocks();
    }
    const int64_t mat = blockIdx.x / ncl;
    const int m = ld - k;  // panel rows (ld = the matrix's row count, >= n)
    // reflectors of this panel: the columns left, at most 32 (and never more
    // than the rows)
    const int w = min(kPanel, min(m, n - k));
    float *Hm = H + mat * (int64_t)ld * n;
    const bool top = crank == 0 && wid == 0;  // holds panel rows 0..31
    // per-warp staging of one 32 x 32 block, row-major with a 36-float pitch:
    // 16-byte accesses by 8 consecutive lanes (one column group each, or one
    // row each) hit 8 distinct 16-byte bank groups
    extern __shared__ float4 panel_stage[];
    float *stg = reinterpret_cast<float *>(panel_stage) + wid * (32 * kStagePitch);

    pdl_wait();  // the previous trailing update (or copy-in) has completed

    int row[NR];
    float p[NR][4];
#pragma unroll
    for (int q = 0; q < NR; ++q) row[q] = crank * ROWS + (q >> 3) * (NW * 32) + wid * 32 + 8 * rg + (q & 7);
    // load: lane = row, one coalesced 128-byte column segment per load, then
    // each lane picks up its 8 rows x 4 columns
#pragma unroll
    for (int b = 0; b < R; ++b) {
        const int r = crank * ROWS + b * (NW * 32) + wid * 32 + lane;
        const float *src = Hm + (int64_t)k * ld + k + r;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            float v[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int col = 4 * t + jj;
                v[jj] = (r < m && col < w) ? src[(int64_t)col * ld] : 0.0f;
            }
            *reinterpret_cast<float4 *>(stg + lane * kStagePitch + 4 * t) = make_float4(v[0], v[1], v[2], v[3]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = *reinterpret_cast<const float4 *>(stg + (8 * rg + i) * kStagePitch + 4 * cgp);
            p[b * 8 + i][0] = v.x;
            p[b * 8 + i][1] = v.y;
            p[b * 8 + i][2] = v.z;
            p[b * 8 + i][3] = v.w;
        }
        __syncwarp();
    }

    // Reduce-scatter of 4 per-lane values over the 4 row groups of a warp
    // (lane bits 3..4): lane (cg, rg) ends with the warp sum for column 4cg+rg.
    auto reduce_scatter4 = [&](float (&d)[4]) -> float {
        const bool up2 = rg & 2;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float send = up2 ? d[i] : d[i + 2];
            const float keep = up2 ? d[i + 2] : d[i];
            d[i] = keep + __shfl_xor_sync(kFull, send, 16);
        }
        const bool up1 = rg & 1;
        const float send = up1 ? d[0] : d[1];
        const float keep = up1 ? d[1] : d[0];
        return keep + __shfl_xor_sync(kFull, send, 8);
    };

#pragma unroll 1
    for (int cb = 0; cb < 8; ++cb) {
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const int c = cb * 4 + cc;
            if (c >= w) break;
            const int par = c & 1;

            // (1) x for my rows (p[q][cc] holds column 4*cgp+cc; the source
            // lane has cgp == cb), sigma and unscaled dots over rows > c
            float x[NR], xm[NR];
#pragma unroll
            for (int q = 0; q < NR; ++q) x[q] = __shfl_sync(kFull, p[q][cc], cb + 8 * rg);
#pragma unroll
            for (int q = 0; q < NR; ++q) xm[q] = (q < 8 && row[q] <= c) ? 0.0f : x[q];
            // (column c's own slot gives sum xm * x = sigma for free)
            float d[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                float a2[2] = {0.0f, 0.0f};
#pragma unroll
                for (int q = 0; q < NR; ++q) a2[q & 1] = fmaf(xm[q], p[q][jj], a2[q & 1]);
                d[jj] = a2[0] + a2[1];
            }
            part[par][wid][4 * cgp + rg] = reduce_scatter4(d);
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (row[q] == c) {
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) rowc_s[par][4 * cgp + jj] = p[q][jj];
                }
            __syncthreads();

            // (2) every warp: CTA (and cluster) totals, reflector, tau * w_j
            float f = 0.0f, rc;
#pragma unroll
            for (int u = 0; u < NW; ++u) f += part[par][u][lane];
            rc = rowc_s[par][lane];
            if constexpr (CLUSTER) {
                cg::cluster_group cl = cg::this_cluster();
                if (wid == 0) {
                    for (int qr = 0; qr < ncl; ++qr) {
                        float *dst = cl.map_shared_rank(&xch[par][crank][0], qr);
                        dst[lane] = f;
                        if (crank == 0) dst[32 + lane] = rc;
                    }
                }
                cl.sync();
                f = 0.0f;
                for (int qr = 0; qr < ncl; ++qr) f += xch[par][qr][lane];
                rc = xch[par][0][32 + lane];
            }
            // safety of the fast path, voted before the reflector (the vote
            // overlaps its chain): within the fast envelope |scale| <= 1e10,
            // so |d| <= 1e17 and |a(c, l)| <= 1e27 keep w_l finite
            const bool early_vote = __any_sync(kFull, !(fabsf(f) <= 1e17f) || (f != 0.0f && fabsf(f) < kDotTiny) ||
                                                          !(fabsf(rc) <= 1e27f));
            const float alpha = __shfl_sync(kFull, rc, c);
            const float sg = __shfl_sync(kFull, f, c);
            // sigma == 0 (an exactly zero tail, or one whose squares
            // underflow) also goes to the robust path, which sorts the two out
            bool fast = reflector_fast_ok(alpha, sg) && !early_vote;
            Reflector r = fast ? reflector_from_float(alpha, sg) : reflector_identity(alpha);
            float wl = rc + r.scale * f;

            if (!fast) {
                // Robust path, LAPACK order (uniform across the CTA and the
                // cluster: every warp saw the same sums).  Round 1: sigma in
                // double over rows > c.
                double sd = 0.0;
#pragma unroll
                for (int q = 0; q < NR; ++q) sd = fma((double)xm[q], (double)xm[q], sd);
                // over the 4 row groups (lane bits 3..4) only
                sd += __shfl_xor_sync(kFull, sd, 8);
                sd += __shfl_xor_sync(kFull, sd, 16);
                if (lane == 0) sigd_part[wid] = sd;
                __syncthreads();
                double sdt = 0.0;
                for (int u = 0; u < NW; ++u) sdt += sigd_part[u];
                if constexpr (CLUSTER) {
                    cg::cluster_group cl = cg::this_cluster();
                    if (wid == 0 && lane == 0)
                        for (int qr = 0; qr < ncl; ++qr) *cl.map_shared_rank(&xchd[crank], qr) = sdt;
                    cl.sync();
                    sdt = 0.0;
                    for (int qr = 0; qr < ncl; ++qr) sdt += xchd[qr];
                }
                r = reflector_from_double(alpha, sdt);
                if (sdt == 0.0) {
                    // exactly zero tail: H = I, v = e_c, w_l = a(c, l)
                    wl = rc;
                } else {
                // Round 2: w_l = v^T a_l over rows >= c with the scaled v
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    float acc = 0.0f;
#pragma unroll
                    for (int q = 0; q < NR; ++q) {
                        const bool below = q >= 8 || row[q] > c;
                        const bool diag = q < 8 && row[q] == c;
                        const float v = below ? reflector_apply(r, x[q]) : (diag ? 1.0f : 0.0f);
                        acc = fmaf(v, p[q][jj], acc);
                    }
                    d[jj] = acc;
                }
                red2[wid][4 * cgp + rg] = reduce_scatter4(d);
                __syncthreads();
                wl = 0.0f;
                for (int u = 0; u < NW; ++u) wl += red2[u][lane];
                if constexpr (CLUSTER) {
                    cg::cluster_group cl = cg::this_cluster();
                    if (wid == 0)
                        for (int qr = 0; qr < ncl; ++qr) cl.map_shared_rank(&xrb[crank][0], qr)[lane] = wl;
                    cl.sync();
                    wl = 0.0f;
                    for (int qr = 0; qr < ncl; ++qr) wl += xrb[qr][lane];
                }
                }
            }
            const float tw = (lane > c) ? r.tau * wl : 0.0f;
            if (top) {
                if (lane < c) Ysm[lane][c] = wl;  // y_l = v_l^T v_c
                if (lane == 0) tau_s[c] = r.tau;
            }

            // (3) rank-1 update of my tile; the column-c owners store v / beta
            float twv[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) twv[jj] = __shfl_sync(kFull, tw, 4 * cgp + jj);
            const bool owner = cgp == cb;
            // v = scale * x; `wide` is CTA-uniform, so branch once and keep the
            // common path free of double conversions
            float vv[NR];
            if (!r.wide) {
#pragma unroll
                for (int q = 0; q < NR; ++q) vv[q] = x[q] * r.scale;
            } else {
#pragma unroll
                for (int q = 0; q < NR; ++q) vv[q] = (float)((double)x[q] * r.scale_d);
            }
#pragma unroll
            for (int q = 0; q < NR; ++q) {
                float v;
                if (q < 8) v = row[q] > c ? vv[q] : (row[q] == c ? 1.0f : 0.0f);
                else v = vv[q];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) p[q][jj] = fmaf(-twv[jj], v, p[q][jj]);
                if (owner) {
                    if (q < 8) {
                        if (row[q] > c) p[q][cc] = v;
                        else if (row[q] == c) p[q][cc] = r.beta;
                    } else {
                        p[q][cc] = v;
                    }
                }
            }
        }
    }
    __syncthreads();
    pdl_trigger();  // the trailing update may be scheduled (it waits for this grid)

    // store: the reverse of the load (coalesced 128-byte column segments)
#pragma unroll
    for (int b = 0; b < R; ++b) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4 *>(stg + (8 * rg + i) * kStagePitch + 4 * cgp) =
                make_float4(p[b * 8 + i][0], p[b * 8 + i][1], p[b * 8 + i][2], p[b * 8 + i][3]);
        __syncwarp();
        const int r = crank * ROWS + b * (NW * 32) + wid * 32 + lane;
        float *dst = Hm + (int64_t)k * ld + k + r;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float4 v = *reinterpret_cast<const float4 *>(stg + lane * kStagePitch + 4 * t);
            const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int col = 4 * t + jj;
                if (r < m && col < w) dst[(int64_t)col * ld] = e[jj];
            }
        }
        __syncwarp();
    }

    // The trailing update needs T only through Y = T^T W; since
    // T = D (I + S D)^-1 with D = diag(tau) and S(l, c) = v_l^T v_c (l < c),
    // it solves (I + D S^T) Y = D W by forward substitution instead.  So the
    // panel stores S (strictly upper; S(l, c) at Sb + mat * s_stride + l * s_ls
    // + c * s_cs) and tau, after its rows (the top warp's stores are on the
    // kernel's critical path; measured C2 -3%).
    if (top) {
        float *Sm = Sb + mat * s_stride;
#pragma unroll 4
        for (int c = 0; c < 32; ++c) Sm[lane * s_ls + c * s_cs] = (lane < c && c < w) ? Ysm[lane][c] : 0.0f;
        if (lane < w) tau[mat * n + k + lane] = tau_s[lane];
    }
    if constexpr (CLUSTER) {
        // keep every CTA's shared memory alive until all remote writes landed
        cg::this_cluster().sync();
    }
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
        return launch_panel_t<4, 1>(H, tau, sb, batch, ld, n, k, s.cluster, st);
    if (s.warps == 4) return launch_panel_t<4, 2>(H, tau, sb, batch, ld, n, k, s.cluster, st);
    if (s.warps == 8 && s.rows_per_thread_blocks == 1)
        return launch_panel_t<8, 1>(H, tau, sb, batch, ld, n, k, s.cluster, st);
    if (s.warps == 8) return launch_panel_t<8, 2>(H, tau, sb, batch, ld, n, k, s.cluster, st);
    return launch_panel_t<16, 2>(H, tau, sb, batch, ld, n, k, s.cluster, st);
}

}  // namespace fqr
