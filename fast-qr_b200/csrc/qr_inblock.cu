// In-block steps of the rank-64 blocked QR (two 32-column panels share one
// trailing update), SIMT fp32:
//   update (GRAM = false): C2 := (I - V1 T1^T V1^T) C2 with C2 = H[k:m, k+32:k+64]
//       and V1 the unit-lower reflectors of columns k .. k+31:
//       W = V1^T C2 (32 x 32), Y = T1^T W, C2 -= V1 Y;
//   gram (GRAM = true): S12 = V1^T V2 over rows k+32 .. m-1 (V2: the
//       reflectors of columns k+32 .. k+63), the off-diagonal block of the
//       rank-64 block's S = strict_upper(V^T V).
// T1 enters through S11 = strict_upper(V1^T V1) and tau (T1 = D (I + S11 D)^-1,
// so Y solves (I + D S11^T) Y = D W by forward substitution), as in the
// trailing update.  The 64 x 64 S block is row-major: S(l, c) at l * 64 + c;
// the panels store S11 and S22 on its diagonal.
//
// The rows are split over a thread-block cluster of up to 8 CTAs (256
// threads each).  Every CTA stages its rows of both 32-column operands in
// shared memory (column-major, like H), computes its part of the 32 x 32
// product, and sends it to every CTA of the cluster through distributed
// shared memory; each CTA sums the parts in rank order, so all hold the same
// product bit for bit.  The reference has no rank-64 blocking; this follows
// the blocked restatement in oracle/geqr2.c (oracle_geqrf_blocked_f64), where
// two panels' reflectors form one block reflector.
#include <cooperative_groups.h>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace fqr {

namespace {

constexpr int kIbThreads = 256;
constexpr int kIbMaxCluster = 8;
constexpr int kIbMaxRows = 512;     // rows per CTA (shared memory: 2 x 32 x (rows + 4) floats)
constexpr int kIbTargetCtas = 296;  // two CTAs per SM on 148 SMs

struct IbShape {
    int cluster;
    int rows;  // rows per CTA, a multiple of 32
};

// Static plan by (batch, rows): as many CTAs per matrix as keep the launch
// within about two CTAs per SM (few large matrices are latency-bound, many
// matrices throughput-bound), at least 64 rows per CTA, at most 256 (two
// CTAs fit on an SM) unless that needs more than 8, then at most 512.
IbShape inblock_shape(int64_t batch, int mrows)
{
    int ncl = (int)(batch >= kIbTargetCtas ? 1 : kIbTargetCtas / batch);
    ncl = ncl < 1 ? 1 : (ncl > kIbMaxCluster ? kIbMaxCluster : ncl);
    const int by_rows = (mrows + 63) / 64;
    if (ncl > by_rows) ncl = by_rows < 1 ? 1 : by_rows;
    int need = (mrows + kIbMaxRows / 2 - 1) / (kIbMaxRows / 2);
    if (need > kIbMaxCluster) need = (mrows + kIbMaxRows - 1) / kIbMaxRows;
    if (ncl < need) ncl = need;
    const int rb = ((mrows + ncl - 1) / ncl + 31) / 32 * 32;
    return {ncl, rb};
}

size_t inblock_smem(int rb, int ncl)
{
    // two operand tiles, 4 slice partials, W, Y by column group, S11, tau,
    // one part per cluster rank
    return ((size_t)2 * 32 * (rb + 4) + 4 * 1024 + 3 * 1024 + 32 + (size_t)ncl * 1024) * sizeof(float);
}

}  // namespace

template <bool GRAM>
__global__ void __launch_bounds__(kIbThreads, 1)
inblock_kernel(float *__restrict__ H, const float *__restrict__ tau, float *__restrict__ S64, int64_t s_stride,
               int ld, int n, int k, int rb)
{
    cg::cluster_group cl = cg::this_cluster();
    const int crank = (int)cl.block_rank(), ncl = (int)cl.num_blocks();
    const int64_t mat = blockIdx.x / ncl;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // operand rows start at row k + roff of the matrix; A = V1 (columns k ..
    // k+31), B = C2 (update) or V2 (gram) (columns k+32 .. k+63)
    const int roff = GRAM ? 32 : 0;
    const int mrows = ld - k - roff;  // a multiple of 4 (ld % 4 == 0, k % 32 == 0)
    const int r0 = crank * rb;
    const int nrows = max(0, min(rb, mrows - r0));
    const int pitch = rb + 4;  // column pitch in floats: 16-byte column groups rotate by one per column
    extern __shared__ float4 ib_smem4[];
    float *As = reinterpret_cast<float *>(ib_smem4);  // A(r, j) at j * pitch + r
    float *Bs = As + 32 * pitch;
    float *part = Bs + 32 * pitch;  // [4 row slices][32 x 32]
    float *Wsm = part + 4 * 1024;   // W(i, c) at i * 32 + c
    float *Yt = Wsm + 1024;         // Y(i, c) at (c % 8) * 128 + i * 4 + c / 8
    float *Ssm = Yt + 1024;         // S11(l, j) at l * 32 + j
    float *taus = Ssm + 1024;       // 32
    float *xch = taus + 32;         // [cluster rank][32 x 32]
    float *Hm = H + mat * (int64_t)ld * n;
    const float *Abase = Hm + (int64_t)k * ld + k + roff + r0;  // A(r, j) at Abase[j * ld + r]
    float *Bbase = Hm + (int64_t)(k + 32) * ld + k + roff + r0;
    float *Sm = S64 + mat * s_stride;  // S(l, j) at Sm[l * 64 + j]

    pdl_wait();  // the panel (and everything before it) has completed

    // ---- stage this CTA's rows of A and B: 16-byte asynchronous copies (4
    // consecutive rows of a column; consecutive threads copy consecutive
    // rows), all in flight at once; rows past the matrix are zero-filled
    const int q4 = rb / 4;
    for (int idx = tid; idx < 32 * q4; idx += kIbThreads) {
        const int j = idx / q4, r = (idx - j * q4) * 4;
        const bool in = r < nrows;
        tc::cp_async16(As + j * pitch + r, in ? Abase + (int64_t)j * ld + r : Hm, in ? 16u : 0u);
        tc::cp_async16(Bs + j * pitch + r, in ? Bbase + (int64_t)j * ld + r : Hm, in ? 16u : 0u);
    }
    tc::cp_async_commit();
    if (!GRAM) {
        for (int e = tid; e < 1024; e += kIbThreads) Ssm[e] = Sm[(e >> 5) * 64 + (e & 31)];
        if (tid < 32) taus[tid] = tau[mat * n + k + tid];
    }
    tc::cp_async_wait_all();
    __syncthreads();
    // unit-lower masks, in the first CTA only (its first 32 rows): V1 (the
    // update's A) and V2 (the Gram block's B) are zero above row j of column
    // j and 1 on it (H holds R and beta there)
    if (crank == 0) {
        float *T = GRAM ? Bs : As;
        for (int e = tid; e < 1024; e += kIbThreads) {
            const int j = e >> 5, r = e & 31;
            if (r <= j) T[j * pitch + r] = (r == j) ? 1.0f : 0.0f;
        }
        __syncthreads();
    }

    // ---- W = A^T B over this CTA's rows: thread = row slice s (a quarter of
    // the rows) x a 4 x 4 block of W, i = ib + 8u, c = cb + 8v (eight
    // consecutive lanes read eight columns that sit in distinct bank groups)
    {
        const int s = tid >> 6, blk = tid & 63, ib = blk >> 3, cb = blk & 7;
        float acc[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[u][v] = 0.0f;
        const int rend = min((s + 1) * q4, nrows);
        for (int r = s * q4; r < rend; r += 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) a[u] = *reinterpret_cast<const float4 *>(As + (ib + 8 * u) * pitch + r);
#pragma unroll
            for (int v = 0; v < 4; ++v) b[v] = *reinterpret_cast<const float4 *>(Bs + (cb + 8 * v) * pitch + r);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    float t = acc[u][v];
                    t = fmaf(a[u].x, b[v].x, t);
                    t = fmaf(a[u].y, b[v].y, t);
                    t = fmaf(a[u].z, b[v].z, t);
                    t = fmaf(a[u].w, b[v].w, t);
                    acc[u][v] = t;
                }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) part[s * 1024 + (ib + 8 * u) * 32 + cb + 8 * v] = acc[u][v];
    }
    __syncthreads();
    // this CTA's product (elements 4 tid .. 4 tid + 3) to every CTA of the
    // cluster (slot crank, 16-byte stores), then the sum in rank order
    {
        const int e = 4 * tid;
        float4 w = *reinterpret_cast<const float4 *>(part + e);
#pragma unroll
        for (int sl = 1; sl < 4; ++sl) {
            const float4 p = *reinterpret_cast<const float4 *>(part + sl * 1024 + e);
            w.x += p.x;
            w.y += p.y;
            w.z += p.z;
            w.w += p.w;
        }
        for (int rk = 0; rk < ncl; ++rk)
            *reinterpret_cast<float4 *>(cl.map_shared_rank(xch, rk) + crank * 1024 + e) = w;
        cl.sync();
        float4 t = *reinterpret_cast<const float4 *>(xch + e);
        for (int rk = 1; rk < ncl; ++rk) {
            const float4 p = *reinterpret_cast<const float4 *>(xch + rk * 1024 + e);
            t.x += p.x;
            t.y += p.y;
            t.z += p.z;
            t.w += p.w;
        }
        if (GRAM) {
            if (crank == 0)
                *reinterpret_cast<float4 *>(Sm + (e >> 5) * 64 + 32 + (e & 31)) = t;  // S12(i, c), 4 consecutive c
        } else {
            *reinterpret_cast<float4 *>(Wsm + e) = t;
        }
    }
    pdl_trigger();  // the next kernel may be scheduled (it waits for this grid)
    if (GRAM) return;
    __syncthreads();

    // ---- Y = T1^T W: column c = 4 * warp + lane / 8 by the 8 lanes of a
    // lane group, lane sub holds rows l = sub + 8u; right-looking forward
    // substitution y_l = tau_l a_l, a_j -= S11(l, j) y_l for j > l
    {
        const int c = 4 * warp + (lane >> 3), sub = lane & 7;
        float a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = Wsm[(sub + 8 * u) * 32 + c];
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const int owner = l & 7, slot = l >> 3;
            const float y = __shfl_sync(kFull, taus[l] * a[slot], (lane & ~7) | owner);
            if (sub == owner) a[slot] = y;
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (sub + 8 * u > l) a[u] = fmaf(-Ssm[l * 32 + sub + 8 * u], y, a[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) Yt[(c & 7) * 128 + (sub + 8 * u) * 4 + (c >> 3)] = a[u];
    }
    __syncthreads();

    // ---- C2 -= V1 Y on this CTA's rows: warp = columns w + 8v, lane = 4
    // consecutive rows; stores go straight to H (512 contiguous bytes per
    // warp and column)
    for (int r = 4 * lane; r < nrows; r += 128) {
        float o[4][4];  // o[q][v]: row r + q, column warp + 8v
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const float4 b = *reinterpret_cast<const float4 *>(Bs + (warp + 8 * v) * pitch + r);
            o[0][v] = b.x;
            o[1][v] = b.y;
            o[2][v] = b.z;
            o[3][v] = b.w;
        }
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
            const float4 a = *reinterpret_cast<const float4 *>(As + i * pitch + r);
            const float4 y = *reinterpret_cast<const float4 *>(Yt + warp * 128 + i * 4);
            const float av[4] = {a.x, a.y, a.z, a.w}, yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int v = 0; v < 4; ++v) o[q][v] = fmaf(-av[q], yv[v], o[q][v]);
        }
#pragma unroll
        for (int v = 0; v < 4; ++v)
            *reinterpret_cast<float4 *>(Bbase + (int64_t)(warp + 8 * v) * ld + r) =
                make_float4(o[0][v], o[1][v], o[2][v], o[3][v]);
    }
}

cudaError_t launch_inblock(float *H, const float *tau, float *S64, int64_t s_stride, int64_t batch, int m, int n,
                           int k, bool gram, cudaStream_t st)
{
    const int mrows = m - k - (gram ? 32 : 0);
    if (batch <= 0 || mrows <= 0) return cudaSuccess;
    if (m % 4 != 0 || k % 32 != 0 || n - k < 64) return cudaErrorInvalidValue;
    const IbShape s = inblock_shape(batch, mrows);
    if (s.rows > kIbMaxRows || s.cluster > kIbMaxCluster) return cudaErrorInvalidValue;
    const size_t smem = inblock_smem(s.rows, s.cluster);
    auto kern = gram ? inblock_kernel<true> : inblock_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)s.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    return launch_dependent(kern, dim3((unsigned)(batch * s.cluster)), dim3(kIbThreads), smem, st, attr, 1, H,
                            tau, S64, s_stride, m, n, k, s.rows);
}

}  // namespace fqr
