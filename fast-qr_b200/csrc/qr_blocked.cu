// Blocked compact-WY Householder QR for n > 64: copy-in and SIMT
// trailing-update kernels (the panel kernel is in qr_panel.cu, the
// tensor-core trailing update in qr_trailing_tc.cu).
//
// Algorithm (tools/blocked_qr_reference.py:98-122,192-262 of the reference,
// "compact-wy" mode): for each panel of kPanel columns starting at k,
//   1. factor the (n-k) x 32 panel (unblocked Householder, LAPACK xGEQR2
//      semantics) and form the 32 x 32 upper-triangular T with
//      Q_panel = I - V T V^T;
//   2. update the trailing columns C = H[k:, k+32:] as
//      C := C - V (T^T (V^T C)).
// The reference runs the same two steps as panel_factor_kernel /
// trailing_update_kernel (submissions/candidate.py:2404-2505, :2507-2716), but
// recomputes T redundantly in every trailing CTA and applies reflectors one
// by one by default; here the panel kernel stores S = V^T V (a by-product of
// its reductions) and tau, T is never formed (the trailing update solves
// (I + D S^T) Y = D W per column, D = diag(tau)), and the trailing update is
// a blocked product.
//
// Working storage is H itself, column-major (column j of matrix b is
// contiguous): the copy-in kernel transposes the row-major input once.
#include <cooperative_groups.h>

#include "common.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace fqr {

// ---------------------------------------------------------------------------
// Copy-in: H(i, j) = A(i, j), column-major H from any-strided A.
// ---------------------------------------------------------------------------

// Row-major contiguous rows (a_cstride == 1): 32x32 tiles through shared
// memory so both the reads (rows) and the writes (columns) are coalesced.
__global__ void __launch_bounds__(256)
copy_in_rowmajor_kernel(const float *__restrict__ A, int64_t batch, int m, int n, int64_t bs, int64_t rs,
                        float *__restrict__ H, int *__restrict__ status, unsigned clear_mask)
{
    __shared__ float tile[32][33];
    pdl_trigger();  // the first panel may be scheduled; it waits for this grid
    if (status && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x < 32 &&
        ((clear_mask >> threadIdx.x) & 1u))
        status[threadIdx.x] = 0;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int j0 = blockIdx.x * 32, i0 = blockIdx.y * 32;
    for (int64_t b = blockIdx.z; b < batch; b += gridDim.z) {
        const float *Am = A + b * bs;
        float *Hm = H + b * (int64_t)m * n;
#pragma unroll
        for (int r = ty; r < 32; r += 8) {
            const int i = i0 + r, j = j0 + tx;
            tile[r][tx] = (i < m && j < n) ? __ldg(Am + (int64_t)i * rs + j) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int r = ty; r < 32; r += 8) {
            const int j = j0 + r, i = i0 + tx;
            if (i < m && j < n) Hm[(int64_t)j * m + i] = tile[tx][r];
        }
        __syncthreads();
    }
}

// Row-major rows with 16-byte alignment (a_cstride == 1; m, n, the row and
// batch strides multiples of 4; A and H 16-byte aligned): 64 x 64 tiles,
// every global access 16 bytes wide -- rows of A read as float4, columns of H
// written as float4 by 16 consecutive threads (256 contiguous bytes).
__global__ void __launch_bounds__(256)
copy_in_rowmajor_v4_kernel(const float *__restrict__ A, int64_t batch, int m, int n, int64_t bs, int64_t rs,
                           float *__restrict__ H, int *__restrict__ status, unsigned clear_mask)
{
    __shared__ float tile[64][65];
    pdl_trigger();  // the first panel may be scheduled; it waits for this grid
    if (status && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x < 32 &&
        ((clear_mask >> threadIdx.x) & 1u))
        status[threadIdx.x] = 0;
    const int t = threadIdx.x;
    const int j0 = blockIdx.x * 64, i0 = blockIdx.y * 64;
    for (int64_t b = blockIdx.z; b < batch; b += gridDim.z) {
        const float *Am = A + b * bs;
        float *Hm = H + b * (int64_t)m * n;
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
            const int f = t + 256 * s4, r = f >> 4, c4 = (f & 15) * 4;  // row, first column
            const int i = i0 + r, j = j0 + c4;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < m && j < n) v = __ldg(reinterpret_cast<const float4 *>(Am + (int64_t)i * rs + j));
            tile[r][c4] = v.x;
            tile[r][c4 + 1] = v.y;
            tile[r][c4 + 2] = v.z;
            tile[r][c4 + 3] = v.w;
        }
        __syncthreads();
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
            const int f = t + 256 * s4, c = f >> 4, r4 = (f & 15) * 4;  // column, first row
            const int j = j0 + c, i = i0 + r4;
            if (i < m && j < n)
                *reinterpret_cast<float4 *>(Hm + (int64_t)j * m + i) =
                    make_float4(tile[r4][c], tile[r4 + 1][c], tile[r4 + 2][c], tile[r4 + 3][c]);
        }
        __syncthreads();
    }
}

// Any other strides (column-major input included): one thread per element,
// writes coalesced along columns of H.
__global__ void __launch_bounds__(256)
copy_in_strided_kernel(const float *__restrict__ A, int64_t batch, int m, int n, int64_t bs, int64_t rs,
                       int64_t cs, float *__restrict__ H, int *__restrict__ status, unsigned clear_mask)
{
    pdl_trigger();
    if (status && blockIdx.x == 0 && threadIdx.x < 32 && ((clear_mask >> threadIdx.x) & 1u))
        status[threadIdx.x] = 0;
    const int64_t mn = (int64_t)m * n;
    const int64_t total = batch * mn;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = e / mn;
        const int64_t r = e - b * mn;
        const int64_t j = r / m, i = r - j * m;
        H[e] = __ldg(A + b * bs + i * rs + j * cs);
    }
}

cudaError_t launch_copy_in(const float *A, int64_t batch, int m, int n, int64_t bs, int64_t rs, int64_t cs,
                           float *H, int *status, unsigned clear_mask, cudaStream_t st)
{
    const bool v4 = cs == 1 && m % 4 == 0 && n % 4 == 0 && rs % 4 == 0 && (batch == 1 || bs % 4 == 0) &&
                    ((uintptr_t)A % 16) == 0 && ((uintptr_t)H % 16) == 0;
    if (v4) {
        dim3 grid((unsigned)((n + 63) / 64), (unsigned)((m + 63) / 64), (unsigned)(batch < 65535 ? batch : 65535));
        copy_in_rowmajor_v4_kernel<<<grid, 256, 0, st>>>(A, batch, m, n, bs, rs, H, status, clear_mask);
    } else if (cs == 1) {
        dim3 grid((unsigned)((n + 31) / 32), (unsigned)((m + 31) / 32), (unsigned)(batch < 65535 ? batch : 65535));
        copy_in_rowmajor_kernel<<<grid, 256, 0, st>>>(A, batch, m, n, bs, rs, H, status, clear_mask);
    } else {
        const int64_t total = batch * (int64_t)m * n;
        int64_t blocks = (total + 255) / 256;
        if (blocks > 148 * 64) blocks = 148 * 64;
        copy_in_strided_kernel<<<(unsigned)blocks, 256, 0, st>>>(A, batch, m, n, bs, rs, cs, H, status, clear_mask);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Trailing update (SIMT FP32): C := C - V (T^T (V^T C)) for one 32-column tile
// of one matrix per CTA.  V is the unit-lower panel H[k:, k:k+32]; T enters
// only through Y = T^T W, solved from S = V^T V (strict upper) and tau.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
trailing_simt_kernel(float *__restrict__ H, const float *__restrict__ Sws, int64_t s_stride,
                     const float *__restrict__ tau,
                     int ld, int n, int k, int c_begin)
{
    __shared__ float Vs[32][33];
    __shared__ float Cs[32][33];
    __shared__ float Ws[32][33];
    __shared__ float Ts[32][33];
    const int lane = threadIdx.x & 31, tg = threadIdx.x >> 5;
    const int64_t mat = blockIdx.y;
    const int c0 = c_begin + blockIdx.x * 32;
    const int nct = (n - c0) < 32 ? (n - c0) : 32;
    const int m = ld - k;  // rows k .. ld-1 (ld = the matrix's row count)
    float *Hm = H + mat * (int64_t)ld * n;
    pdl_wait();  // the panel (and everything before it) has completed

    auto load_chunk = [&](int r0) {
        const int rr = r0 + lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = tg + 8 * i;
            float v = 0.0f;
            if (rr < m) v = rr > j ? Hm[(int64_t)(k + j) * ld + k + rr] : (rr == j ? 1.0f : 0.0f);
            Vs[lane][j] = v;
            Cs[lane][j] = (rr < m && j < nct) ? Hm[(int64_t)(c0 + j) * ld + k + rr] : 0.0f;
        }
    };

    // W = V^T C : thread (c = lane, j = 4tg..4tg+3)
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int r0 = 0; r0 < m; r0 += 32) {
        load_chunk(r0);
        __syncthreads();
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
            const float cv = Cs[r][lane];
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[q] = fmaf(Vs[r][4 * tg + q], cv, acc[q]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) Ws[4 * tg + q][lane] = acc[q];
    const float *Sm = Sws + mat * s_stride;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int cc = tg + 8 * i;
        Ts[lane][cc] = Sm[cc * 32 + lane];  // S(lane, cc), column-major source
    }
    __syncthreads();
    // Y = T^T W with T = D (I + S D)^-1, by forward substitution per column:
    //   Y(c', col) = tau_c' (W(c', col) - sum_{l < c'} S(l, c') Y(l, col))
    if (tg == 0) {
        float y[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
            float a = Ws[c][lane];
#pragma unroll
            for (int l = 0; l < c; ++l) a = fmaf(-Ts[l][c], y[l], a);
            y[c] = tau[mat * n + k + c] * a;
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) Ws[c][lane] = y[c];
    }
    __syncthreads();
    float yreg[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) yreg[j] = Ws[j][lane];

    pdl_trigger();
    // C -= V Y : staged per 32-row chunk, thread (c = lane, rows tg + 8i)
    for (int r0 = 0; r0 < m; r0 += 32) {
        load_chunk(r0);
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = tg + 8 * i;
            float a = Cs[r][lane];
#pragma unroll
            for (int j = 0; j < 32; ++j) a = fmaf(-Vs[r][j], yreg[j], a);
            Cs[r][lane] = a;
        }
        __syncthreads();
        const int rr = r0 + lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = tg + 8 * i;
            if (rr < m && j < nct) Hm[(int64_t)(c0 + j) * ld + k + rr] = Cs[lane][j];
        }
        __syncthreads();
    }
}

cudaError_t launch_trailing(float *H, const float *Sws, int64_t s_stride, const float *tau, int64_t batch, int m,
                            int n, int k, int c_begin, cudaStream_t st)
{
    const int nc = n - c_begin;
    if (nc <= 0) return cudaSuccess;
    const unsigned tiles = (unsigned)((nc + 31) / 32);
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
        const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
        dim3 grid(tiles, (unsigned)nb);
        cudaError_t e = launch_dependent(trailing_simt_kernel, grid, dim3(256), 0, st, nullptr, 0,
                                         H + b0 * (int64_t)m * n, Sws + b0 * s_stride, s_stride, tau + b0 * n,
                                         m, n, k, c_begin);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fqr
