// Q formation and application for the compact (H, tau) that geqrf returns.
//
//   fqr_orgqr_f32 : Q = H_0 H_1 ... H_{n-1}           (torch.linalg.householder_product)
//   fqr_ormqr_f32 : C := Q^T C  or  C := Q C, in place  (torch.ormqr, left side)
//
// Blocked path (n % 4 == 0, n >= 128, 16-byte aligned H and C): gram_kernel
// forms every panel's S_p = strict_upper(V_p^T V_p) once, then each panel's
// block reflector I - V T V^T (or its transpose, T = D (I + S D)^-1, never
// formed) is applied by the tensor-core update kernel of qr_trailing_tc.cu.
// orgqr runs backward from Q = I and touches rows and columns >= k of panel
// k only (the order of LAPACK xORGQR); ormqr runs forward (Q^T) or backward
// (Q) over all columns of C.  Other n up to 512: apply_small_kernel, one
// reflector after the other, each group of 4 threads owning one column of C
// in shared memory.
#include <cuda_runtime.h>

#include "../../include/fastqr.h"
#include "internal.h"

namespace fqr {
namespace {

constexpr int kSmallMaxN = 512;
constexpr int kSmallCols = 64;  // columns of C per CTA of the small path

// S_p (32 x 32, column-major, strictly upper; 0 elsewhere) of panel p of
// matrix mat at S[(mat * panels + p) * 1024].  V is unit lower triangular:
// rows r < j of column j are 0, row j is 1; columns past n are 0.
__global__ void __launch_bounds__(256) gram_kernel(const float *__restrict__ H, int n, int panels,
                                                   float *__restrict__ S)
{
    __shared__ float vs[128][33];
    const int p = blockIdx.x, k = p * kPanel;
    const int64_t mat = blockIdx.y;
    const int m = n - k, w = m < kPanel ? m : kPanel;
    const float *Vb = H + mat * (int64_t)n * n + (int64_t)k * n + k;
    const int t = threadIdx.x;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int r0 = 0; r0 < m; r0 += 128) {
        // 128 rows x 32 columns; consecutive threads read consecutive rows
        for (int idx = t; idx < 128 * kPanel; idx += 256) {
            const int r = idx & 127, j = idx >> 7, rr = r0 + r;
            float v = 0.0f;
            if (j < w && rr < m) v = rr > j ? Vb[(int64_t)j * n + rr] : (rr == j ? 1.0f : 0.0f);
            vs[r][j] = v;
        }
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q = t + 256 * e, l = q & 31, c = q >> 5;
            float a = acc[e];
#pragma unroll 8
            for (int r = 0; r < 128; ++r) a = fmaf(vs[r][l], vs[r][c], a);
            acc[e] = a;
        }
        __syncthreads();
    }
    float *Sm = S + (mat * panels + p) * (kPanel * kPanel);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int q = t + 256 * e, l = q & 31, c = q >> 5;
        Sm[c * kPanel + l] = l < c ? acc[e] : 0.0f;
    }
}

// Q := I (column-major n x n per matrix)
__global__ void identity_kernel(float *__restrict__ Q, int64_t total, int n)
{
    const int64_t nn = (int64_t)n * n;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = i % nn;
        Q[i] = (e / n == e % n) ? 1.0f : 0.0f;
    }
}

// Applies the n reflectors of H to columns [blockIdx.x * 64, +64) of C
// (n x ncols per matrix): ascending order (Q^T C) or descending (Q C).  The
// column block sits in shared memory with a pitch of 4 (mod 32) floats, so
// the 8 columns x 4 row phases of a warp hit 32 distinct banks; each group of
// 4 threads owns one column and needs no CTA barrier between reflectors.
__global__ void __launch_bounds__(256) apply_small_kernel(const float *__restrict__ H,
                                                          const float *__restrict__ tau, int n,
                                                          float *__restrict__ C, int64_t ncols,
                                                          int ascending, int pitch)
{
    extern __shared__ float cs[];
    const int64_t mat = blockIdx.y;
    const int64_t c0 = (int64_t)blockIdx.x * kSmallCols;
    const int nc = (int)((ncols - c0) < kSmallCols ? (ncols - c0) : kSmallCols);
    float *Cm = C + mat * (int64_t)n * ncols + c0 * n;
    for (int idx = threadIdx.x; idx < nc * n; idx += blockDim.x) {
        const int c = idx / n, r = idx % n;
        cs[c * pitch + r] = Cm[(int64_t)c * n + r];
    }
    __syncthreads();
    // every thread runs the loop (the shuffles need whole warps); columns past
    // nc hold stale shared memory and are never written back
    const int cl = threadIdx.x >> 2, part = threadIdx.x & 3;
    const float *Hm = H + mat * (int64_t)n * n;
    const float *tm = tau + mat * n;
    {
        float *col = cs + cl * pitch;
        for (int s = 0; s < n; ++s) {
            const int j = ascending ? s : n - 1 - s;
            const float tj = __ldg(tm + j);
            const float *v = Hm + (int64_t)j * n;  // v_j = 1, v_r = H(r, j) for r > j
            float sum = 0.0f;
            for (int r = j + part; r < n; r += 4) sum = fmaf(r == j ? 1.0f : __ldg(v + r), col[r], sum);
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            const float tw = tj * sum;
            for (int r = j + part; r < n; r += 4) col[r] = fmaf(-tw, r == j ? 1.0f : __ldg(v + r), col[r]);
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < nc * n; idx += blockDim.x) {
        const int c = idx / n, r = idx % n;
        Cm[(int64_t)c * n + r] = cs[c * pitch + r];
    }
}

// Blocked path without the tensor cores (n > 512 where the tensor-core path
// cannot run: n % 4 != 0, or H or C not 16-byte aligned).  Applies panel k's
// block reflector to a 32-column tile of C (rows k .. n-1, columns c0 ..):
// QT: C := (I - V T V^T)^T C = (I - V T^T V^T) C, Y = T^T W by forward
// substitution (the geqrf trailing update); otherwise C := (I - V T V^T) C,
// Y = T W = D (I + S D)^-1 W by backward substitution,
//   Y(c) = tau_c (W(c) - sum_{l > c} S(c, l) Y(l)).
// A last panel of w < 32 reflectors has zero columns w .. 31 (tau 0).
template <bool QT>
__global__ void __launch_bounds__(256) apply_simt_kernel(const float *__restrict__ H, const float *__restrict__ S,
                                                         int64_t s_stride, const float *__restrict__ tau, int n,
                                                         int k, float *__restrict__ C, int64_t ncols,
                                                         int64_t c_begin, int64_t c_end)
{
    __shared__ float Vs[32][33];
    __shared__ float Cs[32][33];
    __shared__ float Ws[32][33];
    __shared__ float Ts[32][33];
    const int lane = threadIdx.x & 31, tg = threadIdx.x >> 5;
    const int64_t mat = blockIdx.y;
    const int64_t c0 = c_begin + (int64_t)blockIdx.x * 32;
    const int nct = (int)((c_end - c0) < 32 ? (c_end - c0) : 32);
    const int m = n - k;
    const int w = m < kPanel ? m : kPanel;
    const float *Hm = H + mat * (int64_t)n * n;
    float *Cm = C + mat * (int64_t)n * ncols;

    // chunk of 32 rows: V (unit lower, columns >= w zero) and the C tile
    auto load_chunk = [&](int r0) {
        const int rr = r0 + lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = tg + 8 * i;
            float v = 0.0f;
            if (rr < m && j < w) v = rr > j ? Hm[(int64_t)(k + j) * n + k + rr] : (rr == j ? 1.0f : 0.0f);
            Vs[lane][j] = v;
            Cs[lane][j] = (rr < m && j < nct) ? Cm[(c0 + j) * n + k + rr] : 0.0f;
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
    const float *Sm = S + mat * s_stride;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int cc = tg + 8 * i;
        Ts[lane][cc] = Sm[cc * kPanel + lane];  // S(lane, cc), column-major source
    }
    __syncthreads();
    if (tg == 0) {
        float y[32];
        if constexpr (QT) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                float a = Ws[c][lane];
#pragma unroll
                for (int l = 0; l < c; ++l) a = fmaf(-Ts[l][c], y[l], a);
                y[c] = (c < w ? tau[mat * n + k + c] : 0.0f) * a;
            }
        } else {
#pragma unroll
            for (int c = 31; c >= 0; --c) {
                float a = Ws[c][lane];
#pragma unroll
                for (int l = c + 1; l < 32; ++l) a = fmaf(-Ts[c][l], y[l], a);
                y[c] = (c < w ? tau[mat * n + k + c] : 0.0f) * a;
            }
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) Ws[c][lane] = y[c];
    }
    __syncthreads();
    float yreg[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) yreg[j] = Ws[j][lane];

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
            if (rr < m && j < nct) Cm[(c0 + j) * n + k + rr] = Cs[lane][j];
        }
        __syncthreads();
    }
}

bool apply_tc_ok(int64_t n, const void *H, const void *C)
{
    return trailing_tc_supported((int)n) && ((uintptr_t)H % 16) == 0 && ((uintptr_t)C % 16) == 0;
}

int panels_of(int64_t n) { return (int)((n + kPanel - 1) / kPanel); }

size_t apply_ws_bytes(int64_t batch, int64_t n)
{
    return (size_t)batch * panels_of(n) * kPanel * kPanel * sizeof(float) + kWsAlign;
}

int status_of(cudaError_t e) { return e == cudaSuccess ? FQR_OK : FQR_ELAUNCH; }

// mode: 0 orgqr (C = Q, starts from I), 1 ormqr with Q^T, 2 ormqr with Q
int run_apply(const float *H, const float *tau, int64_t batch, int64_t n, float *C, int64_t ncols, int mode,
              void *ws, size_t ws_bytes, cudaStream_t st)
{
    if (batch < 0 || n < 0 || ncols < 0) return FQR_EINVAL;
    if (batch == 0 || n == 0 || ncols == 0) return FQR_OK;
    if (n > FQR_MAX_N) return FQR_EUNSUPPORTED;
    if (!H || !tau || !C) return FQR_EINVAL;
    const int ni = (int)n;
    const bool tc = apply_tc_ok(n, H, C);
    // n > 512 off the tensor-core path: the same blocked order with the SIMT
    // update (apply_simt_kernel); smaller such n: one reflector at a time
    const bool blocked = tc || n > kSmallMaxN;
    const size_t need = apply_ws_bytes(batch, n);
    // every argument check before the first CUDA call
    if (blocked && (!ws || ws_bytes < need)) return FQR_EWORKSPACE;
    if (blocked && ((uintptr_t)ws) % kWsAlign) return FQR_EINVAL;
    cudaError_t e;
    if (mode == 0) {
        const int64_t total = batch * n * n;
        const int64_t blocks = (total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096;
        identity_kernel<<<(unsigned)blocks, 256, 0, st>>>(C, total, ni);
        if ((e = cudaGetLastError()) != cudaSuccess) return status_of(e);
    }
    if (!blocked) {
        const int pitch = (ni + 31) / 32 * 32 + 4;
        const size_t smem = (size_t)kSmallCols * pitch * sizeof(float);
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(apply_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
            return FQR_ELAUNCH;
        for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
            const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
            dim3 grid((unsigned)((ncols + kSmallCols - 1) / kSmallCols), (unsigned)nb);
            apply_small_kernel<<<grid, 256, smem, st>>>(H + b0 * n * n, tau + b0 * n, ni, C + b0 * n * ncols,
                                                        ncols, mode == 1 ? 1 : 0, pitch);
            if ((e = cudaGetLastError()) != cudaSuccess) return status_of(e);
        }
        return FQR_OK;
    }
    const int panels = panels_of(n);
    float *S = (float *)ws;
    int *status = (int *)((unsigned char *)ws + need - kWsAlign);
    if ((e = cudaMemsetAsync(status, 0, sizeof(int), st)) != cudaSuccess) return status_of(e);
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
        const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
        gram_kernel<<<dim3((unsigned)panels, (unsigned)nb), 256, 0, st>>>(H + b0 * n * n, ni, panels,
                                                                         S + b0 * panels * kPanel * kPanel);
        if ((e = cudaGetLastError()) != cudaSuccess) return status_of(e);
    }
    const int64_t s_stride = (int64_t)panels * kPanel * kPanel;
    if (!tc) {
        for (int s = 0; s < panels; ++s) {
            const int p = mode == 1 ? s : panels - 1 - s;
            const int k = p * kPanel;
            const int64_t cb = mode == 0 ? k : 0, ce = mode == 0 ? n : ncols;
            for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
                const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
                const dim3 grid((unsigned)((ce - cb + 31) / 32), (unsigned)nb);
                const float *Sp = S + b0 * s_stride + (int64_t)p * kPanel * kPanel;
                float *Cb = C + b0 * n * (mode == 0 ? n : ncols);
                if (mode == 1)
                    apply_simt_kernel<true><<<grid, 256, 0, st>>>(H + b0 * n * n, Sp, s_stride, tau + b0 * n, ni, k,
                                                                  Cb, mode == 0 ? n : ncols, cb, ce);
                else
                    apply_simt_kernel<false><<<grid, 256, 0, st>>>(H + b0 * n * n, Sp, s_stride, tau + b0 * n, ni,
                                                                   k, Cb, mode == 0 ? n : ncols, cb, ce);
                if ((e = cudaGetLastError()) != cudaSuccess) return status_of(e);
            }
        }
        return FQR_OK;
    }
    TrailingMaps maps;
    if (prepare_apply_maps(H, ni, ni, C, mode == 0 ? n : ncols, batch, &maps) != cudaSuccess) return FQR_ECUDA;
    for (int s = 0; s < panels; ++s) {
        const int p = mode == 1 ? s : panels - 1 - s;
        const int k = p * kPanel;
        const int cb = mode == 0 ? k : 0, ce = mode == 0 ? ni : (int)ncols;
        e = launch_apply_tc(maps, H, S + (int64_t)p * kPanel * kPanel, s_stride, tau, status, batch, ni, ni, k,
                            cb, ce, mode == 1, st);
        if (e != cudaSuccess) return status_of(e);
    }
    return FQR_OK;
}

}  // namespace
}  // namespace fqr

extern "C" {

size_t fqr_orgqr_workspace_bytes(int64_t batch, int64_t n)
{
    if (batch <= 0 || n <= 0 || n > FQR_MAX_N) return 0;
    if (!fqr::trailing_tc_supported((int)n) && n <= fqr::kSmallMaxN) return 0;
    return fqr::apply_ws_bytes(batch, n);
}

int fqr_orgqr_f32(const float *H, const float *tau, int64_t batch, int64_t n, float *Q, void *workspace,
                  size_t workspace_bytes, void *stream)
{
    return fqr::run_apply(H, tau, batch, n, Q, n, 0, workspace, workspace_bytes, (cudaStream_t)stream);
}

int fqr_ormqr_f32(const float *H, const float *tau, int64_t batch, int64_t n, float *C, int64_t ncols,
                  int transpose, void *workspace, size_t workspace_bytes, void *stream)
{
    return fqr::run_apply(H, tau, batch, n, C, ncols, transpose ? 1 : 2, workspace, workspace_bytes,
                          (cudaStream_t)stream);
}

// C Q = (Q^T C^T)^T and C Q^T = (Q C^T)^T: a row-major mrows x n C is, read
// column-major, the n x mrows matrix C^T, so the right-side product is the
// left-side one on the same buffer with the transpose flag flipped.
int fqr_ormqr_right_f32(const float *H, const float *tau, int64_t batch, int64_t n, float *C, int64_t mrows,
                        int transpose, void *workspace, size_t workspace_bytes, void *stream)
{
    return fqr::run_apply(H, tau, batch, n, C, mrows, transpose ? 2 : 1, workspace, workspace_bytes,
                          (cudaStream_t)stream);
}

}  // extern "C"
