// Small-n batched Householder QR: one warp per matrix, matrix held in registers.
//
// Replaces the reference's n=32 kernel (submissions/candidate.py:146-226,
// launcher :228-248), which stages each matrix in shared memory and does one
// block-level dot reduction per (k, j) pair.  Here lane L owns column L (and
// column L+32 when n > 32) in registers and the reflector column is broadcast
// with warp shuffles, so every lane forms its own dot product locally -- no
// reductions at all.
//
// Sliding register window: after step k the lane's column is shifted up one
// row (the finished row k goes to a shared-memory stage), so at every step
// the pivot row is a[0] and the tail x is a[1..]; rows below the matrix shift
// in as zeros.  All register indices are compile-time constants, the step
// loop is a runtime loop over one small body (the instruction cache holds
// it; a fully unrolled step loop stalls on instruction fetch), and no row
// masks or branches sit in the inner loops, so the shuffles pipeline.
// Per step k:
//   x_i = a_owner[i] (shuffle from the lane owning column k), i = 1..
//   sigma = ||x||^2,  d = x^T a[1..]  (unscaled, one pass)
//   beta, tau, scale = 1 / (alpha - beta)   (LAPACK xLARFG convention)
//   w = a[0] + scale * d,  a[0] -= tau w,  a[i] -= tau * w * scale * x_i
//   the owner lane stores beta and v = scale * x instead.
// The shared-memory stage then holds the factor transposed for coalesced
// column-major stores of H.
#include "common.cuh"
#include "internal.h"

namespace fqr {

constexpr int kSmallWarps = 4;

// One step of the sliding-window factorisation for register slot S (the
// slot holding column k; lanes with a column j <= k are left unchanged).
// The owner lane keeps its column unscaled (x, not v = scale * x) so the
// update needs no per-element select; its scale is recorded and applied when
// the factor is written out.  Only the first W window rows are touched: the
// caller guarantees rows W .. NP-1 are zero (after k steps the window holds
// rows k .. k+NP-1 of the matrix, and rows n .. are zero), so skipping them
// changes no bit of the result.
template <int NP, int NC, int S, int W>
__device__ __forceinline__ void small_step(float (&a)[NC][NP], int k, int lane, float *stage_row,
                                           float *tau_stage, float *scale_stage,
                                           double *scaled_stage)
{
    const int kl = k & 31;
    const bool owner = lane == kl;
    float x[W];
    float d0[NC], d1[NC];
    uint32_t nzbits = 0;  // OR of |x_i|'s bit patterns: 0 iff the tail is exactly zero
#pragma unroll
    for (int c = 0; c < NC; ++c) d0[c] = d1[c] = 0.0f;
    const float alpha = __shfl_sync(kFull, a[S][0], kl);
#pragma unroll
    for (int i = 1; i < W; ++i) {
        x[i] = __shfl_sync(kFull, a[S][i], kl);
        nzbits |= __float_as_uint(x[i]) & 0x7fffffffu;
        if (i & 1) {
#pragma unroll
            for (int c = 0; c < NC; ++c) d0[c] = fmaf(x[i], a[c][i], d0[c]);
        } else {
#pragma unroll
            for (int c = 0; c < NC; ++c) d1[c] = fmaf(x[i], a[c][i], d1[c]);
        }
    }
    const bool anynz = nzbits != 0;
    // sigma = x^T x is the owner's own dot (its slot S holds column k, whose
    // rows 1.. are x): the same FMAs in the same order, one shuffle instead of
    // a second reduction in every lane
    const float sigma = __shfl_sync(kFull, d0[S] + d1[S], kl);
    Reflector r = reflector_identity(alpha);
    bool fast = true;
    if (anynz) {
        fast = reflector_fast_ok(alpha, sigma);
        if (fast) r = reflector_from_float(alpha, sigma);
    }
    // fast path: a(i, j) -= (tau * w_j * scale) * x_i, one FMA per element
    float tw[NC], tws[NC];
    bool bad = false;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int j = lane + 32 * c;
        const float dj = d0[c] + d1[c];
        const float wj = a[c][0] + r.scale * dj;
        tw[c] = (j > k) ? r.tau * wj : 0.0f;
        tws[c] = tw[c] * r.scale;
        bad |= dot_unsafe(dj, wj) || !isfinite(tws[c]);
    }
    // sigma / alpha are identical in all lanes, so `fast` is warp-uniform;
    // the per-lane checks are made uniform by the vote
    if (fast && anynz) fast = !__any_sync(kFull, bad);
    float rowk[NC];  // finished row k (v_k = 1), taken before the window shifts
    if (fast) {
#pragma unroll
        for (int c = 0; c < NC; ++c) rowk[c] = (owner && c == S) ? r.beta : a[c][0] - tw[c];
#pragma unroll
        for (int i = 1; i < W; ++i) {
#pragma unroll
            for (int c = 0; c < NC; ++c) a[c][i - 1] = fmaf(-tws[c], x[i], a[c][i]);
        }
    } else {
        // LAPACK order: sigma in double, then v, then w_j = v^T a_j
        double sd = 0.0;
#pragma unroll
        for (int i = 1; i < W; ++i) sd = fma((double)x[i], (double)x[i], sd);
        r = reflector_from_double(alpha, sd);
        float wv[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) wv[c] = a[c][0];
#pragma unroll
        for (int i = 1; i < W; ++i) {
            const float v = reflector_apply(r, x[i]);
#pragma unroll
            for (int c = 0; c < NC; ++c) wv[c] = fmaf(v, a[c][i], wv[c]);
        }
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int j = lane + 32 * c;
            tw[c] = (j > k) ? r.tau * wv[c] : 0.0f;
            rowk[c] = (owner && c == S) ? r.beta : a[c][0] - tw[c];
        }
#pragma unroll
        for (int i = 1; i < W; ++i) {
            const float v = reflector_apply(r, x[i]);
#pragma unroll
            for (int c = 0; c < NC; ++c) a[c][i - 1] = fmaf(-tw[c], v, a[c][i]);
        }
    }
    // finished row k (shifted out above), and the owner's column scale
#pragma unroll
    for (int c = 0; c < NC; ++c) stage_row[32 * c] = rowk[c];
    if (lane == 0) {
        tau_stage[k] = r.tau;
        scale_stage[k] = r.wide ? 0.0f : r.scale;
        scaled_stage[k] = r.scale_d;
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) a[c][W - 1] = 0.0f;
}

// Steps [8P, min(8P + 8, kend)) with the window W = NP - 8P (rows past it are
// zero: 8P steps have shifted NP >= n rows up by 8P), then the next phase.
// Eight steps per phase keep one compact runtime loop per phase (NP / 8
// copies of the step body in all) while the per-step work shrinks with the
// tail: sum over steps of W is ~(NP^2 / 2) instead of NP^2.
template <int NP, int NC, int P>
__device__ __forceinline__ void small_phases(float (&a)[NC][NP], int kend, int lane, float *stage, int ld,
                                             float *tau_stage, float *scale_stage, double *scaled_stage)
{
    constexpr int W = NP - 8 * P;
    constexpr int S = (8 * P) / 32;  // register slot of columns 8P .. 8P+7
    const int kb = 8 * P, ke = kend < kb + 8 ? kend : kb + 8;
#pragma unroll 1
    for (int k = kb; k < ke; ++k)
        small_step<NP, NC, S, W>(a, k, lane, stage + k * ld + lane, tau_stage, scale_stage, scaled_stage);
    if constexpr (P + 1 < NP / 8) {
        if (kend > kb + 8)
            small_phases<NP, NC, P + 1>(a, kend, lane, stage, ld, tau_stage, scale_stage, scaled_stage);
    }
}

// The final row (k = n-1) has an empty tail: tau = 0, the row is unchanged.
template <int NP, int NC>
__device__ __forceinline__ void small_last_row(float (&a)[NC][NP], float *stage_row)
{
#pragma unroll
    for (int c = 0; c < NC; ++c) stage_row[32 * c] = a[c][0];
}

template <int NP>
__global__ void __launch_bounds__(kSmallWarps * 32)
geqrf_small_kernel(const float *__restrict__ A, int64_t batch, int n, int64_t bs, int64_t rs,
                   int64_t cs, float *__restrict__ H, float *__restrict__ tau)
{
    constexpr int NC = NP / 32;
    constexpr int LD = NP + 1;  // stage row stride (columns), padded
    constexpr int WS = NP * LD + 2 * NP + 2 * NP;  // floats per warp: stage, tau, scale, scale_d
    extern __shared__ float smem_small[];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int64_t mat = (int64_t)blockIdx.x * kSmallWarps + wid;
    if (mat >= batch) return;  // warp-uniform; the kernel has no block barrier
    float *stage = smem_small + wid * WS;  // [row][col]
    float *tau_stage = stage + NP * LD;
    float *scale_stage = tau_stage + NP;
    double *scaled_stage = reinterpret_cast<double *>(scale_stage + NP);  // 8-byte aligned

    float a[NC][NP];
    const float *Am = A + mat * bs;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int j = lane + 32 * c;
        const bool jin = j < n;
#pragma unroll
        for (int i = 0; i < NP; ++i)
            a[c][i] = (jin && i < n) ? __ldg(Am + (int64_t)i * rs + (int64_t)j * cs) : 0.0f;
    }

    // steps 0 .. n-2 (the last row has an empty tail)
    small_phases<NP, NC, 0>(a, n - 1, lane, stage, LD, tau_stage, scale_stage, scaled_stage);
    small_last_row<NP, NC>(a, stage + (n - 1) * LD + lane);
    if (lane == 0) tau_stage[n - 1] = 0.0f;
    __syncwarp();

    // column-major store: lanes write consecutive rows of one column; rows
    // below the diagonal hold x and become v = scale_j * x here
    float *Hm = H + mat * (int64_t)n * n;
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
        const float sj = j < n - 1 ? scale_stage[j] : 1.0f;
        const bool widej = j < n - 1 && sj == 0.0f;
        const double sdj = widej ? scaled_stage[j] : 1.0;
#pragma unroll
        for (int rb = 0; rb < NC; ++rb) {
            const int i = rb * 32 + lane;
            if (i < n) {
                float h = stage[i * LD + j];
                if (i > j) h = widej ? (float)((double)h * sdj) : h * sj;
                Hm[(int64_t)j * n + i] = h;
            }
        }
    }
#pragma unroll
    for (int rb = 0; rb < NC; ++rb) {
        const int i = rb * 32 + lane;
        if (i < n) tau[mat * n + i] = tau_stage[i];
    }
}

template <int NP>
static size_t small_smem_bytes()
{
    return (size_t)kSmallWarps * (NP * (NP + 1) + 4 * NP) * sizeof(float);
}

cudaError_t launch_small(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs,
                         float *H, float *tau, cudaStream_t st)
{
    const int64_t blocks = (batch + kSmallWarps - 1) / kSmallWarps;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    dim3 grid((unsigned)blocks), block(kSmallWarps * 32);
    if (n <= 32) {
        geqrf_small_kernel<32><<<grid, block, small_smem_bytes<32>(), st>>>(A, batch, n, bs, rs, cs, H, tau);
    } else {
        const size_t smem = small_smem_bytes<64>();
        cudaError_t e = cudaFuncSetAttribute(geqrf_small_kernel<64>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        geqrf_small_kernel<64><<<grid, block, smem, st>>>(A, batch, n, bs, rs, cs, H, tau);
    }
    return cudaGetLastError();
}

}  // namespace fqr
