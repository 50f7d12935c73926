// Small-n batched Householder QR: one warp per matrix, matrix held in registers.
//
// Replaces the reference's n=32 kernel (submissions/candidate.py:146-226,
// launcher :228-248), which stages each matrix in shared memory and does one
// block-level dot reduction per (k, j) pair.  Here lane L owns columns L and
// L+32 (n <= 64) in registers; the reflector column is broadcast with warp
// shuffles so every lane forms its own dot product locally -- no reductions
// at all.  Each step makes two broadcast passes over the tail x = a(k+1:n, k):
//   pass 1: sigma = ||x||^2 and d_j = x^T a(k+1:n, j) for the lane's columns
//   (reflector: beta, tau, scale = 1/(alpha - beta))
//   pass 2: v = scale * x; a(k+1:n, j) -= tau * w_j * v, with
//           w_j = a(k, j) + scale * d_j  (= v^T a(k:n, j), v_k = 1)
// A is read in its own (row-major) layout with coalesced 128-byte row loads;
// H is written column-major through a per-warp shared-memory transpose.
#include "common.cuh"
#include "internal.h"

namespace fqr {

constexpr int kSmallWarps = 4;

template <int NP>
__global__ void __launch_bounds__(kSmallWarps * 32)
geqrf_small_kernel(const float *__restrict__ A, int64_t batch, int n, int64_t bs, int64_t rs,
                   int64_t cs, float *__restrict__ H, float *__restrict__ tau)
{
    constexpr int NC = NP / 32;
    __shared__ float stage[kSmallWarps][32][33];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int64_t mat = (int64_t)blockIdx.x * kSmallWarps + wid;
    if (mat >= batch) return;  // warp-uniform; the kernel has no block barrier

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

    float my_tau[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) my_tau[c] = 0.0f;

#pragma unroll
    for (int k = 0; k < NP - 1; ++k) {
        if (k >= n - 1) break;
        const int kc = k >> 5;   // register slot holding column k
        const int kl = k & 31;   // lane owning column k

        // pass 1: sigma and unscaled partial dots, two accumulators each
        float s0 = 0.0f, s1 = 0.0f;
        float d0[NC], d1[NC];
        bool anynz = false;
#pragma unroll
        for (int c = 0; c < NC; ++c) d0[c] = d1[c] = 0.0f;
#pragma unroll
        for (int i = k + 1; i < NP; ++i) {
            const float x = __shfl_sync(kFull, a[kc][i], kl);
            anynz |= (x != 0.0f);
            if ((i - k) & 1) {
                s0 = fmaf(x, x, s0);
#pragma unroll
                for (int c = 0; c < NC; ++c) d0[c] = fmaf(x, a[c][i], d0[c]);
            } else {
                s1 = fmaf(x, x, s1);
#pragma unroll
                for (int c = 0; c < NC; ++c) d1[c] = fmaf(x, a[c][i], d1[c]);
            }
        }
        const float alpha = __shfl_sync(kFull, a[kc][k], kl);
        const float sigma = s0 + s1;
        Reflector r = reflector_identity(alpha);
        float wv[NC];
        bool fast;
        if (!anynz) {
            fast = true;
        } else {
            fast = reflector_fast_ok(alpha, sigma);
            if (fast) r = reflector_from_float(alpha, sigma);
        }
        bool bad = false;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float dj = d0[c] + d1[c];
            wv[c] = a[c][k] + r.scale * dj;
            bad |= dot_unsafe(dj, wv[c]);
        }
        // all lanes hold identical sigma / alpha, so `fast` is warp-uniform;
        // the dot check is per lane and is made uniform by the vote
        if (fast && anynz) fast = !__any_sync(kFull, bad);
        if (!fast) {
            // LAPACK order: sigma in double, then v, then w_j = v^T a_j
            double sd = 0.0;
#pragma unroll
            for (int i = k + 1; i < NP; ++i) {
                const double x = (double)__shfl_sync(kFull, a[kc][i], kl);
                sd = fma(x, x, sd);
            }
            r = reflector_from_double(alpha, sd);
#pragma unroll
            for (int c = 0; c < NC; ++c) wv[c] = a[c][k];
#pragma unroll
            for (int i = k + 1; i < NP; ++i) {
                const float v = reflector_apply(r, __shfl_sync(kFull, a[kc][i], kl));
#pragma unroll
                for (int c = 0; c < NC; ++c) wv[c] = fmaf(v, a[c][i], wv[c]);
            }
        }

        float tw[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int j = lane + 32 * c;
            tw[c] = (j > k) ? r.tau * wv[c] : 0.0f;
            a[c][k] -= tw[c];  // row k: v_k = 1
        }
        if (lane == kl) a[kc][k] = r.beta;

        // pass 2: apply the reflector below row k; the owner lane stores v
#pragma unroll
        for (int i = k + 1; i < NP; ++i) {
            const float x = __shfl_sync(kFull, a[kc][i], kl);
            const float v = reflector_apply(r, x);
#pragma unroll
            for (int c = 0; c < NC; ++c) a[c][i] = fmaf(-tw[c], v, a[c][i]);
            if (lane == kl) a[kc][i] = v;
        }
        if (lane == kl) my_tau[kc] = r.tau;
    }

    // column-major store through a 32x33 shared-memory transpose per warp
    float *Hm = H + mat * (int64_t)n * n;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
        for (int rb = 0; rb < NC; ++rb) {
#pragma unroll
            for (int ii = 0; ii < 32; ++ii) stage[wid][lane][ii] = a[c][rb * 32 + ii];
            __syncwarp();
            const int i = rb * 32 + lane;
#pragma unroll 8
            for (int jj = 0; jj < 32; ++jj) {
                const int j = c * 32 + jj;
                if (j < n && i < n) Hm[(int64_t)j * n + i] = stage[wid][jj][lane];
            }
            __syncwarp();
        }
        const int j = c * 32 + lane;
        if (j < n) tau[mat * n + j] = my_tau[c];
    }
}

cudaError_t launch_small(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs,
                         float *H, float *tau, cudaStream_t st)
{
    const int64_t blocks = (batch + kSmallWarps - 1) / kSmallWarps;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    dim3 grid((unsigned)blocks), block(kSmallWarps * 32);
    if (n <= 32)
        geqrf_small_kernel<32><<<grid, block, 0, st>>>(A, batch, n, bs, rs, cs, H, tau);
    else
        geqrf_small_kernel<64><<<grid, block, 0, st>>>(A, batch, n, bs, rs, cs, H, tau);
    return cudaGetLastError();
}

}  // namespace fqr
