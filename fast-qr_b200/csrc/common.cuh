// Shared device helpers for the fastqr kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fqr {

constexpr unsigned kFull = 0xffffffffu;

// Householder reflector for one column, LAPACK xLARFG semantics
// (the reference's per-column step: submissions/candidate.py:176-196 in the
// n=32 kernel, :2084-2098 in the blocked panel).  Given alpha = a(k,k) and
// sigma = ||a(k+1:m, k)||^2:
//   sigma == 0 -> tau = 0, beta = alpha, v = x unchanged (H = I)
//   otherwise  -> beta = -sign(alpha) * sqrt(alpha^2 + sigma),
//                 tau = (beta - alpha) / beta,  v = x / (alpha - beta).
// `scale` multiplies x to give v.  When that factor is not representable in
// float (tiny columns), `wide` is set and v must be formed as
// float(double(x) * scale_d); |v| <= 1 always, so the product is safe.
struct Reflector {
    float beta;
    float tau;
    float scale;
    double scale_d;
    bool wide;
};

// Fast path valid when sigma and alpha are far from float over/underflow.
__device__ __forceinline__ bool reflector_fast_ok(float alpha, float sigma) {
    return sigma >= 1e-30f && sigma <= 1e30f && fabsf(alpha) <= 1e15f;
}

__device__ __forceinline__ Reflector reflector_from_float(float alpha, float sigma) {
    Reflector r;
    float rr = sqrtf(fmaf(alpha, alpha, sigma));
    r.beta = signbit(alpha) ? rr : -rr;
    r.tau = (r.beta - alpha) / r.beta;
    r.scale = 1.0f / (alpha - r.beta);
    r.scale_d = (double)r.scale;
    r.wide = false;
    return r;
}

// Robust path: sigma accumulated in double by the caller.
__device__ __forceinline__ Reflector reflector_from_double(float alpha, double sigma) {
    Reflector r;
    if (sigma == 0.0) {
        r.beta = alpha;
        r.tau = 0.0f;
        r.scale = 1.0f;
        r.scale_d = 1.0;
        r.wide = false;
        return r;
    }
    double a = (double)alpha;
    double rr = sqrt(fma(a, a, sigma));
    double b = signbit(alpha) ? rr : -rr;
    r.beta = (float)b;
    r.tau = (float)((b - a) / b);
    r.scale_d = 1.0 / (a - b);
    r.scale = (float)r.scale_d;
    r.wide = !(fabs(r.scale_d) <= 1e30);
    return r;
}

__device__ __forceinline__ float reflector_apply(const Reflector &r, float x) {
    return r.wide ? (float)((double)x * r.scale_d) : x * r.scale;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

}  // namespace fqr
