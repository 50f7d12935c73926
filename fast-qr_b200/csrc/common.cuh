// Shared device helpers for the fastqr kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fqr {

constexpr unsigned kFull = 0xffffffffu;

// Programmatic dependent launch (kernels launched by launch_dependent):
// pdl_wait blocks the calling thread until every kernel this one depends on
// has completed and its memory operations are visible (a no-op when the
// kernel was launched without the attribute); pdl_trigger lets the next
// kernel on the stream be scheduled once every CTA of this one has issued it
// or exited -- it carries no memory ordering.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

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

// The fast kernels form the dot products d_j = x^T a_j with the UNSCALED tail
// x in the same reduction as sigma = ||x||^2 (one reduction per column instead
// of LAPACK's two) and rescale afterwards: w_j = a(k,j) + scale * d_j.  That is
// exact arithmetic-wise but the products x_i a_ij can over/underflow when x is
// far from unit scale.  The fast path is therefore taken only when
//   sigma in [1e-20, 1e20]  (||x|| in [1e-10, 1e10]) and |alpha| <= 1e15,
// and, checked after the reduction, every d_j is finite and not in the
// denormal-product regime (0 < |d_j| < 1e-30); the panel kernel checks the
// stricter |d_j| <= 1e17 and |a(k,j)| <= 1e27 instead, which bound w_j
// without the reflector (|scale| <= 1e10 in the envelope), so its vote
// overlaps the reflector's computation.  Otherwise the column is redone
// in LAPACK order: sigma in double, v = x / (alpha - beta), then w_j = v^T a_j.
constexpr float kSigmaLo = 1e-20f;
constexpr float kSigmaHi = 1e20f;
constexpr float kAlphaHi = 1e15f;
constexpr float kDotTiny = 1e-30f;

__device__ __forceinline__ bool reflector_fast_ok(float alpha, float sigma) {
    return sigma >= kSigmaLo && sigma <= kSigmaHi && fabsf(alpha) <= kAlphaHi;
}

// A fused dot product that the fast path may not use.
__device__ __forceinline__ bool dot_unsafe(float d, float w) {
    return !isfinite(w) || (d != 0.0f && fabsf(d) < kDotTiny);
}

// tau = 0 reflector (exactly zero tail): H = I, v = x = 0.
__device__ __forceinline__ Reflector reflector_identity(float alpha) {
    Reflector r;
    r.beta = alpha;
    r.tau = 0.0f;
    r.scale = 1.0f;
    r.scale_d = 1.0;
    r.wide = false;
    return r;
}

// Inside the fast envelope (sigma in [1e-20, 1e20], |alpha| <= 1e15) every
// operand is a normal float far from the range limits, so branch-free
// hardware approximations are used: rsqrt refined by one Newton step for the
// norm, and the fast reciprocal-multiply division (accurate to ~2 ulp; the
// IEEE-rounded versions add slow-path branches to every column step).
__device__ __forceinline__ Reflector reflector_from_float(float alpha, float sigma) {
    Reflector r;
    const float s = fmaf(alpha, alpha, sigma);
    const float y = rsqrtf(s);
    float rr = s * y;
    rr = fmaf(0.5f * y, fmaf(-rr, rr, s), rr);  // Newton step on sqrt(s)
    r.beta = signbit(alpha) ? rr : -rr;
    r.tau = __fdividef(r.beta - alpha, r.beta);
    r.scale = __fdividef(1.0f, alpha - r.beta);
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
