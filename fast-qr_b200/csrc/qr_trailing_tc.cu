// Trailing update of the blocked QR on the 5th-generation tensor cores:
//   C := C - V (T^T (V^T C))      (C = H[k:n, k+32:n], V = unit-lower panel)
// in 3xTF32 split precision (x = hi + lo; products hi*hi + hi*lo + lo*hi
// accumulate in FP32), which keeps the update at FP32 accuracy -- a plain TF32
// update fails the factor gate (the reference's own evidence,
// tests/test_qr_smoke.py:217-229; restated in tests/test_oracle.py).
//
// One CTA (4 warps, two CTAs per SM) owns a tile of kTN = 128 trailing
// columns of one matrix:
//   phase A  W^T[c][j] = sum_r C(r, c) V(r, j)    tcgen05.mma M=128 (c) N=32 (j),
//            K = rows, accumulated over 32-row chunks into TMEM; the chunks
//            stream in by cp.async through a 3-stage ring (two in flight
//            while one is split and multiplied)
//   phase B  Y = T^T W                            per thread (one column c), by
//            forward substitution with S = V^T V (strict upper) and tau:
//            T = D (I + S D)^-1, so (I + D S^T) Y = D W
//   phase C  P[r][c] = sum_j V(r, j) Y(j, c)      tcgen05.mma M=128 (r) N=128 (c)
//            K = 32 per 128-row chunk; epilogue C(r, c) -= P from TMEM
// Operands sit in shared memory in the no-swizzle K-major "core matrix"
// layout (a core holds 8 rows of the M/N dimension x 4 consecutive K
// elements, 16 bytes per row).  The raw fp32 data is the hi operand (the
// tensor core truncates it to TF32); threads write lo = x - trunc_tf32(x) into
// a second buffer.
// The reference's trailing_update_kernel (submissions/candidate.py:2507-2716)
// is SIMT FP32 with T recomputed in every CTA; nothing here follows it.
#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace fqr {

namespace {

constexpr int kTN = 128;          // trailing columns per CTA
constexpr int kRC = 32;           // rows per phase-A chunk (MMA K)
constexpr int kStages = 3;        // phase-A chunks in flight
constexpr int kRCC = 128;         // rows per phase-C chunk (MMA M)
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kDA = 0;       // TMEM column of W^T (32 columns)
constexpr uint32_t kDC = 128;     // TMEM column of P (128 columns)
constexpr uint64_t kWaitLimit = 1000000000ull;  // 1 s of wall time per wait

// shared memory map (bytes).  Phase A: a ring of kStages chunks, each C^T
// (128 c x 32 r) and V (32 j x 32 r) as raw fp32 -- the hi operand -- plus
// one lo = x - trunc_tf32(x) buffer; K-major cores of 8 rows x 4 K.
constexpr int kCQ = kRC / 4;                    // cores along K in a row of cores
constexpr int kStageBytes = (kTN + kPanel) * kRC * 4;  // 20 KB
constexpr int kOffLoC = kStages * kStageBytes;  // 60 KB
constexpr int kOffLoV = kOffLoC + kTN * kRC * 4;
constexpr int kOffT = kOffLoV + kPanel * kRC * 4;   // S, column-major 32 x 32 (4 KB)
constexpr int kOffTau = kOffT + 4096;               // tau of the panel (128 B)
constexpr int kOffBar = kOffTau + 128;              // mbarrier (8 B) + TMEM base address (4 B)
constexpr int kSmem = kOffBar + 64;                 // ~86 KB: 2 CTAs per SM
// Phase C (reuses the phase-A area): V chunk as the K-major A operand
// (128 r x 32 j) and Y as the K-major B operand (128 c x 32 j), raw + lo.
constexpr int kOffVCraw = 0;
constexpr int kOffVClo = 16384;
constexpr int kOffYraw = 32768;
constexpr int kOffYlo = 49152;
static_assert(kOffYlo + 16384 <= kOffT, "phase-C buffers overlap S");

constexpr uint32_t kIdescA = tc::idesc_tf32(128, 32, 0, 0);   // A = C^T (M = c), B = V (N = j)
constexpr uint32_t kIdescC = tc::idesc_tf32(128, 128, 0, 0);  // A = V (M = r), B = Y (N = c)

// cp.async a [NO columns] x [kRC rows] block of a column-major matrix
// (column o at base + o * ld, panel rows r0 ..) into the K-major core layout:
// core (o/8, r/4) at ((o/8) * kCQ + r/4) * 128 bytes, column o%8 at
// +16 * (o%8).  A warp step copies 8 columns x 4 row quads (64 contiguous
// bytes per column; 512 contiguous bytes of shared memory).  Rows >= rows
// and columns >= cols are zero-filled.
template <int NO>
__device__ __forceinline__ void copy_block(const float *base, int64_t ld, int r0, int rows, int cols,
                                           unsigned char *dst, int warp, int lane)
{
    constexpr int ITER = (NO / 8) * (kCQ / 4);
    const int oc = lane & 7, qi = lane >> 3;
#pragma unroll
    for (int it = warp; it < ITER; it += 4) {
        const int og = it / (kCQ / 4), qg = it % (kCQ / 4);
        const int o = og * 8 + oc;
        const int rq = qg * 4 + qi;  // row quad in the chunk
        const int r = r0 + 4 * rq;
        const bool valid = o < cols && r < rows;
        const float *src = valid ? base + (int64_t)o * ld + r : base;
        tc::cp_async16(dst + (og * kCQ + rq) * 128 + oc * 16, src, valid ? 16u : 0u);
    }
}

// lo = x - trunc_tf32(x) over `bytes` of shared memory, elementwise
__device__ __forceinline__ void make_lo(const unsigned char *raw, unsigned char *lo, int bytes, int tid)
{
#pragma unroll 4
    for (int off = tid * 16; off < bytes; off += kThreads * 16) {
        const float4 v = *reinterpret_cast<const float4 *>(raw + off);
        *reinterpret_cast<float4 *>(lo + off) =
            make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
    }
}

// V chunk as the K-major A operand of phase C (M = rows, K = the 32 panel
// columns): core (r/8, j/4) at ((r/8) * 8 + j/4) * 128 bytes, row r%8 at
// +16 * (r%8).  Thread = row: 4 column loads (coalesced across the warp) per
// 16-byte store; a warp's stores cover 4 contiguous 128-byte cores.
__device__ __forceinline__ void stage_v_kmajor(const float *Vbase, int64_t ld, int r0, int rows,
                                               unsigned char *raw, unsigned char *lo, int tid)
{
    const int r = r0 + tid;  // panel row
    float e[kPanel];
#pragma unroll
    for (int j = 0; j < kPanel; ++j)
        e[j] = (r < rows && r > j) ? __ldg(Vbase + (int64_t)j * ld + r) : (r == j ? 1.0f : 0.0f);
#pragma unroll
    for (int jq = 0; jq < kPanel / 4; ++jq) {
        const uint32_t off = (uint32_t)(((tid >> 3) * 8 + jq) * 128 + (tid & 7) * 16);
        const float4 v = make_float4(e[4 * jq], e[4 * jq + 1], e[4 * jq + 2], e[4 * jq + 3]);
        *reinterpret_cast<float4 *>(raw + off) = v;
        *reinterpret_cast<float4 *>(lo + off) =
            make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
    }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 2)
trailing_tc_kernel(float *__restrict__ H, const float *__restrict__ Sws, const float *__restrict__ tau,
                   int *__restrict__ status, int n, int k)
{
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t mat = blockIdx.y;
    const int c0 = k + kPanel + blockIdx.x * kTN;  // first trailing column of the tile
    const int nct = min(kTN, n - c0);
    const int m = n - k;
    float *Hm = H + mat * (int64_t)n * n;
    const float *Cbase = Hm + (int64_t)c0 * n + k;  // C(r, c) at Cbase[c * n + r]
    const float *Vbase = Hm + (int64_t)k * n + k;   // V(r, j) at Vbase[j * n + r]

    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 8);
    float *Ts = reinterpret_cast<float *>(smem + kOffT);    // S(l, c) at c * 32 + l
    float *taus = reinterpret_cast<float *>(smem + kOffTau);

    // phase-A prologue: the first kStages chunks start streaming at once
    const int nchunks = (m + kRC - 1) / kRC;
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
        if (s < nchunks) {
            unsigned char *st = smem + s * kStageBytes;
            copy_block<kTN>(Cbase, n, s * kRC, m, nct, st, warp, lane);
            copy_block<kPanel>(Vbase, n, s * kRC, m, kPanel, st + kTN * kRC * 4, warp, lane);
        }
        tc::cp_async_commit();
    }

    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        tc::mbar_init(bar, 1);
        tc::fence_mbar_init();
    }
    const float *Sm = Sws + mat * (kPanel * kPanel);
    for (int i = tid; i < kPanel * kPanel; i += kThreads) Ts[i] = Sm[i];
    if (tid < kPanel) taus[tid] = tau[mat * n + k + tid];
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    uint32_t phase = 0;
    bool ok = true;
    const uint32_t sbase = tc::smem_addr(smem);

    // ---- phase A: W^T = C^T V over all rows, kStages chunks in flight -----
    for (int i = 0; i < nchunks && ok; ++i) {
        const int sidx = i % kStages;
        unsigned char *st = smem + sidx * kStageBytes;
        tc::cp_async_wait_pending<kStages - 1>();  // chunk i has landed
        __syncthreads();
        if (i == 0) {
            // V is unit lower triangular: panel rows r < j are 0, row j is 1
            for (int e = tid; e < kPanel * kPanel; e += kThreads) {
                const int j = e >> 5, r = e & 31;
                if (r <= j) {
                    const int off = ((j >> 3) * kCQ + (r >> 2)) * 128 + (j & 7) * 16 + (r & 3) * 4;
                    *reinterpret_cast<float *>(st + kTN * kRC * 4 + off) = r == j ? 1.0f : 0.0f;
                }
            }
            __syncthreads();
        }
        make_lo(st, smem + kOffLoC, kTN * kRC * 4, tid);
        make_lo(st + kTN * kRC * 4, smem + kOffLoV, kPanel * kRC * 4, tid);
        tc::fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t sC = sbase + sidx * kStageBytes, sV = sC + kTN * kRC * 4;
#pragma unroll
            for (int s = 0; s < kRC / 8; ++s) {
                const uint32_t ko = (uint32_t)s * 256;  // 8 rows = 2 cores along K
                const uint64_t ah = tc::smem_desc(sC + ko, 128, kCQ * 128);
                const uint64_t al = tc::smem_desc(sbase + kOffLoC + ko, 128, kCQ * 128);
                const uint64_t bh = tc::smem_desc(sV + ko, 128, kCQ * 128);
                const uint64_t bl = tc::smem_desc(sbase + kOffLoV + ko, 128, kCQ * 128);
                const uint32_t acc = (i > 0 || s > 0) ? 1u : 0u;
                tc::mma_tf32(tmem + kDA, al, bh, kIdescA, acc);
                tc::mma_tf32(tmem + kDA, ah, bl, kIdescA, 1u);
                tc::mma_tf32(tmem + kDA, ah, bh, kIdescA, 1u);
            }
            tc::mma_commit(bar);
        }
        const bool done = tc::mbar_wait(bar, phase, kWaitLimit);
        phase ^= 1u;
        ok = !__syncthreads_or(!done);
        // this chunk's stage and the lo buffers are free again: refill
        const int nx = i + kStages;
        if (nx < nchunks) {
            copy_block<kTN>(Cbase, n, nx * kRC, m, nct, st, warp, lane);
            copy_block<kPanel>(Vbase, n, nx * kRC, m, kPanel, st + kTN * kRC * 4, warp, lane);
        }
        tc::cp_async_commit();
    }
    tc::cp_async_wait_all();

    // ---- phase B: Y = T^T W, thread = tile column c ------------------------
    if (ok) {
        tc::fence_after_sync();
        float w[32];
        tc::tmem_ld_32x32(tmem + ((uint32_t)(32 * warp) << 16) + kDA, w);
        tc::tmem_ld_wait();
        const int c = 32 * warp + lane;
        // Y = T^T W with T = D (I + S D)^-1: forward substitution
        //   y_c = tau_c (w_c - sum_{l < c} S(l, c) y_l)
        float y[32];
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
            float a = w[cc];
#pragma unroll
            for (int l = 0; l < cc; ++l) a = fmaf(-Ts[cc * 32 + l], y[l], a);
            y[cc] = taus[cc] * a;
        }
        __syncthreads();  // every thread is done with the phase-A buffers
        // Y as the K-major B operand of phase C: core (c/8, j/4) at
        // ((c/8) * 8 + j/4) * 128 bytes, column c%8 at +16 * (c%8)
#pragma unroll
        for (int jq = 0; jq < 8; ++jq) {
            const float4 v = make_float4(y[4 * jq], y[4 * jq + 1], y[4 * jq + 2], y[4 * jq + 3]);
            const uint32_t off = (uint32_t)(((c >> 3) * 8 + jq) * 128 + (c & 7) * 16);
            *reinterpret_cast<float4 *>(smem + kOffYraw + off) = v;
            *reinterpret_cast<float4 *>(smem + kOffYlo + off) =
                make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
        }
        tc::fence_before_sync();
    }

    // ---- phase C: C -= V Y, 128 rows per chunk -----------------------------
    for (int r0 = 0; r0 < m && ok; r0 += kRCC) {
        stage_v_kmajor(Vbase, n, r0, m, smem + kOffVCraw, smem + kOffVClo, tid);
        tc::fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int s = 0; s < kPanel / 8; ++s) {
                // A = V (K-major, M = rows), B = Y (K-major, N = columns):
                // 8 K-columns = 2 cores = 256 bytes per step
                const uint64_t ah = tc::smem_desc(sbase + kOffVCraw + (uint32_t)s * 256, 128, 1024);
                const uint64_t al = tc::smem_desc(sbase + kOffVClo + (uint32_t)s * 256, 128, 1024);
                const uint64_t bh = tc::smem_desc(sbase + kOffYraw + (uint32_t)s * 256, 128, 1024);
                const uint64_t bl = tc::smem_desc(sbase + kOffYlo + (uint32_t)s * 256, 128, 1024);
                tc::mma_tf32(tmem + kDC, al, bh, kIdescC, s > 0 ? 1u : 0u);
                tc::mma_tf32(tmem + kDC, ah, bl, kIdescC, 1u);
                tc::mma_tf32(tmem + kDC, ah, bh, kIdescC, 1u);
            }
            tc::mma_commit(bar);
        }
        // epilogue: thread = row r0 + 32 warp + lane.  The first 16 columns of
        // C are loaded while the MMA runs; each later group is loaded before
        // the previous one is stored.
        const int r = r0 + 32 * warp + lane;
        float *Crow = Hm + (int64_t)c0 * n + k + r;
        const bool rv = r < m;
        float cv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) cv[i] = (rv && i < nct) ? Crow[(int64_t)i * n] : 0.0f;
        const bool done = tc::mbar_wait(bar, phase, kWaitLimit);
        phase ^= 1u;
        ok = !__syncthreads_or(!done);
        if (!ok) break;
        tc::fence_after_sync();
#pragma unroll 1
        for (int cg16 = 0; cg16 < kTN / 16; ++cg16) {
            float pv[16];
            tc::tmem_ld_32x16(tmem + ((uint32_t)(32 * warp) << 16) + kDC + 16 * cg16, pv);
            tc::tmem_ld_wait();
            float nxt[16];
            const int nb = 16 * (cg16 + 1);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                nxt[i] = (rv && cg16 + 1 < kTN / 16 && nb + i < nct) ? Crow[(int64_t)(nb + i) * n] : 0.0f;
            if (rv) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = 16 * cg16 + i;
                    if (c < nct) Crow[(int64_t)c * n] = cv[i] - pv[i];
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) cv[i] = nxt[i];
        }
        tc::fence_before_sync();
        __syncthreads();
    }

    if (!ok && tid == 0) {
        atomicOr(status, 1);
        // let the MMA group that did not signal in time drain (bounded)
        // before its tensor memory is released
        tc::mbar_wait(bar, phase ^ 1u, kWaitLimit);
    }
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

bool trailing_tc_supported(int n)
{
    return n % 4 == 0 && n >= 128;
}

cudaError_t launch_trailing_tc(float *H, const float *Sws, const float *tau, int *status, int64_t batch,
                               int n, int k, cudaStream_t st)
{
    const int nc = n - k - kPanel;
    if (nc <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(trailing_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmem);
    if (e != cudaSuccess) return e;
    const unsigned tiles = (unsigned)((nc + kTN - 1) / kTN);
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
        const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
        dim3 grid(tiles, (unsigned)nb);
        trailing_tc_kernel<<<grid, kThreads, kSmem, st>>>(H + b0 * (int64_t)n * n,
                                                          Sws + b0 * kPanel * kPanel, tau + b0 * n,
                                                          status, n, k);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fqr
