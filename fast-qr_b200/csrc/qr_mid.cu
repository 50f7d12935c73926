// Mid-size batched QR (128 <= n <= 256, n % 4 == 0): the whole
// factorisation of one matrix in ONE launch, one CTA (8 warps, two CTAs per
// SM) per matrix.  The blocked chain (copy-in, then per 32-column panel a
// panel launch and a trailing-update launch) costs 16 dependent launches at
// n = 256, each waiting for the slowest matrix of the batch; here every
// matrix runs its own chain inside its CTA:
//   copy-in   A (any strides) -> H (column-major), through shared memory
//   per panel k = 0, 32, ...:
//     panel     32 columns x (n - k) rows in registers, column-owner layout
//               (below); S = V^T V and tau stay in shared memory
//     trailing  C := C - V (T^T (V^T C)) on the tensor cores, tile by tile
//               (128 trailing columns per tile), 3xTF32 as in the blocked
//               path's updates, with the C tile streamed from H by TMA (H
//               stays L2-resident: a batch of 256 matrices of 256^2 is
//               64 MiB) and -P reduce-added back by TMA
// The reference's single-launch kernels for n = 176 and 352/512
// (submissions/candidate.py:356-477, :1107-1237) are SIMT, one reflector at a
// time over the whole trailing matrix; nothing here follows them.  The
// algorithm is the blocked compact-WY restatement of oracle/geqr2.c
// (oracle_geqrf_blocked_f64) with T never formed: the panel keeps
// S = strict_upper(V^T V) and tau, and the update solves (I + D S^T) Y = D W.
//
// Panel, column-owner layout: warp w owns panel columns w, w+8, w+16, w+24
// (slot q = column w + 8q); lane l holds rows k + 32i + l of them (row block
// i; only the panel's own row blocks are held: the column loop is compiled
// once per row-block count).  Per column c, one CTA barrier:
//   * the owner of column c has published its current values (the unscaled
//     tail x and the pivot alpha) to shared memory before the barrier;
//   * every warp reads x, forms sigma = x^T x and the unscaled dots
//     d_q = x^T a_q of its own 4 columns (a reduce-scatter over the lanes and
//     a broadcast back; no cross-warp reduction), and the reflector from
//     (alpha, sigma) -- the same inputs and the same reduction order in every
//     warp, so the same bits everywhere;
//   * w_q = a_q(c) + scale * d_q (v^T a_q), the rank-1 update of its active
//     columns, S(q, c) = w_q for its finished columns q < c;
//   * the owner of column c+1 updates and publishes it first.
// Out-of-envelope columns take LAPACK order as in the blocked panel
// (common.cuh): sigma in double, then w = v^T a with the scaled v.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace fqr {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTN = 128;     // trailing columns per tile
constexpr int kRC = 32;      // rows per phase-A chunk (MMA K = 4 x 8; one 128-byte swizzle row)
constexpr int kRCC = 128;    // rows per phase-C chunk (MMA M)
constexpr int kStages = 4;   // phase-A ring
constexpr int kMaxRB = 8;    // 32-row blocks of the tallest panel (n <= 256)
constexpr uint32_t kTmemCols = 256;
constexpr uint64_t kWaitLimit = 1000000000ull;  // 1 s of wall time per wait

// tensor memory.  Phase A: kDA = C_hi^T [V | V_lo] (64 columns: hi*hi, then
// hi*lo), kDA2 = C_lo^T V (32), kALo + 32 * (chunk % 3): C_lo^T of a chunk,
// the A operand of the second product (three buffers: a chunk's split waits
// only for the MMAs of the chunk two before it).  Phase C (W is dead): P of even and
// odd 128-row chunks in turn (128 columns each), so that a chunk's MMAs run
// during the previous chunk's epilogue.
constexpr uint32_t kDA = 0;
constexpr uint32_t kDA2 = 64;
constexpr uint32_t kALo = 96;
constexpr uint32_t kDP0 = 0;
constexpr uint32_t kDP1 = 128;

// shared memory (bytes from a 1024-byte aligned base).  Phase A ring stage:
// C^T (128 c x 32 r, 16 KB), V (32 j x 32 r, 4 KB), V_lo (4 KB), 128-byte
// swizzled rows; TMA brings C and V, threads write V_lo.
constexpr int kCBytes = kTN * kRC * 4;
constexpr int kVBytes = kPanel * kRC * 4;
constexpr int kLoadBytes = kCBytes + kVBytes;
constexpr int kStageBytes = kLoadBytes + kVBytes;  // 24 KB
constexpr int kRingBytes = kStages * kStageBytes;  // 96 KB
// phase C (reuses the ring): Y_hi, Y_lo (the K-major B operand, 128 c x 32 j
// each), V_hi, V_lo of a 128-row chunk (the K-major A operand, 128 r x 32 j
// each) and one -P piece per warp (32 rows x 32 columns, [c][r], 4 KB)
constexpr int kOffYhi = 0;
constexpr int kOffYlo = 16384;
constexpr int kOffVhi = 32768;
constexpr int kOffVlo = 49152;
constexpr int kOffCQ = 65536;
constexpr int kCQCols = 32;
constexpr int kCQPiece = 32 * kCQCols * 4;  // 4 KB
// panel (reuses the ring): the published column, double-buffered
constexpr int kOffX = 0;
// copy-in (reuses the ring): two 32 x 33 float tiles per warp
constexpr int kOffCopy = 0;
constexpr int kCopyTile = 32 * 33;
// live across phases
constexpr int kOffS = kRingBytes;       // S(l, c) at l * 32 + c (4 KB)
constexpr int kOffTau = kOffS + 4096;   // tau of the panel (128 B)
constexpr int kOffBar = kOffTau + 128;  // mbarriers full[4], mma[3], phase C, test hook, copy-in; TMEM address at +96
constexpr int kSmemUsed = kOffBar + 128;
constexpr int kSmem = kSmemUsed + 1024;  // + alignment slack
static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM");
static_assert(kOffCQ + kWarps * kCQPiece <= kRingBytes, "phase-C buffers overlap S");
static_assert(kWarps * 2 * kCopyTile * 4 <= kRingBytes, "copy-in tiles overlap S");
static_assert(kStageBytes % 1024 == 0 && kCBytes % 1024 == 0, "swizzle atoms need 1024-byte alignment");
static_assert((kStages + 6) * 8 <= 96, "mbarriers overlap the TMEM address slot");

constexpr uint32_t kIdescA = tc::idesc_tf32(128, 64, 0, 0);   // A = C_hi^T (smem), B = [V | V_lo]
constexpr uint32_t kIdescA2 = tc::idesc_tf32(128, 32, 0, 0);  // A = C_lo^T (TMEM), B = V
constexpr uint32_t kIdescC = tc::idesc_tf32(128, 128, 0, 0);  // A = V (M = rows), B = Y (N = c)

// async-proxy accesses (TMA, bulk reduce) <-> generic-proxy accesses, both
// state spaces
__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// Copy-in: A (element (i, j) at Am[i * rs + j * cs]) -> H column-major, in
// 32 x 32 tiles, two per warp at a time (64 loads in flight per lane): lanes
// read 32 consecutive columns of a row (coalesced for row-major A), the
// tiles are transposed through shared memory, and lanes write 32
// consecutive rows of a column.
__device__ __forceinline__ void mid_copy_in(const float *__restrict__ Am, int64_t rs, int64_t cs,
                                            float *__restrict__ Hm, int n, float *tiles)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int nb = (n + 31) >> 5;
    for (int b0 = 2 * w; b0 < nb * nb; b0 += 2 * kWarps) {
        float v[2][32];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int b = b0 + u;
            const int r0 = (b / nb) * 32, c = (b % nb) * 32 + lane;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int r = r0 + i;
                v[u][i] = (b < nb * nb && r < n && c < n) ? __ldg(Am + r * rs + c * cs) : 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float *t = tiles + (2 * w + u) * kCopyTile;
#pragma unroll
            for (int i = 0; i < 32; ++i) t[lane * 33 + i] = v[u][i];  // t[col][row]
        }
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int b = b0 + u;
            if (b >= nb * nb) break;
            const float *t = tiles + (2 * w + u) * kCopyTile;
            const int r = (b / nb) * 32 + lane, c0 = (b % nb) * 32;
#pragma unroll 8
            for (int j = 0; j < 32; ++j)
                if (r < n && c0 + j < n) Hm[(int64_t)(c0 + j) * n + r] = t[j * 33 + lane];
        }
        __syncwarp();
    }
}

// Copy-in by TMA (row-major A, 16-byte aligned rows and matrices): 32 x 32
// tiles of A land in shared memory (128-byte swizzle: row r's 16-byte piece q
// at (q ^ (r % 8)) * 16), up to 24 per round (the whole ring); each warp
// turns its tiles into H columns, lane = tile row: eight 16-byte reads per
// lane (8 consecutive lanes hit 8 distinct bank groups), then per tile column
// one store of 32 consecutive rows.  Returns false if the wait for a round
// gave up (after a second bounded wait for its copies).
__device__ __forceinline__ bool mid_copy_in_tma(const CUtensorMap *tmA, int mat, float *__restrict__ Hm, int n,
                                                unsigned char *smem, uint64_t *bar)
{
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int nbt = (n + 31) >> 5, total = nbt * nbt;
    constexpr int kRound = kRingBytes / 4096;
    uint32_t phase = 0;
    for (int base = 0; base < total; base += kRound) {
        const int cnt = min(kRound, total - base);
        if (tid == 0) {
            tc::mbar_expect_tx(bar, (uint32_t)cnt * 4096u);
            for (int t = 0; t < cnt; ++t) {
                const int b = base + t;
                tc::tma_load_3d(smem + t * 4096, tmA, (b % nbt) * 32, (b / nbt) * 32, mat, bar);
            }
        }
        const bool landed = tc::mbar_wait(bar, phase & 1u, kWaitLimit);
        ++phase;
        if (__syncthreads_or(!landed)) {
            if (tid == 0) tc::mbar_wait(bar, (phase - 1) & 1u, kWaitLimit);
            __syncthreads();
            return false;
        }
        for (int t = w; t < cnt; t += kWarps) {
            const int b = base + t, r = (b / nbt) * 32 + lane, c0 = (b % nbt) * 32;
            const unsigned char *row = smem + t * 4096 + lane * 128;
            float v[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 f = *reinterpret_cast<const float4 *>(row + ((q ^ (lane & 7)) << 4));
                v[4 * q] = f.x;
                v[4 * q + 1] = f.y;
                v[4 * q + 2] = f.z;
                v[4 * q + 3] = f.w;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (r < n && c0 + j < n) Hm[(int64_t)(c0 + j) * n + r] = v[j];
        }
        __syncthreads();  // the tiles are read before the next round lands
    }
    return true;
}

// Reduce-scatter of 4 per-lane values over a warp: returns the warp total of
// slot lane >> 3 (two halving levels over lane bits 4, 3, then three
// butterfly levels over bits 2, 1, 0).
__device__ __forceinline__ float reduce_scatter4(const float (&d)[4], int lane)
{
    const bool b4 = lane & 16, b3 = lane & 8;
    float e[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float send = b4 ? d[t] : d[t + 2];
        const float keep = b4 ? d[t + 2] : d[t];
        e[t] = keep + __shfl_xor_sync(kFull, send, 16);
    }
    const float send = b3 ? e[0] : e[1];
    const float keep = b3 ? e[1] : e[0];
    float g = keep + __shfl_xor_sync(kFull, send, 8);
    g += __shfl_xor_sync(kFull, g, 4);
    g += __shfl_xor_sync(kFull, g, 2);
    g += __shfl_xor_sync(kFull, g, 1);
    return g;
}

// Panel factorisation of columns k .. k+wp-1 (wp = min(32, n - k)) over rows
// k .. n-1 of one matrix, column-owner layout (file comment).  NRB: the
// panel's 32-row blocks, ceil((n - k) / 32).  Leaves the factored columns in
// H, tau in global memory, and S(l, c) = v_l^T v_c (l < c; 0 elsewhere) at
// Ts[l * 32 + c] and tau at taus[] in shared memory for the trailing update.
template <int NRB>
__device__ __forceinline__ void mid_panel(float *__restrict__ Hm, float *__restrict__ tau_m, int n, int k,
                                       float *xs, float *Ts, float *taus)
{
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int nrow = n - k;            // panel rows
    const int wp = min(kPanel, nrow);  // reflectors
    constexpr int XB = kMaxRB * 32;    // floats per published-column buffer
    float P[NRB][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int j = w + 8 * q;
        const float *src = Hm + (int64_t)(k + j) * n + k + lane;
#pragma unroll
        for (int i = 0; i < NRB; ++i)
            P[i][q] = (j < wp && 32 * i + lane < nrow) ? __ldcg(src + 32 * i) : 0.0f;
    }
    for (int t = tid; t < kPanel * kPanel; t += kThreads) Ts[t] = 0.0f;
    if (tid < kPanel) taus[tid] = 0.0f;
    if (w == 0) {
#pragma unroll
        for (int i = 0; i < NRB; ++i) xs[32 * i + lane] = P[i][0];
    }
    __syncthreads();

#pragma unroll 1
    for (int c = 0; c < wp; ++c) {
        const float *xp = xs + (c & 1) * XB;
        // (1) the published column: tail x (rows > k + c) and alpha
        float x[NRB];
#pragma unroll
        for (int i = 0; i < NRB; ++i) x[i] = xp[32 * i + lane];
        const float alpha = xp[c];
        if (lane <= c) x[0] = 0.0f;
        // sigma and the unscaled dots of this warp's 4 columns (column c's own
        // slot, finished columns' slots and active ones alike)
        float s2[2] = {0.0f, 0.0f}, d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < NRB; ++i) {
            s2[i & 1] = fmaf(x[i], x[i], s2[i & 1]);
#pragma unroll
            for (int q = 0; q < 4; ++q) d[q] = fmaf(x[i], P[i][q], d[q]);
        }
        float rc[4];  // the pivot row k + c of this warp's columns
#pragma unroll
        for (int q = 0; q < 4; ++q) rc[q] = __shfl_sync(kFull, P[0][q], c);
        const float sg = warp_sum(s2[0] + s2[1]);
        const float g = reduce_scatter4(d, lane);  // slot lane >> 3, summed over the warp
        float D[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) D[q] = __shfl_sync(kFull, g, 8 * q);

        // (2) the reflector: the same (alpha, sigma) bits in every warp
        const bool fast = reflector_fast_ok(alpha, sg);
        Reflector r;
        double sd = 1.0;
        if (fast) {
            r = reflector_from_float(alpha, sg);
        } else {
            double t = 0.0;
#pragma unroll
            for (int i = 0; i < NRB; ++i) t = fma((double)x[i], (double)x[i], t);
            sd = warp_sum(t);
            r = reflector_from_double(alpha, sd);
        }
        // v over this lane's rows (0 above the pivot, 1 on it)
        float v[NRB];
        if (!r.wide) {
#pragma unroll
            for (int i = 0; i < NRB; ++i) v[i] = x[i] * r.scale;
        } else {
#pragma unroll
            for (int i = 0; i < NRB; ++i) v[i] = (float)((double)x[i] * r.scale_d);
        }
        if (lane == c) v[0] = 1.0f;
        // w_q = v^T a_q over rows >= k + c.  Fast: from the unscaled dots, when
        // none of this warp's could have over- or underflowed (|d| < 1e28 keeps
        // scale * d finite: |scale| <= 1e10 inside the envelope); else LAPACK
        // order with the scaled v (per warp: the reflector is the same either way)
        float wv[4];
        const bool dots_ok =
            fast && !__any_sync(kFull, !(fabsf(g) < 1e28f) || (g != 0.0f && fabsf(g) < kDotTiny));
        if (dots_ok) {
#pragma unroll
            for (int q = 0; q < 4; ++q) wv[q] = fmaf(r.scale, D[q], rc[q]);
        } else if (sd == 0.0) {
            // exactly zero tail: H = I, v = e_c, w = the pivot row
#pragma unroll
            for (int q = 0; q < 4; ++q) wv[q] = rc[q];
        } else {
            float d2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int i = 0; i < NRB; ++i)
#pragma unroll
                for (int q = 0; q < 4; ++q) d2[q] = fmaf(v[i], P[i][q], d2[q]);
            const float g2 = reduce_scatter4(d2, lane);
#pragma unroll
            for (int q = 0; q < 4; ++q) wv[q] = __shfl_sync(kFull, g2, 8 * q);
        }

        // (3) the owner of column c + 1 updates and publishes it first
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (w + 8 * q == c + 1 && c + 1 < wp) {
                const float tw = r.tau * wv[q];
                float *xn = xs + ((c + 1) & 1) * XB;
#pragma unroll
                for (int i = 0; i < NRB; ++i) {
                    P[i][q] = fmaf(-tw, v[i], P[i][q]);
                    xn[32 * i + lane] = P[i][q];
                }
            }
        }
        // (4) S of the finished columns, tau, the other updates
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (w + 8 * q < c) Ts[(w + 8 * q) * kPanel + c] = wv[q];
            if (w == (c & 7)) taus[c] = r.tau;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int j = w + 8 * q;
            if (j > c + 1 && j < wp) {
                const float tw = r.tau * wv[q];
#pragma unroll
                for (int i = 0; i < NRB; ++i) P[i][q] = fmaf(-tw, v[i], P[i][q]);
            } else if (j == c) {
                // column c becomes beta on the pivot row and v below it
#pragma unroll
                for (int i = 0; i < NRB; ++i) {
                    if (i > 0 || lane > c) P[i][q] = v[i];
                    else if (lane == c) P[i][q] = r.beta;
                }
            }
        }
        __syncthreads();
    }

    // store the factored columns (rows k ..) and tau
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int j = w + 8 * q;
        if (j < wp) {
            float *dst = Hm + (int64_t)(k + j) * n + k + lane;
#pragma unroll
            for (int i = 0; i < NRB; ++i)
                if (32 * i + lane < nrow) dst[32 * i] = P[i][q];
        }
    }
    if (tid < wp) tau_m[k + tid] = taus[tid];
    // the trailing update reads these columns by TMA (async proxy)
    fence_proxy_async_all();
    __syncthreads();
}

// The panel at k, compiled for its row-block count.
__device__ __forceinline__ void mid_panel_any(float *Hm, float *tau_m, int n, int k, float *xs, float *Ts,
                                              float *taus)
{
    switch ((n - k + 31) >> 5) {
    case 1: mid_panel<1>(Hm, tau_m, n, k, xs, Ts, taus); break;
    case 2: mid_panel<2>(Hm, tau_m, n, k, xs, Ts, taus); break;
    case 3: mid_panel<3>(Hm, tau_m, n, k, xs, Ts, taus); break;
    case 4: mid_panel<4>(Hm, tau_m, n, k, xs, Ts, taus); break;
    case 5: mid_panel<5>(Hm, tau_m, n, k, xs, Ts, taus); break;
    case 6: mid_panel<6>(Hm, tau_m, n, k, xs, Ts, taus); break;
    case 7: mid_panel<7>(Hm, tau_m, n, k, xs, Ts, taus); break;
    default: mid_panel<8>(Hm, tau_m, n, k, xs, Ts, taus); break;
    }
}

// Barrier use counts, the same in every thread.  The kernel reuses its
// barriers for every tile of every panel: phase-A chunks are numbered across
// the whole factorisation, chunk g going through ring stage g % kStages (its
// (g / kStages)-th use), TMEM lo buffer g % 3 and MMA barrier g % 3 (its
// (g / 3)-th use: a wait is never two phases behind, so parities cannot
// alias); phase-C MMA groups are counted the same way.
struct MidSync {
    uint32_t chunk;  // phase-A chunks issued so far (all waited for)
    uint32_t cgrp;   // phase-C MMA groups issued so far (all waited for)
};

// Split of one phase-A stage by all 256 threads.  C: thread t owns trailing
// column c = t % 128 (operand row c, 128 swizzled bytes) and chunk rows
// 16 h .. 16 h + 15, h = t / 128 (the 16-byte pieces 4 h .. 4 h + 3); their lo
// parts go to TMEM lane c, columns 16 h .. of the chunk's lo buffer (the hi
// operand is the raw stage).  V: one 16-byte piece per thread, lo into the
// slot after V; for the diagonal chunk (panel rows 0 .. 31) V is made unit
// lower in place (H holds R and beta there).
__device__ __forceinline__ void mid_split(unsigned char *st, uint32_t a_lo, bool diag, int tid)
{
    {
        const int c = tid & 127, h = tid >> 7;
        float lv[16];
        const unsigned char *row = st + c * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int q = 4 * h + u;
            const float4 v = *reinterpret_cast<const float4 *>(row + ((q ^ (c & 7)) << 4));
            lv[4 * u] = tc::tf32_lo(v.x);
            lv[4 * u + 1] = tc::tf32_lo(v.y);
            lv[4 * u + 2] = tc::tf32_lo(v.z);
            lv[4 * u + 3] = tc::tf32_lo(v.w);
        }
        tc::tmem_st_32x16(a_lo + 16u * h, lv);
    }
    const int off = kCBytes + tid * 16;  // 256 pieces of 16 bytes: all of V
    float4 v = *reinterpret_cast<const float4 *>(st + off);
    if (diag) {
        // reflector j = operand row (off - kCBytes) / 128; its 16-byte piece
        // holds panel rows 4 * ((piece ^ j) & 7) .. + 3
        const int vo = off - kCBytes;
        const int j = vo >> 7;
        const int r0 = 4 * ((((vo >> 4) & 7) ^ j) & 7);
        float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (r0 + q <= j) e[q] = (r0 + q == j) ? 1.0f : 0.0f;
        v = make_float4(e[0], e[1], e[2], e[3]);
        *reinterpret_cast<float4 *>(st + off) = v;
    }
    *reinterpret_cast<float4 *>(st + kVBytes + off) =
        make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
}

// Reflectors 16 h .. 16 h + 15 of row r0 + (tid % 128) of the panel's V, into
// registers: unit lower, zero past the matrix; loads bypass L1 (H was
// written in this launch).
__device__ __forceinline__ void mid_load_v(const float *Vbase, int ld, int r0, int rows, int tid, float (&e)[16])
{
    const int r = r0 + (tid & 127), h = tid >> 7;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        const int j = 16 * h + u;
        e[u] = (r < rows && r > j) ? __ldcg(Vbase + (int64_t)j * ld + r) : (r == j ? 1.0f : 0.0f);
    }
}

// ... and into phase C's K-major A operand (M = rows, K = the 32 reflectors)
// in the 128-byte swizzle layout: row r's 128 bytes at r * 128, its 16-byte
// piece jq (reflectors 4 jq .. 4 jq + 3) at (jq ^ (r % 8)) * 16
__device__ __forceinline__ void mid_store_v(const float (&e)[16], unsigned char *hi, unsigned char *lo, int tid)
{
    const int r = tid & 127, h = tid >> 7;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int jq = 4 * h + u;
        const uint32_t off = (uint32_t)(r * 128 + ((jq ^ (r & 7)) << 4));
        const float4 v = make_float4(e[4 * u], e[4 * u + 1], e[4 * u + 2], e[4 * u + 3]);
        *reinterpret_cast<float4 *>(hi + off) = v;
        *reinterpret_cast<float4 *>(lo + off) =
            make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
    }
}

// The trailing update of panel k: C := C - V (T^T (V^T C)) for C = H[k:n,
// k+32:n], 128 columns per tile, tiles in turn:
//   A  W^T = C^T V over 32-row chunks through a 4-stage TMA ring: A = C_hi
//      straight from the stage against B = [V | V_lo] (N = 64), and A = C_lo
//      (split by the threads into TMEM) against B = V (N = 32), as in the
//      rank-64 update (qr_trailing64.cu)
//   B  Y = T^T W per thread of the first warpgroup (tile column c):
//      y_l = tau_l (w_l - sum_{i<l} S(i, l) y_i), Y hi / lo to shared memory
//      as the K-major B operand
//   C  P = V Y per 128-row chunk (A = V hi / lo staged in shared memory,
//      M = 128 rows, N = 128 columns) into two TMEM accumulators in turn;
//      each warp stages -P in 32 x 32 pieces (the two warpgroups take two
//      column quarters each) that TMA reduce-adds into H, as in the rank-32
//      update (qr_trailing_tc.cu)
// Returns false if a bounded wait gave up (after letting the copies and MMAs
// in flight drain); every exit is CTA-uniform.  force_timeout (a test hook):
// the first wait of the call is made on a barrier that nothing completes,
// with a short limit, so the failure path runs without any fault.
__device__ __forceinline__ bool mid_trailing(const CUtensorMap *tmC, const CUtensorMap *tmV,
                                             const CUtensorMap *tmCQ, const float *Hm, int mat, int n, int k,
                                             unsigned char *smem, uint32_t tmem, MidSync &sy, bool force_timeout)
{
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, half = tid >> 7;
    const uint32_t sbase = tc::smem_addr(smem);
    const uint32_t lane_q = tmem + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's TMEM lanes
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kOffBar);  // [kStages]
    uint64_t *mmab = full + kStages;                                // [3]
    uint64_t *cbar = full + kStages + 3;                            // phase C
    uint64_t *never = full + kStages + 4;                           // the test hook's barrier
    const float *Ts = reinterpret_cast<const float *>(smem + kOffS);
    const float *taus = reinterpret_cast<const float *>(smem + kOffTau);
    float *piece = reinterpret_cast<float *>(smem + kOffCQ + warp * kCQPiece);  // this warp's -P piece
    const int m = n - k;
    const int nchunks = (m + kRC - 1) / kRC;
    const int ncc = (m + kRCC - 1) / kRCC;
    const float *Vbase = Hm + (int64_t)k * n + k;  // V(r, j) at Vbase[j * n + r]
    bool ok = true;

    for (int c0 = k + kPanel; c0 < n && ok; c0 += kTN) {
        const int nct = min(kTN, n - c0);
        const int nqc = (nct + kCQCols - 1) / kCQCols;
        const uint32_t g0 = sy.chunk;  // global number of this tile's chunk 0
        if (tid == 0) {
            for (int s = 0; s < kStages && s < nchunks; ++s) {
                const uint32_t si = (g0 + s) % kStages;
                unsigned char *st = smem + si * kStageBytes;
                tc::mbar_expect_tx(&full[si], kLoadBytes);
                tc::tma_load_3d(st, tmC, k + s * kRC, c0, mat, &full[si]);
                tc::tma_load_3d(st + kCBytes, tmV, k + s * kRC, k, mat, &full[si]);
            }
        }
        // progress of this tile (the same in every thread), for the drain
        // after a wait that gave up
        int loads = kStages < nchunks ? kStages : nchunks;  // chunks whose copies were issued
        int landed_n = 0;                                   // ... whose arrival was waited for
        int mma_n = 0, mma_done = 0;                        // chunks whose MMAs were issued / waited for
        int cg_n = 0, cg_done = 0;                          // phase-C groups issued / waited for
        bool bad = false;

        // ---- phase A --------------------------------------------------------
        for (int i = 0; i < nchunks; ++i) {
            const uint32_t g = g0 + i, si = g % kStages;
            unsigned char *st = smem + si * kStageBytes;
            bool landed;
            if (force_timeout && i == 0)
                landed = tc::mbar_wait(never, 0u, 2000000ull);  // 2 ms; nothing arrives
            else
                landed = tc::mbar_wait(&full[si], (g / kStages) & 1u, kWaitLimit);
            if (landed) ++landed_n;
            // run by every thread (the TMEM stores are warp-collective); after a
            // wait that gave up it moves garbage that no MMA reads
            tc::fence_after_sync();
            const uint32_t lo = kALo + 32u * (g % 3u);
            mid_split(st, lane_q + lo, i == 0, tid);
            tc::tmem_st_wait();
            tc::fence_proxy_async_smem();
            tc::fence_before_sync();
            ok = !__syncthreads_or(!landed || bad);
            if (!ok) break;
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t sC = sbase + si * kStageBytes;
                const uint32_t sV = sC + kCBytes;
#pragma unroll
                for (int s = 0; s < kRC / 8; ++s) {
                    const uint32_t ko = (uint32_t)s * 32;
                    const uint64_t ac = tc::smem_desc_sw128(sC + ko);
                    const uint64_t bv = tc::smem_desc_sw128(sV + ko);  // V rows, then V_lo rows
                    const uint32_t acc = (i > 0 || s > 0) ? 1u : 0u;
                    tc::mma_tf32(tmem + kDA, ac, bv, kIdescA, acc);
                    tc::mma_tf32_ts(tmem + kDA2, tmem + lo + 8u * s, bv, kIdescA2, acc);
                }
                tc::mma_commit(&mmab[g % 3]);
            }
            ++mma_n;
            if (i >= 2) {
                // chunk i-2's MMAs: afterwards its stage and TMEM lo buffer are
                // free (chunk i-1's may still run)
                const uint32_t gp = g - 2;
                const bool done = tc::mbar_wait(&mmab[gp % 3], (gp / 3) & 1u, kWaitLimit);
                if (done) ++mma_done;
                const int nx = i - 2 + kStages;
                if (!done) {
                    bad = true;  // made uniform by the next __syncthreads_or
                } else if (tid == 0 && nx < nchunks) {
                    const uint32_t fs = gp % kStages;  // = (g0 + nx) % kStages
                    unsigned char *fr = smem + fs * kStageBytes;
                    tc::mbar_expect_tx(&full[fs], kLoadBytes);
                    tc::tma_load_3d(fr, tmC, k + nx * kRC, c0, mat, &full[fs]);
                    tc::tma_load_3d(fr + kCBytes, tmV, k + nx * kRC, k, mat, &full[fs]);
                }
                if (done && nx < nchunks) ++loads;
            }
        }
        ok = !__syncthreads_or(!ok || bad);
        if (ok) {
            // the last two chunks' MMAs
            bool done = true;
            for (int i = nchunks >= 2 ? nchunks - 2 : 0; i < nchunks && done; ++i) {
                const uint32_t gl = g0 + i;
                done = tc::mbar_wait(&mmab[gl % 3], (gl / 3) & 1u, kWaitLimit);
                if (done) ++mma_done;
            }
            ok = !__syncthreads_or(!done);
        }
        sy.chunk = g0 + nchunks;

        // ---- phase B: Y = T^T W, thread = tile column c ----------------------
        // (both warpgroups first start loading their halves of V(0))
        float e[16];
        if (ok) mid_load_v(Vbase, n, 0, m, tid, e);
        if (ok && half == 0) {
            tc::fence_after_sync();
            float a[32], t[32];
            tc::tmem_ld_32x32(lane_q + kDA, a);  // hi * V_hi
            tc::tmem_ld_wait();
            tc::tmem_ld_32x32(lane_q + kDA + 32u, t);  // hi * V_lo
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] += t[j];
            tc::tmem_ld_32x32(lane_q + kDA2, t);  // lo * V_hi
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] += t[j];
            // y_l = tau_l (w_l - sum_{i<l} S(i, l) y_i), right-looking: once y_l
            // is known it is subtracted from every later a_j (row l of S read
            // four entries at a time; every thread reads the same address), so
            // the dependency chain is one multiply and one FMA per reflector
#pragma unroll
            for (int l = 0; l < kPanel; ++l) {
                a[l] *= taus[l];
#pragma unroll
                for (int j4 = (l + 1) / 4; j4 < kPanel / 4; ++j4) {
                    const float4 s4 = *reinterpret_cast<const float4 *>(Ts + l * kPanel + 4 * j4);
                    const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (4 * j4 + u > l) a[4 * j4 + u] = fmaf(-sv[u], a[l], a[4 * j4 + u]);
                }
            }
            // Y as the K-major B operand: column c's 32 values at c * 128,
            // 16-byte piece jq at (jq ^ (c % 8)) * 16
            const int c = tid;
#pragma unroll
            for (int jq = 0; jq < 8; ++jq) {
                const float4 v = make_float4(a[4 * jq], a[4 * jq + 1], a[4 * jq + 2], a[4 * jq + 3]);
                const uint32_t off = (uint32_t)(c * 128 + ((jq ^ (c & 7)) << 4));
                *reinterpret_cast<float4 *>(smem + kOffYhi + off) = v;
                *reinterpret_cast<float4 *>(smem + kOffYlo + off) =
                    make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
            }
        }
        if (ok) {
            mid_store_v(e, smem + kOffVhi, smem + kOffVlo, tid);
            tc::fence_proxy_async_smem();
        }
        tc::fence_before_sync();

        // ---- phase C: C -= V Y, 128 rows per chunk -------------------------
        // MMA(j) writes P[j % 2]; it is issued once MMA(j-1) has completed (it
        // read the V buffer) and V(j) is staged, so it runs during the
        // epilogue of chunk j-1.  V rows are loaded one chunk ahead.
        auto issue_c = [&](int j) {
            if (tid == 0) {
                tc::fence_after_sync();
                const uint32_t d = tmem + ((j & 1) ? kDP1 : kDP0);
#pragma unroll
                for (int s = 0; s < kPanel / 8; ++s) {
                    // A = V (M = rows), B = Y (N = columns), both K-major and
                    // 128-byte swizzled: 8 K elements = +32 bytes per step
                    const uint32_t ko = (uint32_t)s * 32u;
                    const uint64_t ah = tc::smem_desc_sw128(sbase + kOffVhi + ko);
                    const uint64_t al = tc::smem_desc_sw128(sbase + kOffVlo + ko);
                    const uint64_t bh = tc::smem_desc_sw128(sbase + kOffYhi + ko);
                    const uint64_t bl = tc::smem_desc_sw128(sbase + kOffYlo + ko);
                    tc::mma_tf32(d, al, bh, kIdescC, s > 0 ? 1u : 0u);
                    tc::mma_tf32(d, ah, bl, kIdescC, 1u);
                    tc::mma_tf32(d, ah, bh, kIdescC, 1u);
                }
                tc::mma_commit(cbar);
            }
            ++cg_n;
        };
        if (ok) {
            ok = !__syncthreads_or(false);  // Y and V(0) staged
            issue_c(0);
            if (ncc > 1) mid_load_v(Vbase, n, kRCC, m, tid, e);
        }
        for (int j = 0; j < ncc && ok; ++j) {
            const bool done = tc::mbar_wait(cbar, (sy.cgrp + (uint32_t)cg_done) & 1u, kWaitLimit);
            if (done) ++cg_done;
            if (done && j + 1 < ncc) {
                mid_store_v(e, smem + kOffVhi, smem + kOffVlo, tid);  // MMA(j) has read V(j)
                tc::fence_proxy_async_smem();
            }
            tc::fence_before_sync();
            ok = !__syncthreads_or(!done);
            if (!ok) break;
            if (j + 1 < ncc) issue_c(j + 1);
            if (j + 2 < ncc) mid_load_v(Vbase, n, (j + 2) * kRCC, m, tid, e);
            tc::fence_after_sync();
            const uint32_t pc = lane_q + ((j & 1) ? kDP1 : kDP0);
            // epilogue: thread = row 128 j + tid % 128; warpgroup h takes
            // column quarters 2h and 2h + 1; each warp stages its 32 rows of a
            // quarter ([c][r], 4 KB) and lane 0 reduce-adds them into C (rows
            // and columns past the matrix are outside the tensor map)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int q = 2 * half + u;
                if (q >= nqc) break;
                float pv[32];
                tc::tmem_ld_32x32(pc + kCQCols * q, pv);
                tc::tmem_ld_wait();
                // the warp's previous reduce has read its piece
                if (lane == 0) tc::bulk_wait_group_read<0>();
                __syncwarp();
#pragma unroll
                for (int cc = 0; cc < kCQCols; ++cc) piece[cc * 32 + lane] = -pv[cc];
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::tma_reduce_add_3d(tmCQ, k + kRCC * j + 32 * (warp & 3), c0 + kCQCols * q, mat, piece);
                    tc::bulk_commit_group();
                }
            }
            tc::fence_before_sync();
        }
        sy.cgrp += (uint32_t)cg_done;
        // the staged -P pieces are read before the next tile's copies land
        // in the ring
        if (lane == 0) tc::bulk_wait_group_read<0>();
        __syncthreads();

        if (!ok && tid == 0) {
            // let copies and MMA groups that did not signal in time drain
            // (bounded) before the shared and tensor memory is released
            for (int i = landed_n; i < loads; ++i) {
                const uint32_t g = g0 + i;
                tc::mbar_wait(&full[g % kStages], (g / kStages) & 1u, kWaitLimit);
            }
            for (int i = mma_done; i < mma_n; ++i) {
                const uint32_t g = g0 + i;
                if (!tc::mbar_wait(&mmab[g % 3], (g / 3) & 1u, kWaitLimit)) break;
            }
            for (int u = cg_done; u < cg_n; ++u)
                if (!tc::mbar_wait(cbar, (sy.cgrp + (uint32_t)(u - cg_done)) & 1u, kWaitLimit)) break;
        }
    }
    // the reduce-adds are complete and visible before the next panel reads H
    if (lane == 0) tc::bulk_wait_group<0>();
    fence_proxy_async_all();
    __syncthreads();
    return ok;
}

}  // namespace

// One CTA per matrix: copy-in, then per 32-column panel the panel and the
// trailing update, all in this launch.
__global__ void __launch_bounds__(kThreads, 2)
mid_kernel(const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmV,
           const __grid_constant__ CUtensorMap tmCQ, const __grid_constant__ CUtensorMap tmA,
           const float *__restrict__ A, int64_t a_bs, int64_t a_rs,
           int64_t a_cs, float *__restrict__ H, float *__restrict__ tau, int *__restrict__ status, int n,
           int flags)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = tc::smem_addr(smem_raw);
    unsigned char *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int64_t mat = blockIdx.x;
    float *Hm = H + mat * (int64_t)n * n;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);  // full[4], mma[3], phase C, test hook, copy-in
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 96);
    const bool tma_copy = flags & kMidFlagTmaCopy;
    if (tid == 0) {
        tc::prefetch_tensormap(&tmC);
        tc::prefetch_tensormap(&tmV);
        tc::prefetch_tensormap(&tmCQ);
        if (tma_copy) tc::prefetch_tensormap(&tmA);
        for (int i = 0; i < kStages + 6; ++i) tc::mbar_init(&bars[i], 1);
        tc::fence_mbar_init();
    }
    __syncthreads();  // the barriers are initialised before the copy-in waits on one
    // (every CTA that allocates tensor memory in this library holds >= 98 KB
    // of shared memory, so at most two share an SM and their 256-column
    // allocations never wait)
    if (warp == 0) {
        __syncwarp();
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    bool ok = true;
    if (tma_copy)
        ok = mid_copy_in_tma(&tmA, (int)mat, Hm, n, smem, &bars[kStages + 5]);
    else
        mid_copy_in(A + mat * a_bs, a_rs, a_cs, Hm, n, reinterpret_cast<float *>(smem + kOffCopy));
    fence_proxy_async_all();  // H is read by TMA in the first trailing update
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    float *xs = reinterpret_cast<float *>(smem + kOffX);
    float *Ts = reinterpret_cast<float *>(smem + kOffS);
    float *taus = reinterpret_cast<float *>(smem + kOffTau);
    MidSync sy = {0u, 0u};
    for (int k = 0; k < n && ok; k += kPanel) {
        mid_panel_any(Hm, tau + mat * n, n, k, xs, Ts, taus);
        if (k + kPanel < n)
            ok = mid_trailing(&tmC, &tmV, &tmCQ, Hm, (int)mat, n, k, smem, tmem, sy,
                              (flags & kMidFlagForceTimeout) && k == 0);
    }
    if (!ok && tid == 0) atomicOr(status, 1);
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

bool mid_supported(int64_t m, int64_t n, const void *H)
{
    return m == n && n % 4 == 0 && n >= 128 && n <= kMidMaxN && ((uintptr_t)H % 16) == 0;
}

cudaError_t launch_mid(const float *A, int64_t batch, int n, int64_t bs, int64_t rs, int64_t cs, float *H,
                       float *tau, int *status, int status_words, int flags, cudaStream_t st)
{
    static_assert(kMidMaxN <= 32 * kMaxRB, "the panel holds at most kMaxRB row blocks");
    if (!mid_supported(n, n, H) || batch > 0x7fffffff) return cudaErrorInvalidValue;
    TrailingMaps maps;
    cudaError_t e = prepare_trailing_tc(H, batch, n, n, &maps);
    if (e != cudaSuccess) return e;
    // A by TMA tiles when its rows and matrices are 16-byte aligned
    // (row-major, contiguous columns); any other layout by plain loads
    CUtensorMap tmA = maps.c;  // (unused unless the flag is set)
    const bool tma_copy = cs == 1 && ((uintptr_t)A % 16) == 0 && rs % 4 == 0 && rs >= n &&
                          (batch == 1 || (bs % 4 == 0 && bs >= (int64_t)n * rs));
    if (tma_copy) {
        e = encode_rowmajor_tiles(A, batch, n, n, bs, rs, &tmA);
        if (e != cudaSuccess) return e;
        flags |= kMidFlagTmaCopy;
    }
    e = cudaFuncSetAttribute(mid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    // the status words of this call start clear (the kernel only sets them)
    e = cudaMemsetAsync(status, 0, (size_t)status_words * sizeof(int), st);
    if (e != cudaSuccess) return e;
    mid_kernel<<<dim3((unsigned)batch), dim3(kThreads), kSmem, st>>>(maps.c, maps.v, maps.cq, tmA, A, bs, rs, cs,
                                                                     H, tau, status, n, flags);
    return cudaGetLastError();
}

}  // namespace fqr
