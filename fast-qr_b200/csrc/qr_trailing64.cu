// Rank-64 trailing update of the blocked QR on the 5th-generation tensor
// cores: C := C - V (T^T (V^T C)) with V the 64 unit-lower reflectors of two
// consecutive 32-column panels (columns k .. k+63) and C = H[k:m, k+64:n], in
// 3xTF32 split precision like the rank-32 update (qr_trailing_tc.cu).  One
// pass over C applies both panels, so the update moves half the HBM bytes of
// two rank-32 passes (the rank-32 update is HBM-bound at large n: each pass
// reads C twice and writes it once), and every MMA has twice the N.
//
// One CTA (4 warps, two CTAs per SM) owns kTN = 128 trailing columns:
//   phase A  W^T = C^T V   M=128 (c), K = rows in 32-row chunks: A = C_hi
//            straight from the TMA stage (128-byte swizzle, K-major), B =
//            [V | V_lo] (N=128), and A = C_lo (threads split it into tensor
//            memory), B = V (N=64); a 3-stage ring of 32 KB chunks
//   phase B  Y = T^T W     per thread (column c): T = D (I + S D)^-1 with the
//            64 x 64 row-major S (staged in shared memory) and tau;
//            right-looking forward substitution
//   phase C  P = V Y       M=128 (rows), N=128 (c), K=64 per 128-row chunk:
//            A = V_hi / V_lo in tensor memory (each thread stores its row),
//            B = Y_hi / Y_lo in shared memory; -P is TMA reduce-added into C
//            in 32 x 32 pieces, warp by warp
// The reference has no tensor-core path; this is the same compact-WY update
// as oracle/geqr2.c's blocked restatement with two panels per block.
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace fqr {

namespace {

constexpr int kR = 64;            // reflectors per update
constexpr int kTN = 128;          // trailing columns per CTA
constexpr int kRC = 32;           // rows per phase-A chunk (one 128-byte swizzle row)
constexpr int kStages = 3;        // phase-A ring
constexpr int kRCC = 128;         // rows per phase-C chunk (MMA M)
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;
// tensor memory, phase A: kDA = C_hi^T [V | V_lo] (128 columns), kDA2 =
// C_lo^T V (64), kALo + 32 * (chunk & 1): C_lo^T of a chunk (the A operand)
constexpr uint32_t kDA = 0;
constexpr uint32_t kDA2 = 128;
constexpr uint32_t kALo = 192;
// phase C (W is dead): V_hi / V_lo of a 128-row chunk (the A operand), P
constexpr uint32_t kVHi = 0;
constexpr uint32_t kVLo = 64;
constexpr uint32_t kDP = 128;
constexpr uint64_t kWaitLimit = 1000000000ull;  // 1 s of wall time per wait
constexpr int kFlagEarlyTrigger = 1;

// shared memory (bytes from a 1024-byte aligned base).  Phase A stage: C^T
// (128 c x 32 r, 16 KB), V (64 j x 32 r, 8 KB), V_lo (8 KB), all 128-byte
// swizzled rows; TMA brings C and V, threads write V_lo.
constexpr int kCBytes = kTN * kRC * 4;
constexpr int kVBytes = kR * kRC * 4;
constexpr int kLoadBytes = kCBytes + kVBytes;
constexpr int kStageBytes = kLoadBytes + kVBytes;  // 32 KB
constexpr int kOffTau = kStages * kStageBytes;     // tau of the 64 reflectors
constexpr int kOffBar = kOffTau + 256;             // mbarriers: full[3], mma[2], phase C; TMEM address
constexpr int kSmemUsed = kOffBar + 128;
constexpr int kSmem = kSmemUsed + 1024;  // + alignment slack: ~98 KB, two CTAs per SM
static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM");
// phase C (reuses the ring): Y_hi and Y_lo as the K-major B operand (two
// 16 KB atoms of 32 j each: [j / 32][c][32]) and two -P pieces per warp
// (32 rows x 32 columns, [c][r] as in H); phase B stages S in the -P area
constexpr int kOffYhi = 0;
constexpr int kOffYlo = 32768;
constexpr int kOffCQ = 65536;
constexpr int kCQCols = 32;
constexpr int kCQBytes = kRCC * kCQCols * 4;  // 16 KB: 4 warps x 4 KB
static_assert(kOffCQ + 2 * kCQBytes <= kOffTau, "phase-C buffers overlap tau");
static_assert(kR * kR * 4 <= 2 * kCQBytes, "S does not fit the -P area");
constexpr int kMaxSplit = 8;                        // cluster ranks per tile at most (a power of two)
constexpr int kXchgBytes = kR * kThreads * 4;       // 32 KB: one W part, any nsplit
static_assert(2 * kXchgBytes <= kOffCQ, "W exchange areas overlap S");
static_assert(kStageBytes % 1024 == 0 && kCBytes % 1024 == 0 && kVBytes % 1024 == 0, "1024-byte atoms");

constexpr uint32_t kIdescA = tc::idesc_tf32(128, 128, 0, 0);  // A = C_hi^T (smem), B = [V | V_lo]
constexpr uint32_t kIdescA2 = tc::idesc_tf32(128, 64, 0, 0);  // A = C_lo^T (TMEM), B = V
constexpr uint32_t kIdescC = tc::idesc_tf32(128, 128, 0, 0);  // A = V (TMEM, M = rows), B = Y (N = c)

// Split of one phase-A stage.  C: thread tid owns column c = tid (operand
// row tid, 128 swizzled bytes); its lo parts go to its TMEM lane (the hi
// operand is the raw stage).  V: 16-byte pieces, lo into the slot after V;
// in the first two chunks (rows 0 .. 63 of the block) V is made unit lower
// in place (H holds R and beta there).
__device__ __forceinline__ void split_stage64(unsigned char *raw, uint32_t a_lo, int chunk, int tid)
{
    {
        float lv[32];
        const unsigned char *row = raw + tid * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(row + ((q ^ (tid & 7)) << 4));
            lv[4 * q] = tc::tf32_lo(v.x);
            lv[4 * q + 1] = tc::tf32_lo(v.y);
            lv[4 * q + 2] = tc::tf32_lo(v.z);
            lv[4 * q + 3] = tc::tf32_lo(v.w);
        }
        tc::tmem_st_32x32(a_lo, lv);
    }
    const bool masked = chunk < 2;
#pragma unroll
    for (int off = kCBytes + tid * 16; off < kLoadBytes; off += kThreads * 16) {
        float4 v = *reinterpret_cast<const float4 *>(raw + off);
        if (masked) {
            // reflector j = operand row (off - kCBytes) / 128; its 16-byte
            // piece holds block rows 32 * chunk + 4 * ((piece ^ j) & 7) .. + 3
            const int vo = off - kCBytes;
            const int j = vo >> 7;
            const int r0 = kRC * chunk + 4 * ((((vo >> 4) & 7) ^ j) & 7);
            float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (r0 + q <= j) e[q] = (r0 + q == j) ? 1.0f : 0.0f;
            v = make_float4(e[0], e[1], e[2], e[3]);
            *reinterpret_cast<float4 *>(raw + off) = v;
        }
        *reinterpret_cast<float4 *>(raw + kVBytes + off) =
            make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
    }
}

// Row r0 + tid of V (64 reflectors) into registers: unit lower (rows <= j
// hold R / beta in H), zero past the matrix.  Coalesced across the warp.
__device__ __forceinline__ void load_v64(const float *Vbase, int64_t ld, int r0, int rows, int tid,
                                         float (&e)[kR])
{
    const int r = r0 + tid;
#pragma unroll
    for (int j = 0; j < kR; ++j)
        e[j] = (r < rows && r > j) ? __ldg(Vbase + (int64_t)j * ld + r) : (r == j ? 1.0f : 0.0f);
}

// ... and into this thread's TMEM lane as phase C's A operand: hi (raw;
// the tensor core truncates) at kVHi, lo at kVLo
__device__ __forceinline__ void store_v64(const float (&e)[kR], uint32_t lane_q)
{
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = e[32 * h + j];
        tc::tmem_st_32x32(lane_q + kVHi + 32u * h, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = tc::tf32_lo(e[32 * h + j]);
        tc::tmem_st_32x32(lane_q + kVLo + 32u * h, v);
    }
}

}  // namespace

template <bool SPLIT>
__global__ void __launch_bounds__(kThreads, 2)
trailing64_kernel(const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ CUtensorMap tmCQ, const float *__restrict__ H,
                  const float *__restrict__ S64, int64_t s_stride, const float *__restrict__ tau,
                  int *__restrict__ status, int ld, int n, int k, int64_t b0, int flags, int nsplit,
                  int rows_per)
{
    const bool early_trigger = flags & kFlagEarlyTrigger;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = tc::smem_addr(smem_raw);
    unsigned char *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t mat = b0 + blockIdx.y;
    const int c_begin = k + kR;
    // nsplit > 1: a cluster of nsplit CTAs (consecutive in x) shares one tile,
    // CTA `half` taking block rows [half * rows_per, (half + 1) * rows_per)
    // (rows_per a multiple of 128); their W parts are summed through
    // distributed shared memory before phase B
    const int half = SPLIT ? (int)(blockIdx.x % nsplit) : 0;
    const int c0 = c_begin + (int)(SPLIT ? blockIdx.x / nsplit : blockIdx.x) * kTN;  // first column of the tile
    const int nct = min(kTN, n - c0);
    const int m = ld - k;  // rows k .. ld-1
    const int r_begin = half * rows_per;  // this CTA's first block row
    const int mloc = SPLIT ? max(0, min(m, r_begin + rows_per) - r_begin) : m;
    const int g0 = r_begin / kRC;                             // its first 32-row chunk
    const float *Hm = H + mat * (int64_t)ld * n;
    const float *Vbase = Hm + (int64_t)k * ld + k;  // V(r, j) at Vbase[j * ld + r]
    const float *Sm = S64 + mat * s_stride;         // S(l, j) at Sm[l * 64 + j]

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kOffBar);  // [kStages]
    uint64_t *mmab = full + kStages;                                // [2]
    uint64_t *cbar = full + kStages + 2;                            // phase-C MMA
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 64);
    float *taus = reinterpret_cast<float *>(smem + kOffTau);
    const uint32_t sbase = tc::smem_addr(smem);
    const int nchunks = (mloc + kRC - 1) / kRC;  // this CTA's chunks

    if (tid == 0) {
        tc::prefetch_tensormap(&tmC);
        tc::prefetch_tensormap(&tmV);
        tc::prefetch_tensormap(&tmCQ);
        for (int i = 0; i < kStages + 3; ++i) tc::mbar_init(&full[i], 1);
        tc::fence_mbar_init();
    }
    // (every CTA that allocates tensor memory in this library holds >= 98 KB
    // of shared memory, so at most two share an SM and their 256-column
    // allocations never wait)
    if (warp == 0) {
        __syncwarp();
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    pdl_wait();  // the in-block steps (and everything before them) have completed
    if (tid == 0) {
        for (int s = 0; s < kStages && s < nchunks; ++s) {
            unsigned char *st = smem + s * kStageBytes;
            tc::mbar_expect_tx(&full[s], kLoadBytes);
            tc::tma_load_3d(st, &tmC, k + (g0 + s) * kRC, c0, (int)mat, &full[s]);
            tc::tma_load_3d(st + kCBytes, &tmV, k + (g0 + s) * kRC, k, (int)mat, &full[s]);
        }
    }
    if (tid < kR) taus[tid] = tau[mat * n + k + tid];
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_q = tmem + ((uint32_t)(32 * warp) << 16);  // this warp's TMEM lanes
    int loads = kStages < nchunks ? kStages : nchunks;
    uint32_t mma_issued[2] = {0, 0}, mma_waited[2] = {0, 0};
    bool ok = true, bad = false;

    // ---- phase A: W^T = C^T V over all rows --------------------------------
    // Every exit from the loop is uniform (at the CTA-wide __syncthreads_or).
    for (int i = 0; i < nchunks; ++i) {
        const int sidx = i % kStages, b = i & 1;
        unsigned char *st = smem + sidx * kStageBytes;
        const bool landed = tc::mbar_wait(&full[sidx], (uint32_t)(i / kStages) & 1u, kWaitLimit);
        tc::fence_after_sync();
        split_stage64(st, lane_q + kALo + 32u * b, g0 + i, tid);
        tc::tmem_st_wait();
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        ok = !__syncthreads_or(!landed || bad);
        if (!ok) break;
        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t sC = sbase + sidx * kStageBytes;
            const uint32_t sV = sC + kCBytes;
#pragma unroll
            for (int s = 0; s < kRC / 8; ++s) {
                const uint32_t ko = (uint32_t)s * 32;
                const uint64_t ac = tc::smem_desc_sw128(sC + ko);
                const uint64_t bv = tc::smem_desc_sw128(sV + ko);  // V rows, then V_lo rows
                const uint32_t acc = (i > 0 || s > 0) ? 1u : 0u;
                tc::mma_tf32(tmem + kDA, ac, bv, kIdescA, acc);
                tc::mma_tf32_ts(tmem + kDA2, tmem + kALo + 32u * b + 8u * s, bv, kIdescA2, acc);
            }
            tc::mma_commit(&mmab[b]);
        }
        ++mma_issued[b];
        if (i >= 1) {
            // chunk i-1's MMAs: afterwards its ring stage and TMEM A buffer are free
            const int pb = b ^ 1;
            const bool done = tc::mbar_wait(&mmab[pb], mma_waited[pb] & 1u, kWaitLimit);
            if (done) ++mma_waited[pb];
            const int nx = i - 1 + kStages;
            if (!done) {
                bad = true;
            } else if (tid == 0 && nx < nchunks) {
                unsigned char *fr = smem + ((i - 1) % kStages) * kStageBytes;
                uint64_t *fb = &full[(i - 1) % kStages];
                tc::mbar_expect_tx(fb, kLoadBytes);
                tc::tma_load_3d(fr, &tmC, k + (g0 + nx) * kRC, c0, (int)mat, fb);
                tc::tma_load_3d(fr + kCBytes, &tmV, k + (g0 + nx) * kRC, k, (int)mat, fb);
            }
            if (done && nx < nchunks) ++loads;
        }
    }
    ok = !__syncthreads_or(!ok || bad);
    if (ok) {
        const int lb = (nchunks - 1) & 1;
        const bool done = tc::mbar_wait(&mmab[lb], mma_waited[lb] & 1u, kWaitLimit);
        if (done) ++mma_waited[lb];
        ok = !__syncthreads_or(!done);
    }
    if (early_trigger) pdl_trigger();

    const int ncc = (mloc + kRCC - 1) / kRCC;  // this CTA's 128-row chunks
    const int nqc = (nct + kCQCols - 1) / kCQCols;
    float e[kR];  // V rows of the next phase-C chunk

    // ---- phase B: Y = T^T W, thread = tile column c ------------------------
    // W^T row c = hi*hi + hi*lo + lo*hi parts (three 64-column slices)
    float a[kR];
    auto read_w = [&]() {
        tc::fence_after_sync();
        float t[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            tc::tmem_ld_32x32(lane_q + kDA + 32u * h, t);  // hi * V_hi
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) a[32 * h + j] = t[j];
            tc::tmem_ld_32x32(lane_q + kDA + 64u + 32u * h, t);  // hi * V_lo
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) a[32 * h + j] += t[j];
            tc::tmem_ld_32x32(lane_q + kDA2 + 32u * h, t);  // lo * V_hi
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) a[32 * h + j] += t[j];
        }
    };
    if constexpr (SPLIT) {
        if (ok) read_w();
        // The cluster's W parts are summed by a reduce-scatter and an
        // all-gather over distributed shared memory: rank r owns the slice of
        // q = 64 / nsplit reflector columns [r q, r q + q).  Every rank writes
        // slice r of its part into rank r's area A (slot = source rank), each
        // rank sums its slice over the sources in rank order, then writes the
        // sum into every rank's area B (slot = owner rank).  So all ranks hold
        // bitwise the same W, and 64 KB serve any nsplit (2, 4 or 8): area A
        // and B are nsplit x q x 128 threads floats each.  Both lie in the
        // phase-A ring.  Every CTA passes all three cluster barriers, whatever
        // its `ok` (a CTA whose wait gave up has set the status word; the
        // call's results are then reported invalid).
        cg::cluster_group cl = cg::this_cluster();
        const int q = kR / nsplit;  // 32, 16 or 8 floats per slice
        float *xa = reinterpret_cast<float *>(smem);               // [src][q / 4][thread][4]
        float *xg = reinterpret_cast<float *>(smem + kXchgBytes);  // [owner][q / 4][thread][4]
        cl.sync();  // every CTA of the cluster is done with its ring
        if (ok) {
            // register indices stay compile-time constants (a[] in registers);
            // only the destination rank and offset are computed
#pragma unroll
            for (int j4 = 0; j4 < kR / 4; ++j4) {
                const int j = 4 * j4, own = j / q, jq = (j - own * q) / 4;
                *reinterpret_cast<float4 *>(cl.map_shared_rank(xa, own) + half * (q * kThreads) +
                                            (jq * kThreads + tid) * 4) = make_float4(a[j], a[j + 1], a[j + 2], a[j + 3]);
            }
        }
        cl.sync();
        if (ok) {
            for (int j4 = 0; j4 < q / 4; ++j4) {
                float4 sum = *reinterpret_cast<const float4 *>(xa + (j4 * kThreads + tid) * 4);
                for (int rk = 1; rk < nsplit; ++rk) {
                    const float4 v =
                        *reinterpret_cast<const float4 *>(xa + rk * (q * kThreads) + (j4 * kThreads + tid) * 4);
                    sum.x += v.x;
                    sum.y += v.y;
                    sum.z += v.z;
                    sum.w += v.w;
                }
                for (int rk = 0; rk < nsplit; ++rk)
                    *reinterpret_cast<float4 *>(cl.map_shared_rank(xg, rk) + half * (q * kThreads) +
                                                (j4 * kThreads + tid) * 4) = sum;
            }
        }
        cl.sync();
        if (ok) {
#pragma unroll
            for (int j4 = 0; j4 < kR / 4; ++j4) {
                // column 4 j4 lives in owner j / q's slot, at float4 (j mod q) / 4
                const int j = 4 * j4, own = j / q, jq = (j - own * q) / 4;
                const float4 v = *reinterpret_cast<const float4 *>(xg + own * (q * kThreads) + (jq * kThreads + tid) * 4);
                a[j] = v.x;
                a[j + 1] = v.y;
                a[j + 2] = v.z;
                a[j + 3] = v.w;
            }
        }
    }
    // S (16 KB) into the ring's third stage, which phase C uses only later
    // (for its -P pieces; the exchange slots are below it): all phase-A
    // copies and MMAs are complete
    float *Ss = reinterpret_cast<float *>(smem + kOffCQ);  // S(l, j) at l * 64 + j
    if (ok) {
#pragma unroll
        for (int q = 0; q < kR * kR / 4 / kThreads; ++q) {
            const int o = 4 * (tid + q * kThreads);
            *reinterpret_cast<float4 *>(Ss + o) = __ldg(reinterpret_cast<const float4 *>(Sm + o));
        }
    }
    __syncthreads();
    if (ok) {
        if constexpr (!SPLIT) read_w();
        const int c = tid;
        // y_l = tau_l a_l, then a_j -= S(l, j) y_l for j > l (S row l read
        // as float4 from the 16-byte group holding l + 1; every thread reads
        // the same address)
#pragma unroll
        for (int l = 0; l < kR; ++l) {
            a[l] *= taus[l];
#pragma unroll
            for (int j4 = (l + 1) / 4; j4 < kR / 4; ++j4) {
                const float4 s4 = *reinterpret_cast<const float4 *>(Ss + l * kR + 4 * j4);
                const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (4 * j4 + q > l) a[4 * j4 + q] = fmaf(-sv[q], a[l], a[4 * j4 + q]);
            }
        }
        // Y as the K-major B operand: column c's j in [32h, 32h + 32) at atom h,
        // row c, 16-byte piece (j % 32) / 4 at ((piece ^ c) % 8) * 16
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int jq = 0; jq < 8; ++jq) {
                const int j = 32 * h + 4 * jq;
                const float4 v = make_float4(a[j], a[j + 1], a[j + 2], a[j + 3]);
                const uint32_t off = (uint32_t)(h * 16384 + c * 128 + ((jq ^ (c & 7)) << 4));
                *reinterpret_cast<float4 *>(smem + kOffYhi + off) = v;
                *reinterpret_cast<float4 *>(smem + kOffYlo + off) =
                    make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
            }
    }
    // S is read (phase C's -P pieces overwrite it); the barrier also keeps
    // the V loads below from being hoisted into phase B's register peak
    __syncthreads();
    if (ok) {
        // V of phase-C chunk 0 into this warp's TMEM lanes (W there is read)
        load_v64(Vbase, ld, r_begin, m, tid, e);
        store_v64(e, lane_q);
        tc::tmem_st_wait();
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
    }

    // ---- phase C: C -= V Y, 128 rows per chunk -----------------------------
    // P is single-buffered: MMA(j+1) is issued once every warp has drained
    // P(j) into registers and stored V(j+1) into tensor memory; it runs while
    // the warps write P(j) out.
    uint32_t c_issued = 0, c_waited = 0;
    auto issue_c = [&]() {
        if (tid == 0) {
            tc::fence_after_sync();
#pragma unroll
            for (int s = 0; s < kR / 8; ++s) {
                // B = Y: atom s / 4, +32 bytes per 8 K elements inside it
                const uint32_t ko = (uint32_t)(s >> 2) * 16384u + (uint32_t)(s & 3) * 32u;
                const uint64_t bh = tc::smem_desc_sw128(sbase + kOffYhi + ko);
                const uint64_t bl = tc::smem_desc_sw128(sbase + kOffYlo + ko);
                tc::mma_tf32_ts(tmem + kDP, tmem + kVLo + 8u * s, bh, kIdescC, s > 0 ? 1u : 0u);
                tc::mma_tf32_ts(tmem + kDP, tmem + kVHi + 8u * s, bl, kIdescC, 1u);
                tc::mma_tf32_ts(tmem + kDP, tmem + kVHi + 8u * s, bh, kIdescC, 1u);
            }
            tc::mma_commit(cbar);
        }
        ++c_issued;
    };
    if (ok) {
        ok = !__syncthreads_or(false);  // Y and V(0) staged
        issue_c();
        if (ncc > 1) load_v64(Vbase, ld, r_begin + kRCC, m, tid, e);
    }
    for (int j = 0; j < ncc && ok; ++j) {
        const bool done = tc::mbar_wait(cbar, c_waited & 1u, kWaitLimit);
        if (done) ++c_waited;
        // stage V(j+1) (MMA(j) has read V(j)), then drain P(j): every
        // quarter this tile writes
        float pv[4][32];
        if (done) {
            tc::fence_after_sync();
            if (j + 1 < ncc) {
                store_v64(e, lane_q);
                tc::tmem_st_wait();
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (q < nqc) tc::tmem_ld_32x32(lane_q + kDP + kCQCols * q, pv[q]);
            tc::tmem_ld_wait();
        }
        tc::fence_before_sync();
        ok = !__syncthreads_or(!done);
        if (!ok) break;
        if (j + 1 < ncc) issue_c();
        // epilogue: thread = row 128 j + tid; each warp stages its 32 rows of
        // a quarter ([c][r], 4 KB) and lane 0 reduce-adds them into C (rows
        // and columns past C are outside the tensor map)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (q >= nqc) break;
            const int u = j * nqc + q;
            float *cs = reinterpret_cast<float *>(smem + kOffCQ + (u & 1) * kCQBytes) + warp * (32 * kCQCols);
            if (lane == 0) tc::bulk_wait_group_read<1>();
            __syncwarp();
#pragma unroll
            for (int c = 0; c < kCQCols; ++c) cs[c * 32 + lane] = -pv[q][c];
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::tma_reduce_add_3d(&tmCQ, k + r_begin + kRCC * j + 32 * warp, c0 + kCQCols * q, (int)mat,
                                      cs);
                tc::bulk_commit_group();
            }
        }
        if (j + 2 < ncc) load_v64(Vbase, ld, r_begin + (j + 2) * kRCC, m, tid, e);
    }
    if (!early_trigger) pdl_trigger();
    if (lane == 0) tc::bulk_wait_group<0>();  // each warp's reduces complete before shared memory goes away

    if (!ok && tid == 0) {
        atomicOr(status, 1);
        // let copies and MMA groups that did not signal in time drain
        // (bounded) before the shared and tensor memory is released
        for (int i = 0; i < loads; ++i) {
            if (i + kStages >= loads)
                tc::mbar_wait(&full[i % kStages], (uint32_t)(i / kStages) & 1u, kWaitLimit);
        }
        for (int b = 0; b < 2; ++b)
            while (mma_waited[b] < mma_issued[b])
                if (!tc::mbar_wait(&mmab[b], mma_waited[b]++ & 1u, kWaitLimit)) break;
        while (c_waited < c_issued)
            if (!tc::mbar_wait(cbar, c_waited++ & 1u, kWaitLimit)) break;
    }
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

// Static plan by (the call's batch, n, k): when all tiles of the call fit
// one CTA per SM (few large matrices, or the late blocks of a larger batch),
// each tile's rows are split over a cluster of 2, 4 or 8 CTAs: the largest
// split that still fits two CTAs per SM (296 on 148 SMs) and leaves each rank
// >= 256 rows.  That shortens the per-CTA chain of row chunks, at the cost of
// the W exchange and of phase B run in every rank.  Otherwise one CTA per
// tile.  Measured at n = 4096 (ms per call): one matrix 14.75 -> 11.96 (two
// ranks) -> 10.14 (up to eight), two 16.75 -> 13.50 -> 12.03, four 19.4 ->
// 16.05 -> 15.65; 16 matrices unchanged.  Splitting the many-tile case too (to
// keep the tiles in flight L2-resident for phase C's re-read) was slower:
// 16 matrices 26.6 -> 32.2 ms (1024-row ranks), 36.9 ms (512-row ranks).
static int trailing64_split(int64_t batch_all, int64_t tiles, int rows)
{
    if (rows < 256 || tiles * batch_all > 148) return 1;
    int ns = 2;
    while (ns < kMaxSplit && tiles * batch_all * ns * 2 <= 296 && rows >= ns * 2 * 256) ns *= 2;
    // every rank must own at least one row (rows per rank: a multiple of 128)
    while (ns > 1 && (int64_t)(ns - 1) * ((rows + ns * kRCC - 1) / (ns * kRCC) * kRCC) >= rows) ns /= 2;
    return ns;
}

cudaError_t launch_trailing64_tc(const TrailingMaps &maps, float *H, const float *S64, int64_t s_stride,
                                 const float *tau, int *status, int64_t batch, int64_t batch_all, int m, int n,
                                 int k, cudaStream_t st)
{
    if (n - k - kR <= 0) return cudaSuccess;
    if (m - k < kR) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(trailing64_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(trailing64_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    const unsigned tiles = (unsigned)((n - k - kR + kTN - 1) / kTN);
    const int rows = m - k;
    const int nsplit = trailing64_split(batch_all, tiles, rows);
    // rows per cluster rank: a multiple of the 128-row phase-C chunk
    const int rows_per = nsplit > 1 ? (rows + nsplit * kRCC - 1) / (nsplit * kRCC) * kRCC : rows;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
        const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
        e = launch_dependent(nsplit > 1 ? trailing64_kernel<true> : trailing64_kernel<false>,
                             dim3(tiles * nsplit, (unsigned)nb), dim3(kThreads), kSmem, st,
                             nsplit > 1 ? attr : nullptr, nsplit > 1 ? 1 : 0, maps.c, maps.v64, maps.cq, H, S64,
                             s_stride, tau, status, m, n, k, b0, kFlagEarlyTrigger, nsplit, rows_per);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fqr
