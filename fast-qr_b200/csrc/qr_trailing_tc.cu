// Trailing update of the blocked QR on the 5th-generation tensor cores:
//   C := C - V (T^T (V^T C))      (C = H[k:n, k+32:n], V = unit-lower panel)
// in 3xTF32 split precision (x = hi + lo; products hi*hi + hi*lo + lo*hi
// accumulate in FP32), which keeps the update at FP32 accuracy -- a plain TF32
// update fails the factor gate (the reference's own evidence,
// tests/test_qr_smoke.py:217-229; restated in tests/test_oracle.py).
//
// One CTA (4 warps, two CTAs per SM) owns a tile of kTN = 128 trailing
// columns of one matrix:
//   phase A  W^T[c][j] = sum_r C(r, c) V(r, j)    tcgen05.mma M=128 (c), K = rows,
//            accumulated over 32-row chunks into TMEM: C_hi against
//            [V_hi | V_lo] (N=64) and C_lo against V_hi (N=32).  Thread 0
//            streams the chunks by TMA (tensor maps over H, 128-byte
//            swizzle: each column's 32 rows are one 128-byte operand row)
//            through a 4-stage ring; while the MMAs of chunk i-1 run, every
//            thread loads its column of chunk i from the stage and stores hi
//            and lo into tensor memory, where the MMAs read their A operand
//            (only V, the B operand, is read from shared memory).
//   phase B  Y = T^T W                            per thread (one column c), by
//            forward substitution with S = V^T V (strict upper) and tau:
//            T = D (I + S D)^-1, so (I + D S^T) Y = D W
//   phase C  P[r][c] = sum_j V(r, j) Y(j, c)      tcgen05.mma M=128 (r) N=128 (c)
//            K = 32 per 128-row chunk, into two TMEM accumulators in turn so
//            that the next chunk's MMA runs during this chunk's epilogue;
//            the epilogue writes -P in 32-column quarters to shared memory
//            and TMA reduce-adds them into C
// The raw fp32 data is the hi operand (the tensor core truncates it to TF32);
// threads write lo = x - trunc_tf32(x) into a second buffer of the same
// layout.  Phase C's V and Y operands are staged by threads in the
// 128-byte swizzle K-major layout as well.
// The reference's trailing_update_kernel (submissions/candidate.py:2507-2716)
// is SIMT FP32 with T recomputed in every CTA; nothing here follows it.
#include <cooperative_groups.h>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace fqr {

namespace {

constexpr int kTN = 128;          // trailing columns per CTA
constexpr int kRC = 32;           // rows per phase-A chunk (MMA K; one 128-byte swizzle row)
constexpr int kStages = 4;        // phase-A ring of raw chunks (fills phase C's 96 KB area)
constexpr int kRCC = 128;         // rows per phase-C chunk (MMA M)
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;
// phase A accumulates W^T in three parts: kDA holds C_hi^T [V_hi | V_lo]
// (64 columns: the hi*hi then the hi*lo products), kDA2 holds C_lo^T V_hi.
// Its A operands (C_hi^T and C_lo^T of a 32-row chunk: 128 lanes x 32
// columns each) sit in tensor memory too, double-buffered by chunk parity.
constexpr uint32_t kDA = 0;
constexpr uint32_t kDA2 = 64;
constexpr uint32_t kAHi = 96;   // + 64 * (chunk & 1)
constexpr uint32_t kALo = 128;  // + 64 * (chunk & 1)
constexpr uint32_t kDP0 = 0;      // P of even phase-C chunks (128 columns; W is dead by then)
constexpr uint32_t kDP1 = 128;    // P of odd phase-C chunks
constexpr uint64_t kWaitLimit = 1000000000ull;  // 1 s of wall time per wait
// kernel flags: trigger the next kernel's launch at the start of phase C
// (else after it)
constexpr int kFlagEarlyTrigger = 1;
// test hook (fqr_debug_force_timeout): the first phase-A wait of every CTA is
// made on a barrier that nothing completes, with a 2 ms limit, so that the
// failure path (drain, status word) runs without any fault
constexpr int kFlagForceTimeout = 2;

// shared memory map (bytes, from a 1024-byte aligned base).  Phase A: a ring
// of kStages chunks, each C^T (128 c x 32 r, 16 KB), V (32 j x 32 r, 4 KB)
// as raw fp32 in the 128-byte swizzle layout, then V's lo part (4 KB) right
// after V, so that [V | V_lo] is one N = 64 operand.  C's hi and lo parts go
// from the stage through registers into tensor memory (the MMAs' A
// operand), so shared memory carries C once by TMA and once to registers:
// phase A is bound by shared-memory bandwidth.
constexpr int kCBytes = kTN * kRC * 4;                   // 16 KB
constexpr int kVBytes = kPanel * kRC * 4;                // 4 KB
constexpr int kLoadBytes = kCBytes + kVBytes;            // 20 KB arrive by TMA per chunk
constexpr int kStageBytes = kLoadBytes + kVBytes;        // 24 KB
constexpr int kOffT = 96 * 1024;                         // S, column-major 32 x 32 (4 KB), after phase C's area
constexpr int kOffTau = kOffT + 4096;                    // tau of the panel (128 B)
constexpr int kOffBar = kOffTau + 128;  // mbarriers: full[4], mma[2], phase C, test hook; TMEM address at +64
constexpr int kSmemUsed = kOffBar + 128;
constexpr int kSmem = kSmemUsed + 1024;                  // + alignment slack: ~109 KB, 2 CTAs per SM
static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM");
static_assert((kStages + 4) * 8 <= 64, "mbarriers overlap the TMEM address slot");
// Phase C (reuses the phase-A area): V chunk as the K-major A operand
// (128 r x 32 j) and Y as the K-major B operand (128 c x 32 j), raw + lo, and
// two -P quarters (128 rows x 32 columns; each warp's 32 rows a 4 KB slice,
// [c][r] as they sit in H) that TMA reduce-adds into C, warp by warp.
constexpr int kOffVCraw = 0;
constexpr int kOffVClo = 16384;
constexpr int kOffYraw = 32768;
constexpr int kOffYlo = 49152;
constexpr int kOffCQ = 65536;
constexpr int kCQCols = 32;
constexpr int kCQBytes = kRCC * kCQCols * 4;  // 16 KB
static_assert(kOffCQ + 2 * kCQBytes <= kOffT, "phase-C buffers overlap S");
constexpr int kMaxSplit = 8;                     // cluster ranks per tile at most (a power of two)
constexpr int kXchgBytes = kPanel * kThreads * 4;  // 16 KB: one W part, any split
static_assert(kOffCQ + 2 * kXchgBytes <= kOffT, "W exchange areas overlap S");
static_assert(2 * 32 * kThreads * 4 <= 2 * kCQBytes, "two W exchange slots exceed the -P area");
static_assert(kStages * kStageBytes <= kOffT, "phase-A ring overlaps S");
static_assert(kStageBytes % 1024 == 0 && kCBytes % 1024 == 0, "swizzle atoms need 1024-byte alignment");

constexpr uint32_t kIdescA = tc::idesc_tf32(128, 64, 0, 0);   // A = C^T (M = c), B = [V | V_lo] (N = 2 x j)
constexpr uint32_t kIdescA2 = tc::idesc_tf32(128, 32, 0, 0);  // A = C_lo^T, B = V
constexpr uint32_t kIdescC = tc::idesc_tf32(128, 128, 0, 0);  // A = V (M = r), B = Y (N = c)

// The split of one stage (lo = x - trunc_tf32(x)).  C: thread tid owns
// trailing column c = tid of the tile, i.e. A row tid, whose 32 rows are one
// 128-byte swizzled row of the stage (16-byte piece q at (q ^ (c & 7)) * 16);
// it loads them once and stores hi and lo into its TMEM lane (a_hi / a_lo are
// the warp's lane-quarter addresses).  V: elementwise into the slot after V;
// for the first chunk V is also made unit lower triangular in place (panel
// rows r < j hold R, row j holds beta).  Every thread of a warp runs the
// tensor-memory stores (they are warp-collective).
__device__ __forceinline__ void split_stage(unsigned char *raw, uint32_t a_hi, uint32_t a_lo, bool first,
                                            int tid)
{
    {
        float hv[32], lv[32];
        const unsigned char *row = raw + tid * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(row + ((q ^ (tid & 7)) << 4));
            hv[4 * q] = v.x;
            hv[4 * q + 1] = v.y;
            hv[4 * q + 2] = v.z;
            hv[4 * q + 3] = v.w;
            lv[4 * q] = tc::tf32_lo(v.x);
            lv[4 * q + 1] = tc::tf32_lo(v.y);
            lv[4 * q + 2] = tc::tf32_lo(v.z);
            lv[4 * q + 3] = tc::tf32_lo(v.w);
        }
        tc::tmem_st_32x32(a_hi, hv);
        tc::tmem_st_32x32(a_lo, lv);
    }
#pragma unroll
    for (int off = kCBytes + tid * 16; off < kLoadBytes; off += kThreads * 16) {
        float4 v = *reinterpret_cast<const float4 *>(raw + off);
        if (first) {
            // V row j (= operand row) at (off - kCBytes) / 128; its 16-byte
            // chunk holds panel rows 4 * ((chunk ^ j) & 7) .. + 3
            const int vo = off - kCBytes;
            const int j = vo >> 7;
            const int r0 = 4 * ((((vo >> 4) & 7) ^ j) & 7);
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

// V rows r0 + tid of a phase-C chunk, one per thread, into registers (32
// loads, coalesced across the warp); panel rows r <= j get the unit lower
// triangle (H holds R and beta there), rows past the matrix get 0.
__device__ __forceinline__ void load_v_rows(const float *Vbase, int64_t ld, int r0, int rows, int wv, int tid,
                                            float (&e)[kPanel])
{
    const int r = r0 + tid;  // panel row
#pragma unroll
    for (int j = 0; j < kPanel; ++j)
        e[j] = (j < wv && r < rows && r > j) ? __ldg(Vbase + (int64_t)j * ld + r) : (r == j ? 1.0f : 0.0f);
}
// ... then as the K-major A operand of phase C (M = rows, K = the 32 panel
// columns) in the 128-byte swizzle layout: row r's 128 bytes at r * 128,
// its 16-byte piece q (columns 4q .. 4q+3) at (q ^ (r % 8)) * 16, so eight
// consecutive threads store to eight distinct bank groups.  (The tensor core
// reads this layout at 78 cycles per M=128, N<=128, K=8 tf32 MMA, against
// 120 for the no-swizzle core-matrix layout, measured on B200.)
__device__ __forceinline__ void store_v_rows(const float (&e)[kPanel], unsigned char *raw, unsigned char *lo,
                                             int tid)
{
#pragma unroll
    for (int jq = 0; jq < kPanel / 4; ++jq) {
        const uint32_t off = (uint32_t)(tid * 128 + ((jq ^ (tid & 7)) << 4));
        const float4 v = make_float4(e[4 * jq], e[4 * jq + 1], e[4 * jq + 2], e[4 * jq + 3]);
        *reinterpret_cast<float4 *>(raw + off) = v;
        *reinterpret_cast<float4 *>(lo + off) =
            make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
    }
}

}  // namespace

template <bool ApplyT, bool SPLIT = false>
__global__ void __launch_bounds__(kThreads, 2)
trailing_tc_kernel(const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmCQ, const float *__restrict__ H,
                   const float *__restrict__ Sws, int64_t s_stride, const float *__restrict__ tau,
                   int *__restrict__ status, int ld, int hcols, int k, int c_begin, int c_end, int64_t b0,
                   int flags, int nsplit, int rows_per)
{
    const bool early_trigger = flags & kFlagEarlyTrigger;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = tc::smem_addr(smem_raw);
    unsigned char *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t mat = b0 + blockIdx.y;
    // tile = kTN columns of [c_begin, c_end) of the target matrix; phase A
    // reads the whole kTN-wide box (its extra columns are never used), phase C
    // touches only the tile's own columns
    // SPLIT: a cluster of nsplit CTAs (consecutive in x) shares one tile, CTA
    // `half` taking block rows [half * rows_per, (half + 1) * rows_per)
    // (rows_per a multiple of 128); their W parts are summed through
    // distributed shared memory before phase B
    const int half = SPLIT ? (int)(blockIdx.x % nsplit) : 0;
    const int c0 = c_begin + (int)(SPLIT ? blockIdx.x / nsplit : blockIdx.x) * kTN;  // first column of the tile
    const int nct = min(kTN, c_end - c0);
    // H: ld rows x hcols columns per matrix (column-major); the reflectors of
    // columns k .. k+31 (fewer at the end), tau hcols values per matrix
    const int m = ld - k;                          // rows k .. ld-1
    const int r_begin = half * rows_per;           // this CTA's first block row
    const int mloc = SPLIT ? max(0, min(m, r_begin + rows_per) - r_begin) : m;
    const int g0 = r_begin / kRC;                  // its first 32-row chunk
    const int wv = min(kPanel, min(m, hcols - k));  // reflectors of the panel
    const float *Hm = H + mat * (int64_t)ld * hcols;
    const float *Vbase = Hm + (int64_t)k * ld + k;  // V(r, j) at Vbase[j * ld + r]

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kOffBar);  // [kStages]
    uint64_t *mmab = full + kStages;                                // [2]
    uint64_t *cbar = full + kStages + 2;                            // phase-C MMA
    uint64_t *never = full + kStages + 3;                           // the test hook's barrier
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 64);
    float *Ts = reinterpret_cast<float *>(smem + kOffT);    // S(l, c) at c * 32 + l
    float *taus = reinterpret_cast<float *>(smem + kOffTau);
    const uint32_t sbase = tc::smem_addr(smem);
    const int nchunks = (mloc + kRC - 1) / kRC;  // this CTA's chunks

    // thread 0: barriers, then the first kStages chunks (and S with chunk 0)
    // start streaming at once
    // (barriers, tensor-map prefetch and the TMEM allocation overlap the end
    // of the previous kernel; at most two CTAs of this kernel fit on an SM by
    // shared memory, so the two 256-column allocations never wait)
    if (tid == 0) {
        tc::prefetch_tensormap(&tmC);
        tc::prefetch_tensormap(&tmV);
        tc::prefetch_tensormap(&tmCQ);
        for (int i = 0; i < kStages + 4; ++i) tc::mbar_init(&full[i], 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        __syncwarp();
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    pdl_wait();  // the panel (and everything before it) has completed
    if (tid == 0) {
        for (int s = 0; s < kStages && s < nchunks; ++s) {
            unsigned char *st = smem + s * kStageBytes;
            tc::mbar_expect_tx(&full[s], kLoadBytes + (s == 0 ? 4096u : 0u));
            tc::tma_load_3d(st, &tmC, k + (g0 + s) * kRC, c0, (int)mat, &full[s]);
            tc::tma_load_3d(st + kCBytes, &tmV, k + (g0 + s) * kRC, k, (int)mat, &full[s]);
            if (s == 0) tc::bulk_load(smem + kOffT, Sws + mat * s_stride, 4096u, &full[0]);
        }
    }
    float tau_r = 0.0f;
    if (tid < wv) tau_r = tau[mat * hcols + k + tid];  // stored to shared memory after phase A
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // copies and MMA groups issued / waited for per barrier (the same in
    // every thread; thread 0 uses them to drain after a timeout)
    int loads = kStages < nchunks ? kStages : nchunks;  // chunks whose TMA was issued
    uint32_t mma_issued[2] = {0, 0}, mma_waited[2] = {0, 0};
    bool ok = true, bad = false;  // bad: this thread saw an MMA wait give up

    // ---- phase A: W^T = C^T V over all rows --------------------------------
    // Every exit from the loop is uniform: it happens only at the CTA-wide
    // __syncthreads_or, which also folds in an MMA wait that gave up in the
    // previous iteration.
    for (int i = 0; i < nchunks; ++i) {
        const int sidx = i % kStages, b = i & 1;
        unsigned char *st = smem + sidx * kStageBytes;
        const bool landed = (flags & kFlagForceTimeout) && i == 0
                                ? tc::mbar_wait(never, 0u, 2000000ull)
                                : tc::mbar_wait(&full[sidx], (uint32_t)(i / kStages) & 1u, kWaitLimit);
        // run by every thread (the TMEM stores are warp-collective); after a
        // wait that gave up it moves garbage that no MMA reads: the loop
        // ends at the barrier below
        const uint32_t lane_q = tmem + ((uint32_t)(32 * warp) << 16);
        tc::fence_after_sync();  // after the wait for chunk i-2's MMAs, which read this A buffer
        split_stage(st, lane_q + kAHi + 64u * b, lane_q + kALo + 64u * b, g0 + i == 0, tid);
        tc::tmem_st_wait();
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        ok = !__syncthreads_or(!landed || bad);
        if (!ok) break;
        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t sV = sbase + sidx * kStageBytes + kCBytes;
#pragma unroll
            for (int s = 0; s < kRC / 8; ++s) {
                const uint32_t ko = (uint32_t)s * 32;  // 8 K elements inside the swizzle atom
                const uint64_t bv = tc::smem_desc_sw128(sV + ko);  // V rows, then V_lo rows
                const uint32_t acc = (i > 0 || s > 0) ? 1u : 0u;
                // A from tensor memory: K elements 8s .. 8s+7 are columns 8s ..
                tc::mma_tf32_ts(tmem + kDA, tmem + kAHi + 64u * b + 8u * s, bv, kIdescA, acc);
                tc::mma_tf32_ts(tmem + kDA2, tmem + kALo + 64u * b + 8u * s, bv, kIdescA2, acc);
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
                bad = true;  // made uniform by the next __syncthreads_or
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
        const int lb = (nchunks - 1) & 1;  // the last chunk's MMAs
        const bool done = tc::mbar_wait(&mmab[lb], mma_waited[lb] & 1u, kWaitLimit);
        if (done) ++mma_waited[lb];
        ok = !__syncthreads_or(!done);
    }
    if (tid < kPanel) taus[tid] = tau_r;
    __syncthreads();

    // the next kernel may be scheduled (it waits for this grid): from here
    // when the launch is large (the next panel's CTAs are placed while this
    // grid's last wave finishes), else after phase C, so that waiting CTAs do
    // not hold SMs the other half of a split batch could use
    if (early_trigger) pdl_trigger();

    // ---- phase C set-up
    const int ncc = (mloc + kRCC - 1) / kRCC;  // this CTA's 128-row chunks
    // quarters per chunk that hold tile columns: a tile narrower than kTN (the
    // end of [c_begin, c_end)) must not touch the quarters beyond c_end
    const int nqc = (nct + kCQCols - 1) / kCQCols;
    float e[kPanel];  // V rows of the next phase-C chunk
    if (ok) load_v_rows(Vbase, ld, r_begin, m, wv, tid, e);

    // ---- phase B: Y = T^T W, thread = tile column c ------------------------
    // W^T row c = hi*hi + hi*lo + lo*hi parts (three 32-column slices)
    const uint32_t wrow = tmem + ((uint32_t)(32 * warp) << 16);
    auto read_w = [&](float (&w)[32]) {
        float y[32];
        tc::tmem_ld_32x32(wrow + kDA, w);
        tc::tmem_ld_wait();
        tc::tmem_ld_32x32(wrow + kDA + 32, y);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] += y[j];
        tc::tmem_ld_32x32(wrow + kDA2, y);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] += y[j];
    };
    float wsum[32];
    if constexpr (SPLIT) {
        // The cluster's W parts are summed by a reduce-scatter and an
        // all-gather over distributed shared memory: rank r owns the slice of
        // q = 32 / nsplit columns [r q, r q + q).  Every rank writes slice r of
        // its part into rank r's area A (slot = source rank), each rank sums
        // its slice over the sources in rank order and writes the sum into
        // every rank's area B (slot = owner rank), so all ranks hold bitwise
        // the same W.  Areas A and B (16 KB each, any nsplit of 2, 4 or 8) lie
        // in the -P staging area, which phase C uses only later.  Every CTA
        // passes all three cluster barriers, whatever its `ok` (a CTA whose
        // wait gave up has set the status word; the results are reported
        // invalid).
        if (ok) {
            tc::fence_after_sync();
            read_w(wsum);
        }
        cg::cluster_group cl = cg::this_cluster();
        const int q = kPanel / nsplit;  // 16, 8 or 4 floats per slice
        float *xa = reinterpret_cast<float *>(smem + kOffCQ);                // [src][q / 4][thread][4]
        float *xg = reinterpret_cast<float *>(smem + kOffCQ + kXchgBytes);   // [owner][q / 4][thread][4]
        cl.sync();  // every CTA of the cluster is done with its phase-A ring
        if (ok) {
            // register indices stay compile-time constants; only the
            // destination rank and offset are computed
#pragma unroll
            for (int j4 = 0; j4 < kPanel / 4; ++j4) {
                const int j = 4 * j4, own = j / q, jq = (j - own * q) / 4;
                *reinterpret_cast<float4 *>(cl.map_shared_rank(xa, own) + half * (q * kThreads) +
                                            (jq * kThreads + tid) * 4) =
                    make_float4(wsum[j], wsum[j + 1], wsum[j + 2], wsum[j + 3]);
            }
        }
        cl.sync();
        if (ok) {
            for (int j4 = 0; j4 < q / 4; ++j4) {
                float4 t = *reinterpret_cast<const float4 *>(xa + (j4 * kThreads + tid) * 4);
                for (int rk = 1; rk < nsplit; ++rk) {
                    const float4 v =
                        *reinterpret_cast<const float4 *>(xa + rk * (q * kThreads) + (j4 * kThreads + tid) * 4);
                    t.x += v.x;
                    t.y += v.y;
                    t.z += v.z;
                    t.w += v.w;
                }
                for (int rk = 0; rk < nsplit; ++rk)
                    *reinterpret_cast<float4 *>(cl.map_shared_rank(xg, rk) + half * (q * kThreads) +
                                                (j4 * kThreads + tid) * 4) = t;
            }
        }
        cl.sync();
        if (ok) {
#pragma unroll
            for (int j4 = 0; j4 < kPanel / 4; ++j4) {
                const int j = 4 * j4, own = j / q, jq = (j - own * q) / 4;
                const float4 v =
                    *reinterpret_cast<const float4 *>(xg + own * (q * kThreads) + (jq * kThreads + tid) * 4);
                wsum[j] = v.x;
                wsum[j + 1] = v.y;
                wsum[j + 2] = v.z;
                wsum[j + 3] = v.w;
            }
        }
    }
    if (ok) {
        tc::fence_after_sync();
        float w[32], y[32];
        if constexpr (SPLIT) {
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = wsum[j];
        } else {
            read_w(w);
        }
        const int c = 32 * warp + lane;
        // T = D (I + S D)^-1 with D = diag(tau), S = strict_upper(V^T V).
        if constexpr (ApplyT) {
            // Y = T^T W (apply H^T): (I + D S^T) Y = D W, forward substitution
            //   y_c = tau_c (w_c - sum_{l < c} S(l, c) y_l)
#pragma unroll
            for (int cc = 0; cc < 32; ++cc) {
                float a = w[cc];
#pragma unroll
                for (int l = 0; l < cc; ++l) a = fmaf(-Ts[cc * 32 + l], y[l], a);
                y[cc] = taus[cc] * a;
            }
        } else {
            // Y = T W (apply H): (I + S D) Z = W, Y = D Z, back substitution
            //   y_c = tau_c (w_c - sum_{l > c} S(c, l) y_l)
#pragma unroll
            for (int cc = 31; cc >= 0; --cc) {
                float a = w[cc];
#pragma unroll
                for (int l = cc + 1; l < 32; ++l) a = fmaf(-Ts[l * 32 + cc], y[l], a);
                y[cc] = taus[cc] * a;
            }
        }
        // Y as the K-major B operand of phase C, 128-byte swizzle layout:
        // column c's 32 values at c * 128, 16-byte piece jq at (jq ^ (c % 8)) * 16
#pragma unroll
        for (int jq = 0; jq < 8; ++jq) {
            const float4 v = make_float4(y[4 * jq], y[4 * jq + 1], y[4 * jq + 2], y[4 * jq + 3]);
            const uint32_t off = (uint32_t)(c * 128 + ((jq ^ (c & 7)) << 4));
            *reinterpret_cast<float4 *>(smem + kOffYraw + off) = v;
            *reinterpret_cast<float4 *>(smem + kOffYlo + off) =
                make_float4(tc::tf32_lo(v.x), tc::tf32_lo(v.y), tc::tf32_lo(v.z), tc::tf32_lo(v.w));
        }
        store_v_rows(e, smem + kOffVCraw, smem + kOffVClo, tid);
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();  // the W load precedes phase C's MMAs into the same columns
    }

    // ---- phase C: C -= V Y, 128 rows per chunk -----------------------------
    // MMA(j) writes P[j % 2]; it is issued once MMA(j-1) has completed and
    // chunk j's V rows (loaded into registers one chunk ahead) are staged, so
    // it runs during the epilogue of chunk j-1.  The epilogue works in C
    // quarters of 32 columns that TMA loads two ahead and stores back.
    uint32_t c_issued = 0, c_waited = 0;
    auto issue_c = [&](int j) {
        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t d = tmem + ((j & 1) ? kDP1 : kDP0);
#pragma unroll
            for (int s = 0; s < kPanel / 8; ++s) {
                // A = V (K-major, M = rows), B = Y (K-major, N = columns),
                // both 128-byte swizzled: 8 K elements = +32 bytes per step
                const uint32_t ko = (uint32_t)s * 32;
                const uint64_t ah = tc::smem_desc_sw128(sbase + kOffVCraw + ko);
                const uint64_t al = tc::smem_desc_sw128(sbase + kOffVClo + ko);
                const uint64_t bh = tc::smem_desc_sw128(sbase + kOffYraw + ko);
                const uint64_t bl = tc::smem_desc_sw128(sbase + kOffYlo + ko);
                tc::mma_tf32(d, al, bh, kIdescC, s > 0 ? 1u : 0u);
                tc::mma_tf32(d, ah, bl, kIdescC, 1u);
                tc::mma_tf32(d, ah, bh, kIdescC, 1u);
            }
            tc::mma_commit(cbar);
        }
        ++c_issued;
    };
    if (ok) {
        ok = !__syncthreads_or(false);  // Y and V(0) staged
        issue_c(0);
        if (ncc > 1) load_v_rows(Vbase, ld, r_begin + kRCC, m, wv, tid, e);
    }
    for (int j = 0; j < ncc && ok; ++j) {
        const bool done = tc::mbar_wait(cbar, c_waited & 1u, kWaitLimit);
        if (done) ++c_waited;
        if (done && j + 1 < ncc) {
            store_v_rows(e, smem + kOffVCraw, smem + kOffVClo, tid);
            tc::fence_proxy_async_smem();
        }
        ok = !__syncthreads_or(!done);
        if (!ok) break;
        if (j + 1 < ncc) issue_c(j + 1);
        if (j + 2 < ncc) load_v_rows(Vbase, ld, r_begin + (j + 2) * kRCC, m, wv, tid, e);
        tc::fence_after_sync();
        const uint32_t pc = tmem + ((uint32_t)(32 * warp) << 16) + ((j & 1) ? kDP1 : kDP0);
        // epilogue: thread = row j * 128 + tid of the tile.  -P goes to a
        // shared quarter (32 columns) that TMA adds into C at the L2: no load
        // of C, half the shared-memory traffic of load/subtract/store, and
        // C - P and C + (-P) round identically.  Rows and columns past the
        // end of C are outside the tensor map and are not written.  Each
        // warp stages and reduce-adds its own 32 rows (a 4 KB slice of the
        // two quarter buffers), so the epilogue needs no CTA barrier: lane 0
        // of the warp owns the warp's bulk groups.
        for (int q = 0; q < nqc; ++q) {
            const int u = j * nqc + q;
            float pv[32];
            tc::tmem_ld_32x32(pc + kCQCols * q, pv);
            tc::tmem_ld_wait();
            float *cs = reinterpret_cast<float *>(smem + kOffCQ + (u & 1) * kCQBytes) + warp * (32 * kCQCols);
            // the warp's reduce of quarter u-2 (same slice) has read it; the
            // one of quarter u-1 may still be in flight
            if (lane == 0) tc::bulk_wait_group_read<1>();
            __syncwarp();
#pragma unroll
            for (int c = 0; c < kCQCols; ++c) cs[c * 32 + lane] = -pv[c];
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::tma_reduce_add_3d(&tmCQ, k + r_begin + kRCC * j + 32 * warp, c0 + kCQCols * q, (int)mat,
                                      cs);
                tc::bulk_commit_group();
            }
        }
        tc::fence_before_sync();
    }
    if (!early_trigger) pdl_trigger();
    if (lane == 0) tc::bulk_wait_group<0>();  // each warp's reduces complete before shared memory goes away

    if (!ok && tid == 0) {
        atomicOr(status, 1);
        // let copies and MMA groups that did not signal in time drain
        // (bounded) before the shared and tensor memory is released
        for (int i = 0; i < loads; ++i) {
            // full[s] completes once per chunk issued into stage s; waiting on
            // the parity of the last one covers the earlier ones
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

bool trailing_tc_supported(int ld)
{
    return ld % 4 == 0 && ld >= 128;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

}  // namespace

cudaError_t prepare_apply_maps(const float *H, int ld, int hcols, float *C, int64_t c_cols, int64_t batch,
                               TrailingMaps *maps)
{
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    // H and C as 3-D tensors: x = row (contiguous), y = column, z = matrix
    const cuuint64_t hdims[3] = {(cuuint64_t)ld, (cuuint64_t)hcols, (cuuint64_t)batch};
    const cuuint64_t hstrides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)ld * (cuuint64_t)hcols * 4};
    const cuuint64_t cdims[3] = {(cuuint64_t)ld, (cuuint64_t)c_cols, (cuuint64_t)batch};
    const cuuint64_t cstrides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)ld * (cuuint64_t)c_cols * 4};
    const cuuint32_t box_c[3] = {kRC, kTN, 1}, box_v[3] = {kRC, kPanel, 1}, unit[3] = {1, 1, 1};
    const cuuint32_t box_v64[3] = {kRC, 2 * kPanel, 1};
    const cuuint32_t box_cq[3] = {32, kCQCols, 1};  // one warp's 32 rows of a quarter
    if (enc(&maps->c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, C, cdims, cstrides, box_c, unit,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&maps->v, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(H), hdims, hstrides, box_v, unit,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&maps->cq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, C, cdims, cstrides, box_cq, unit,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&maps->v64, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(H), hdims, hstrides, box_v64,
            unit, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    return cudaSuccess;
}

cudaError_t encode_rowmajor_tiles(const float *A, int64_t batch, int rows, int cols, int64_t bs, int64_t rs,
                                  CUtensorMap *map)
{
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    // x = column (contiguous), y = row, z = matrix; 32 x 32 boxes, 128-byte swizzle
    const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
    const cuuint64_t strides[2] = {(cuuint64_t)rs * 4, (cuuint64_t)(batch > 1 ? bs : (int64_t)rows * rs) * 4};
    const cuuint32_t box[3] = {32, 32, 1}, unit[3] = {1, 1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(A), dims, strides, box, unit,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    return cudaSuccess;
}

cudaError_t prepare_trailing_tc(float *H, int64_t batch, int m, int n, TrailingMaps *maps)
{
    return prepare_apply_maps(H, m, n, H, n, batch, maps);
}

// Static plan by n: a large launch triggers the next kernel early (its CTAs
// are placed while the last wave finishes).
static int trailing_flags(int ld)
{
    return (ld > 256 ? kFlagEarlyTrigger : 0) | ((debug_flags() & kMidFlagForceTimeout) ? kFlagForceTimeout : 0);
}

cudaError_t launch_apply_tc(const TrailingMaps &maps, const float *H, const float *Sws, int64_t s_stride,
                            const float *tau, int *status, int64_t batch, int ld, int hcols, int k, int c_begin,
                            int c_end, bool apply_t, cudaStream_t st)
{
    if (c_end <= c_begin || k >= hcols || k >= ld) return cudaSuccess;
    auto kern = apply_t ? trailing_tc_kernel<true> : trailing_tc_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    const unsigned tiles = (unsigned)((c_end - c_begin + kTN - 1) / kTN);
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
        const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
        dim3 grid(tiles, (unsigned)nb);
        e = launch_dependent(kern, grid, dim3(kThreads), kSmem, st, nullptr, 0, maps.c, maps.v, maps.cq, H, Sws,
                             s_stride, tau, status, ld, hcols, k, c_begin, c_end, b0, trailing_flags(ld), 1,
                             ld - k);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Ranks per tile: 1 (one CTA per tile) unless all tiles of the call fit one
// CTA per SM and a tile has >= 256 rows; then the largest split of 2, 4 or 8
// that still fits two CTAs per SM (296 on 148 SMs) with >= 128 rows (one
// phase-C chunk) per rank.  Measured at n = 1024 (ms per call): one matrix
// 1.78 -> 1.68, two 2.01 -> 1.87, eight 1.99 -> 1.88 against two ranks;
// >= 256 rows per rank gained ~1%; many-tile calls are unchanged.
static int trailing_split(int64_t batch_all, int64_t tiles, int rows)
{
    if (rows < 256 || tiles * batch_all > 148) return 1;
    int ns = 2;
    while (ns < kMaxSplit && tiles * batch_all * ns * 2 <= 296 && rows >= ns * 2 * kRCC) ns *= 2;
    // every rank must own at least one row (rows per rank: a multiple of 128)
    while (ns > 1 && (int64_t)(ns - 1) * ((rows + ns * kRCC - 1) / (ns * kRCC) * kRCC) >= rows) ns /= 2;
    return ns;
}

cudaError_t launch_trailing_tc(const TrailingMaps &maps, float *H, const float *Sws, int64_t s_stride,
                               const float *tau, int *status, int64_t batch, int64_t batch_all, int m, int n, int k,
                               cudaStream_t st)
{
    if (n - k - kPanel <= 0) return cudaSuccess;
    // Static plan by (the call's batch, n, k), as for the rank-64 update:
    // when all tiles of the call fit one CTA per SM, a cluster of CTAs shares
    // each tile's rows (trailing_split)
    const int64_t tiles = (n - k - kPanel + kTN - 1) / kTN;
    const int rows = m - k;
    const int kSplit = trailing_split(batch_all, tiles, rows);
    if (kSplit == 1)
        return launch_apply_tc(maps, H, Sws, s_stride, tau, status, batch, m, n, k, k + kPanel, n, true, st);
    auto kern = trailing_tc_kernel<true, true>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    const int rows_per = (rows + kSplit * kRCC - 1) / (kSplit * kRCC) * kRCC;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
        const int64_t nb = (batch - b0) < 65535 ? (batch - b0) : 65535;
        e = launch_dependent(kern, dim3((unsigned)(tiles * kSplit), (unsigned)nb), dim3(kThreads), kSmem, st, attr,
                             1, maps.c, maps.v, maps.cq, H, Sws, s_stride, tau, status, m, n, k, k + kPanel, n, b0,
                             trailing_flags(m), kSplit, rows_per);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fqr
