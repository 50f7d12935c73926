// C ABI of libfastqr.so (declared in include/fastqr.h).
//
// Static dispatch on (batch, m, n) only:
//   m == n <= 64 : one warp per matrix, registers (qr_small.cu)
//   (m == n in [128, 256], n % 4 == 0, with fqr_debug_plan(1) only: one
//                  launch, one CTA per matrix running its whole blocked
//                  factorisation, qr_mid.cu)
//   otherwise    : blocked compact-WY: copy-in, then per 32-column panel a
//                  panel kernel and a trailing-update kernel (qr_blocked.cu);
//                  for n >= 2048 (and m <= 4096) per 64 columns two panels,
//                  the in-block update between them, the cross Gram block
//                  and one rank-64 trailing update; rectangular m x n (m > n)
//                  always takes this path
// No path inspects matrix values and there is no CPU fallback: a failed
// launch is reported as a status code.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/fastqr.h"
#include "internal.h"

namespace {

using fqr::kWsAlign;

// Streams a batch is split over (static plan by batch and n).  Parts on
// concurrent streams fill the SMs one part's chain leaves idle, but a small
// batch leaves SMs idle either way and one chain of launches is shorter (half
// the launches to enqueue, too).  One part up to 64 matrices and 17M matrix
// elements (n < 2048) or up to 140M elements (n >= 2048), else two (n < 2048)
// or four (64 x 1024^2 was 16% slower with one part).  Measured
// against the earlier fixed two / four parts, steps back to back: 32 and
// 64 x 256^2 -2.7% and -2.0%, 8 x 1024^2 -0.6%, 2 and 4 x 4096^2 -1.2% and
// -0.4% (per call with a synchronize after each: -9%, -8.6%, -5%, -8.4%);
// 128 x 256^2 was 2.7% slower with one part.  Three parts at n < 2048
// measured +4% to +18%.
constexpr int kMaxSplitParts = 4;
int split_parts(int64_t batch, int64_t n)
{
    const double elems = (double)batch * (double)n * (double)n;
    const int want = n >= 2048 ? (elems <= 140e6 ? 1 : 4) : (batch <= 64 && elems <= 17e6 ? 1 : 2);
    return batch < want ? (int)batch : want;
}

bool use_tc(int64_t n) { return fqr::trailing_tc_supported((int)n); }

bool small_path(int64_t n) { return n <= 64; }

std::atomic<int> g_debug_flags{0};
std::atomic<int> g_debug_plan{0};  // 1: the one-launch mid-size kernel where it applies

// The one-launch mid-size kernel (qr_mid.cu) is not in the static plan: the
// blocked path measured faster at every batch size tried for 128 <= n <= 256
// (B200, batch 1 .. 1024).  fqr_debug_plan(1) selects it (aligned H, which
// every torch / cudaMalloc allocation is).
bool mid_path(int64_t n) { return g_debug_plan.load() == 1 && fqr::mid_supported(n, n, nullptr); }

int status_from(cudaError_t e)
{
    if (e == cudaSuccess) return FQR_OK;
    if (e == cudaErrorInvalidValue || e == cudaErrorInvalidConfiguration) return FQR_ELAUNCH;
    return FQR_ELAUNCH;
}

}  // namespace

int fqr::debug_flags() { return g_debug_flags.load(); }

extern "C" {

int fqr_version(void) { return 100; }

int fqr_debug_plan(int mode) { return g_debug_plan.exchange(mode == 1 ? 1 : 0); }

int fqr_debug_force_timeout(int enable)
{
    return g_debug_flags.exchange(enable ? fqr::kMidFlagForceTimeout : 0) != 0;
}

const char *fqr_status_string(int status)
{
    switch (status) {
    case FQR_OK: return "ok";
    case FQR_EINVAL: return "invalid argument (null pointer, negative size or bad stride)";
    case FQR_EUNSUPPORTED: return "unsupported size (n outside the dispatch table)";
    case FQR_ELAUNCH: return "kernel launch failed";
    case FQR_ETIMEOUT: return "device-side bounded wait timed out";
    case FQR_EWORKSPACE: return "workspace missing or too small";
    case FQR_ECUDA: return "CUDA runtime error";
    case FQR_ENOALLOC_LIMIT:
        return "problem needs more scratch than fqr_geqrf_f32_noalloc's static area "
               "(n > 64 with batch > FQR_NOALLOC_MAX_BATCH)";
    default: return "unknown status";
    }
}

size_t fqr_workspace_bytes(int64_t batch, int64_t n)
{
    if (batch <= 0 || n <= 0 || n > FQR_MAX_N || small_path(n)) return 0;
    // a status block, then one S block per matrix (32 x 32, or 64 x 64 for
    // the rank-64 plan)
    return fqr::ws_total_bytes(batch, n, n);
}

int fqr_launch_count(int64_t batch, int64_t n)
{
    if (batch <= 0 || n <= 0) return 0;
    if (n > FQR_MAX_N) return -1;
    if (small_path(n) || mid_path(n)) return 1;
    const bool outer = use_tc(n) && fqr::use_outer64(n, n);
    // copy-in + per panel (panel + trailing), the last panel has no trailing;
    // the rank-64 plan has per 64-column block two panels, the in-block
    // update and (all but the last block) the Gram block and one trailing
    // update, then rank-32 steps for the columns left
    const int64_t blocks = outer ? n / fqr::kOuter : 0;
    const int64_t rest = n - blocks * fqr::kOuter;
    const int64_t panels = (rest + fqr::kPanel - 1) / fqr::kPanel;
    auto range = [blocks, rest, panels](int64_t b) {
        const int64_t chunks = (b + 65534) / 65535;
        int64_t t = 1 + panels + (panels > 0 ? panels - 1 : 0) * chunks;
        if (blocks > 0) {
            const int64_t full = rest > 0 ? blocks : blocks - 1;  // blocks with a trailing update
            t += blocks * 3 + full * (1 + chunks);
        }
        return t;
    };
    // a batch of two or more runs as split_parts(batch, n) parts on as many
    // streams
    const int64_t parts = split_parts(batch, n);
    int64_t total = 0;
    for (int64_t p = 0; p < parts; ++p) total += range(batch * (p + 1) / parts - batch * p / parts);
    return (int)total;
}

int fqr_plan_describe(int64_t batch, int64_t n, char *buf, size_t len)
{
    if (!buf || len == 0) return FQR_EINVAL;
    if (n > FQR_MAX_N || n < 0 || batch < 0) {
        snprintf(buf, len, "unsupported");
        return FQR_EUNSUPPORTED;
    }
    if (small_path(n)) {
        snprintf(buf, len, "small: warp-per-matrix registers, n<=%d, %lld warps, 1 launch",
                 n <= 32 ? 32 : 64, (long long)batch);
    } else if (mid_path(n)) {
        snprintf(buf, len,
                 "mid: one CTA per matrix (%lld CTAs, 2 per SM), panel %d cols in registers + tcgen05 3xTF32 "
                 "rank-%d update per panel, 1 launch",
                 (long long)batch, fqr::kPanel, fqr::kPanel);
    } else {
        const fqr::PanelShape s = fqr::panel_shape((int)n);
        const bool outer = use_tc(n) && fqr::use_outer64(n, n);
        snprintf(buf, len,
                 "blocked: panel %d cols (first panel %d warps x %d row blocks, cluster %d), "
                 "trailing %s rank %d, %d launches",
                 fqr::kPanel, s.warps, s.rows_per_thread_blocks, s.cluster,
                 use_tc(n) ? "tcgen05 3xTF32" : "simt fp32", outer ? fqr::kOuter : fqr::kPanel,
                 fqr_launch_count(batch, n));
    }
    return FQR_OK;
}

}  // extern "C"

namespace {

// Optional per-stage timing: CUDA events recorded on the launch stream around
// every kernel, summed per stage after a final stream synchronize.
struct StageTimer {
    cudaStream_t st;
    cudaEvent_t ev[2 * 1024];
    int stage[1024];
    int count = 0;
    bool ok = true;
    void begin(int s)
    {
        if (count >= 1024) { ok = false; return; }
        if (cudaEventCreate(&ev[2 * count]) != cudaSuccess ||
            cudaEventCreate(&ev[2 * count + 1]) != cudaSuccess) { ok = false; return; }
        stage[count] = s;
        cudaEventRecord(ev[2 * count], st);
    }
    void end()
    {
        if (!ok) return;
        cudaEventRecord(ev[2 * count + 1], st);
        ++count;
    }
    int finish(float *ms, int nstages)
    {
        cudaError_t e = cudaStreamSynchronize(st);
        for (int i = 0; i < nstages; ++i) ms[i] = 0.0f;
        for (int i = 0; i < count; ++i) {
            float t = 0.0f;
            if (e == cudaSuccess) cudaEventElapsedTime(&t, ev[2 * i], ev[2 * i + 1]);
            if (stage[i] < nstages) ms[stage[i]] += t;
            cudaEventDestroy(ev[2 * i]);
            cudaEventDestroy(ev[2 * i + 1]);
        }
        if (e != cudaSuccess) return FQR_ECUDA;
        return ok ? FQR_OK : FQR_ELAUNCH;
    }
};

// The blocked path for one batch range of m x n matrices (m >= n): copy-in,
// then per 32-column panel a panel kernel and a trailing update, all on `st`;
// with the rank-64 plan, per 64 columns: panel(k), the update of columns
// k+32 .. k+63 by panel k's reflectors, panel(k+32), the Gram block
// V1^T V2 and one trailing update with all 64 reflectors.
int enqueue_blocked(const float *A, int64_t batch, int64_t batch_all, int m, int n, int64_t a_bstride,
                    int64_t a_rstride, int64_t a_cstride, float *H, float *tau, float *Sws, int *status_base,
                    int part, unsigned clear_mask, bool tc, cudaStream_t st, StageTimer *tm)
{
    // status_base[part] records a bounded wait that gave up; the copy-in
    // clears the words of clear_mask
    int *status = status_base + part;
    fqr::TrailingMaps maps;
    if (tc && fqr::prepare_trailing_tc(H, batch, m, n, &maps) != cudaSuccess) return FQR_ECUDA;
    const int64_t s_stride = fqr::s_block_floats(m, n);
    cudaError_t e;
    auto step = [&](int stage, auto &&launch) -> bool {
        if (tm) tm->begin(stage);
        e = launch();
        if (tm) tm->end();
        return e == cudaSuccess;
    };
    if (!step(FQR_STAGE_COPY_IN, [&] {
            return fqr::launch_copy_in(A, batch, m, n, a_bstride, a_rstride, a_cstride, H, status_base, clear_mask,
                                       st);
        }))
        return status_from(e);
    int k = 0;
    if (tc && fqr::use_outer64(m, n)) {
        // S of both panels on the diagonal of one 64 x 64 row-major block per
        // matrix; the Gram step adds the off-diagonal block
        const fqr::SBlock s11{Sws, s_stride, fqr::kOuter, 1};
        const fqr::SBlock s22{Sws + fqr::kPanel * fqr::kOuter + fqr::kPanel, s_stride, fqr::kOuter, 1};
        for (; n - k >= fqr::kOuter; k += fqr::kOuter) {
            if (!step(FQR_STAGE_PANEL, [&] { return fqr::launch_panel(H, tau, s11, batch, m, n, k, st); }) ||
                !step(FQR_STAGE_INBLOCK,
                      [&] { return fqr::launch_inblock(H, tau, Sws, s_stride, batch, m, n, k, false, st); }) ||
                !step(FQR_STAGE_PANEL,
                      [&] { return fqr::launch_panel(H, tau, s22, batch, m, n, k + fqr::kPanel, st); }))
                return status_from(e);
            if (n - k > fqr::kOuter &&
                (!step(FQR_STAGE_INBLOCK,
                       [&] { return fqr::launch_inblock(H, tau, Sws, s_stride, batch, m, n, k, true, st); }) ||
                 !step(FQR_STAGE_TRAILING, [&] {
                     return fqr::launch_trailing64_tc(maps, H, Sws, s_stride, tau, status, batch, batch_all, m, n,
                                                      k, st);
                 })))
                return status_from(e);
        }
    }
    // rank-32 steps (the whole matrix, or the columns the rank-64 blocks
    // left); a wide block (m < n) has m reflectors, and every trailing update
    // also covers its columns m .. n-1
    const fqr::SBlock s32{Sws, s_stride, 1, fqr::kPanel};
    const int kend = m < n ? m : n;
    for (; k < kend; k += fqr::kPanel) {
        if (!step(FQR_STAGE_PANEL, [&] { return fqr::launch_panel(H, tau, s32, batch, m, n, k, st); }))
            return status_from(e);
        // the panel's reflectors (fewer than 32 only in the last panel) reach
        // every column right of them: k + 32 .. n-1, or, for the last panel of
        // a wide block, k + m - k .. n-1
        const int w = fqr::kPanel < m - k ? (fqr::kPanel < n - k ? fqr::kPanel : n - k) : (m - k < n - k ? m - k : n - k);
        const int cb = k + w;
        if (cb < n && !step(FQR_STAGE_TRAILING, [&] {
                if (!tc) return fqr::launch_trailing(H, Sws, s_stride, tau, batch, m, n, k, cb, st);
                if (w == fqr::kPanel)
                    return fqr::launch_trailing_tc(maps, H, Sws, s_stride, tau, status, batch, batch_all, m, n, k, st);
                return fqr::launch_apply_tc(maps, H, Sws, s_stride, tau, status, batch, m, n, k, cb, n, true, st);
            }))
            return status_from(e);
    }
    return FQR_OK;
}

// Batches of two or more matrices run as split_parts(batch, n) parts on as
// many streams: the caller's and internal ones per device, which first wait
// for everything enqueued on the caller's stream before the call and which the
// caller's stream waits for at the end, so the call orders like a single
// launch.  The parts' kernels fill each other's idle SMs (the last, partial
// wave of every trailing launch; the single-CTA-per-matrix panels, whose time
// is a per-matrix latency chain).
constexpr int kSplitParts = kMaxSplitParts;
struct SplitStreams {
    bool ready = false;
    cudaStream_t side[kSplitParts - 1] = {};
    cudaEvent_t fork = nullptr, join[kSplitParts - 1] = {};
    std::mutex mu;
};
constexpr int kMaxDevices = 64;
SplitStreams g_split[kMaxDevices];

int enqueue_blocked_split(const float *A, int64_t batch, int m, int n, int64_t a_bstride, int64_t a_rstride,
                          int64_t a_cstride, float *H, float *tau, float *Sws, int *status, bool tc,
                          cudaStream_t st)
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FQR_ECUDA;
    SplitStreams &sp = g_split[dev];
    std::lock_guard<std::mutex> lock(sp.mu);
    if (!sp.ready) {
        if (cudaEventCreateWithFlags(&sp.fork, cudaEventDisableTiming) != cudaSuccess) return FQR_ECUDA;
        for (int i = 0; i < kSplitParts - 1; ++i)
            if (cudaStreamCreateWithFlags(&sp.side[i], cudaStreamNonBlocking) != cudaSuccess ||
                cudaEventCreateWithFlags(&sp.join[i], cudaEventDisableTiming) != cudaSuccess)
                return FQR_ECUDA;
        sp.ready = true;
    }
    const int parts = split_parts(batch, n);
    const size_t mn = (size_t)m * (size_t)n;
    if (cudaEventRecord(sp.fork, st) != cudaSuccess) return FQR_ECUDA;
    for (int i = 0; i + 1 < parts; ++i)
        if (cudaStreamWaitEvent(sp.side[i], sp.fork, 0) != cudaSuccess) return FQR_ECUDA;
    // part p: matrices [batch*p/parts, batch*(p+1)/parts) and status word p,
    // which its copy-in clears; part 0 (on the caller's stream) also clears
    // the words no part of this call uses, so that all of them read clear
    int rc = FQR_OK;
    const unsigned unused = (((1u << kSplitParts) - 1u) & ~((1u << parts) - 1u));
    for (int p = 0; p < parts; ++p) {
        const int64_t lo = batch * p / parts, hi = batch * (p + 1) / parts;
        const int r = enqueue_blocked(A + lo * a_bstride, hi - lo, batch, m, n, a_bstride, a_rstride, a_cstride,
                                      H + lo * mn, tau + lo * n, Sws + lo * fqr::s_block_floats(m, n),
                                      status, p, (1u << p) | (p == 0 ? unused : 0u), tc,
                                      p == 0 ? st : sp.side[p - 1], nullptr);
        if (rc == FQR_OK) rc = r;
    }
    // join even after a failure, so nothing of this call stays unordered with
    // later work on the caller's stream
    cudaError_t j = cudaSuccess;
    for (int i = 0; i + 1 < parts; ++i) {
        if (j == cudaSuccess) j = cudaEventRecord(sp.join[i], sp.side[i]);
        if (j == cudaSuccess) j = cudaStreamWaitEvent(st, sp.join[i], 0);
    }
    if (rc != FQR_OK) return rc;
    return j == cudaSuccess ? FQR_OK : FQR_ECUDA;
}

// status_word: where the tensor-core kernels record a bounded wait that gave
// up (NULL: the words after the S blocks in the workspace).  split: whether
// a batch of two or more may run as two halves on two streams.
// m: rows (m == n for the square entry points; m < n, a wide block, only
// through the rectangular entry, with tau [batch][n]).
int run_geqrf(const float *A, int64_t batch, int64_t m, int64_t n, int64_t a_bstride, int64_t a_rstride,
              int64_t a_cstride, float *H, float *tau, void *workspace, size_t workspace_bytes,
              cudaStream_t st, StageTimer *tm, int *status_word = nullptr, bool split = true,
              int64_t batch_in_flight = 0)
{
    if (batch < 0 || n < 0 || m < 0) return FQR_EINVAL;
    if (batch == 0 || n == 0) return FQR_OK;
    if (m > FQR_MAX_N || n > FQR_MAX_N) return FQR_EUNSUPPORTED;
    if ((int64_t)m * n > (int64_t)FQR_MAX_N * FQR_MAX_N) return FQR_EUNSUPPORTED;
    if (!A || !H || !tau) return FQR_EINVAL;
    if (a_rstride == 0 || a_cstride == 0 || (batch > 1 && a_bstride == 0)) return FQR_EINVAL;
    const int ni = (int)n, mi = (int)m;

    if (m == n && small_path(n)) {
        if (tm) tm->begin(FQR_STAGE_SMALL);
        cudaError_t e = fqr::launch_small(A, batch, ni, a_bstride, a_rstride, a_cstride, H, tau, st);
        if (tm) tm->end();
        return status_from(e);
    }

    const size_t need = fqr::ws_total_bytes(batch, m, n);
    if (!workspace || workspace_bytes < need) return FQR_EWORKSPACE;
    if (((uintptr_t)workspace) % kWsAlign) return FQR_EINVAL;
    // the status block first, then the S blocks
    float *Sws = (float *)((unsigned char *)workspace + kWsAlign);
    int *status = status_word ? status_word : (int *)workspace;
    if (m == n && g_debug_plan.load() == 1 && fqr::mid_supported(m, n, H)) {
        // one launch; an own status word (host entry, one per chunk) or the
        // whole status block of the workspace
        if (tm) tm->begin(FQR_STAGE_MID);
        cudaError_t e = fqr::launch_mid(A, batch, ni, a_bstride, a_rstride, a_cstride, H, tau, status,
                                        status_word ? 1 : kSplitParts, g_debug_flags.load(), st);
        if (tm) tm->end();
        return status_from(e);
    }
    const bool tc = use_tc(m) && ((uintptr_t)H % 16) == 0;
    if (split && !tm && batch >= 2)
        return enqueue_blocked_split(A, batch, mi, ni, a_bstride, a_rstride, a_cstride, H, tau, Sws, status,
                                     tc, st);
    // an own status word (host entry, one per chunk) or both words of the
    // workspace's status block
    return enqueue_blocked(A, batch, batch_in_flight > batch ? batch_in_flight : batch, mi, ni, a_bstride,
                           a_rstride, a_cstride, H, tau, Sws, status, 0,
                           status_word ? 1u : (1u << kSplitParts) - 1u, tc, st, tm);
}

}  // namespace

int fqr::geqrf_enqueue(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                       int64_t a_rstride, int64_t a_cstride, float *H, float *tau, void *workspace,
                       size_t workspace_bytes, cudaStream_t st)
{
    return run_geqrf(A, batch, n, n, a_bstride, a_rstride, a_cstride, H, tau, workspace,
                     workspace_bytes, st, nullptr);
}

int fqr::geqrf_enqueue_status(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                              int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                              void *workspace, size_t workspace_bytes, int *status_word,
                              int64_t batch_in_flight, cudaStream_t st)
{
    return run_geqrf(A, batch, n, n, a_bstride, a_rstride, a_cstride, H, tau, workspace,
                     workspace_bytes, st, nullptr, status_word, false, batch_in_flight);
}

extern "C" {

int fqr_geqrf_f32(const float *A, int64_t batch, int64_t n, int64_t a_bstride, int64_t a_rstride,
                  int64_t a_cstride, float *H, float *tau, void *workspace, size_t workspace_bytes,
                  void *stream)
{
    return run_geqrf(A, batch, n, n, a_bstride, a_rstride, a_cstride, H, tau, workspace,
                     workspace_bytes, (cudaStream_t)stream, nullptr);
}

size_t fqr_geqrf_rect_workspace_bytes(int64_t batch, int64_t m, int64_t n)
{
    if (batch <= 0 || n <= 0 || m <= 0 || m > FQR_MAX_N || n > FQR_MAX_N) return 0;
    if (m == n) return fqr_workspace_bytes(batch, n);
    return fqr::ws_total_bytes(batch, m, n);
}

int fqr_geqrf_rect_f32(const float *A, int64_t batch, int64_t m, int64_t n, int64_t a_bstride,
                       int64_t a_rstride, int64_t a_cstride, float *H, float *tau, void *workspace,
                       size_t workspace_bytes, void *stream)
{
    // a wide block has m reflectors: tau[b][m .. n-1] = 0, set first (the
    // updates read the tau of all 32 columns of the last panel), once the
    // arguments have passed the checks run_geqrf makes
    const bool wide = m > 0 && m < n && batch > 0 && n <= FQR_MAX_N;
    if (wide && (!A || !H || !tau)) return FQR_EINVAL;
    if (wide && (!workspace || workspace_bytes < fqr::ws_total_bytes(batch, m, n))) return FQR_EWORKSPACE;
    if (wide &&
        cudaMemset2DAsync(tau + m, (size_t)n * sizeof(float), 0, (size_t)(n - m) * sizeof(float), (size_t)batch,
                          (cudaStream_t)stream) != cudaSuccess)
        return FQR_ECUDA;
    return run_geqrf(A, batch, m, n, a_bstride, a_rstride, a_cstride, H, tau, workspace, workspace_bytes,
                     (cudaStream_t)stream, nullptr);
}

int fqr_check_status(const void *workspace, size_t workspace_bytes, int64_t batch, void *stream)
{
    if (batch <= 0) return FQR_OK;
    // the status block is the workspace's first 256 bytes
    if (!workspace || workspace_bytes < kSplitParts * sizeof(int)) return FQR_EINVAL;
    // one word per part of a batch split over streams; every call clears all
    // of them (each part its own, part 0 the unused ones)
    int v[kSplitParts] = {};
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemcpyAsync(v, workspace, sizeof(v), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return FQR_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return FQR_ECUDA;
    int any = 0;
    for (int i = 0; i < kSplitParts; ++i) any |= v[i];
    return any ? FQR_ETIMEOUT : FQR_OK;
}

int fqr_geqrf_f32_profile(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                          int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                          void *workspace, size_t workspace_bytes, void *stream, float *stage_ms)
{
    if (!stage_ms) return FQR_EINVAL;
    StageTimer *tm = new StageTimer();
    tm->st = (cudaStream_t)stream;
    int rc = run_geqrf(A, batch, n, n, a_bstride, a_rstride, a_cstride, H, tau, workspace,
                       workspace_bytes, (cudaStream_t)stream, tm);
    int rc2 = tm->finish(stage_ms, FQR_NUM_STAGES);
    delete tm;
    return rc != FQR_OK ? rc : rc2;
}

}  // extern "C"
