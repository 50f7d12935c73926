// fqr_geqrf_f32_host: batched QR of matrices held in HOST memory.
//
// The batch is cut into chunks.  Each chunk is copied host->device, factored
// and copied back device->host on one of up to kMaxSlots internal streams,
// each stream with its own device staging slot, so that the upload of chunk
// c+1, the factorisation of chunk c and the download of chunk c-1 run at the
// same time (the two copy directions use separate copy engines).  A call made
// through the device-pointer entry point pays the two transfers one after the
// other and after the kernels; here the whole call costs about one transfer
// plus the factorisation and download of a single chunk.
//
// Ordering with the caller: an event recorded on `stream` is waited on by
// every internal stream before its first copy, and `stream` waits on an event
// recorded at the end of each internal stream, so the call behaves like any
// other asynchronous work on `stream`.  The host buffers must stay valid and
// unmodified until `stream` has passed the call.  Copies overlap only when the
// host buffers are page-locked (cudaHostAlloc / cudaHostRegister); pageable
// buffers still give correct results, with the copies staged by the driver.
//
// The internal streams and events are created once per device, on the first
// call made with that device current, and live until the process exits.
// The enqueue sequence of a call holds a per-device mutex (the events are
// shared); kernels of concurrent calls still overlap on the GPU when their
// workspaces differ.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/fastqr.h"
#include "internal.h"

namespace {

using fqr::kWsAlign;

constexpr int kMaxSlots = 4;
constexpr int kMaxChunks = 8;
constexpr size_t kMinChunkBytes = size_t(1) << 20;  // 1 MiB of input per chunk at least
constexpr int kMaxDevices = 64;

constexpr size_t align_up(size_t x) { return (x + kWsAlign - 1) / kWsAlign * kWsAlign; }

// Chunking plan: a function of (batch, n) only.
struct HostPlan {
    int64_t chunk;     // matrices per chunk (the last one may be shorter)
    int64_t nchunks;
    int slots;         // staging slots = internal streams used
    size_t off_a, off_h, off_tau, off_ws, ws_bytes, slot_bytes;
    size_t status_bytes;  // per-chunk status words, at the start of the workspace
    size_t total;
};

bool host_plan(int64_t batch, int64_t n, HostPlan *p)
{
    if (batch <= 0 || n <= 0 || n > FQR_MAX_N) return false;
    const size_t mat = (size_t)n * (size_t)n * sizeof(float);
    const size_t all = mat * (size_t)batch;
    size_t target = all / kMaxChunks;
    if (target < kMinChunkBytes) target = kMinChunkBytes;
    int64_t chunk = (int64_t)((target + mat - 1) / mat);
    const int64_t min_chunk = (batch + kMaxChunks - 1) / kMaxChunks;  // at most kMaxChunks chunks
    if (chunk < min_chunk) chunk = min_chunk;
    if (chunk > batch) chunk = batch;
    if (chunk < 1) chunk = 1;
    p->chunk = chunk;
    p->nchunks = (batch + chunk - 1) / chunk;
    p->slots = (int)(p->nchunks < kMaxSlots ? p->nchunks : kMaxSlots);
    p->ws_bytes = fqr_workspace_bytes(chunk, n);
    p->off_a = 0;
    p->off_h = align_up((size_t)chunk * mat);
    p->off_tau = p->off_h + align_up((size_t)chunk * mat);
    p->off_ws = p->off_tau + align_up((size_t)chunk * (size_t)n * sizeof(float));
    p->slot_bytes = p->off_ws + align_up(p->ws_bytes);
    p->status_bytes = align_up((size_t)p->nchunks * sizeof(int));
    p->total = p->status_bytes + (size_t)p->slots * p->slot_bytes;
    return true;
}

struct DeviceStreams {
    bool ready = false;
    cudaStream_t st[kMaxSlots] = {};
    cudaEvent_t fork = nullptr;
    cudaEvent_t done[kMaxSlots] = {};
    std::mutex mu;
};
DeviceStreams g_dev[kMaxDevices];

// Internal streams and events of the current device (created once).
int device_streams(DeviceStreams **out)
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FQR_ECUDA;
    DeviceStreams &d = g_dev[dev];
    *out = &d;
    if (d.ready) return FQR_OK;
    if (cudaEventCreateWithFlags(&d.fork, cudaEventDisableTiming) != cudaSuccess) return FQR_ECUDA;
    for (int s = 0; s < kMaxSlots; ++s) {
        if (cudaStreamCreateWithFlags(&d.st[s], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&d.done[s], cudaEventDisableTiming) != cudaSuccess)
            return FQR_ECUDA;
    }
    d.ready = true;
    return FQR_OK;
}

}  // namespace

extern "C" {

size_t fqr_host_workspace_bytes(int64_t batch, int64_t n)
{
    HostPlan p;
    return host_plan(batch, n, &p) ? p.total : 0;
}

int fqr_geqrf_f32_host(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                       int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                       void *workspace, size_t workspace_bytes, void *stream)
{
    if (batch < 0 || n < 0) return FQR_EINVAL;
    if (batch == 0 || n == 0) return FQR_OK;
    if (n > FQR_MAX_N) return FQR_EUNSUPPORTED;
    if (!A || !H || !tau) return FQR_EINVAL;
    // each host matrix must be one dense n x n block (row- or column-major)
    const bool rowmajor = a_rstride == n && a_cstride == 1;
    const bool colmajor = a_rstride == 1 && a_cstride == n;
    if (n > 1 && !rowmajor && !colmajor) return FQR_EINVAL;
    if (batch > 1 && a_bstride < n * n) return FQR_EINVAL;
    HostPlan p;
    if (!host_plan(batch, n, &p)) return FQR_EUNSUPPORTED;
    if (!workspace || workspace_bytes < p.total) return FQR_EWORKSPACE;
    if (((uintptr_t)workspace) % kWsAlign) return FQR_EINVAL;

    DeviceStreams *d = nullptr;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FQR_ECUDA;
    std::lock_guard<std::mutex> lock(g_dev[dev].mu);
    int rc = device_streams(&d);
    if (rc != FQR_OK) return rc;

    cudaStream_t caller = (cudaStream_t)stream;
    unsigned char *ws = (unsigned char *)workspace;
    int *status = (int *)ws;
    const size_t mat_elems = (size_t)n * (size_t)n;
    const size_t mat_bytes = mat_elems * sizeof(float);
    // device copy of a chunk: same per-matrix layout, batch stride n*n
    const int64_t d_rs = colmajor ? 1 : n, d_cs = colmajor ? n : 1;

    if (cudaMemsetAsync(status, 0, p.status_bytes, caller) != cudaSuccess) return FQR_ECUDA;
    if (cudaEventRecord(d->fork, caller) != cudaSuccess) return FQR_ECUDA;
    for (int s = 0; s < p.slots; ++s)
        if (cudaStreamWaitEvent(d->st[s], d->fork, 0) != cudaSuccess) return FQR_ECUDA;

    for (int64_t c = 0; c < p.nchunks; ++c) {
        const int s = (int)(c % p.slots);
        cudaStream_t st = d->st[s];
        const int64_t b0 = c * p.chunk;
        const int64_t cb = (b0 + p.chunk <= batch) ? p.chunk : batch - b0;
        unsigned char *slot = ws + p.status_bytes + (size_t)s * p.slot_bytes;
        float *dA = (float *)(slot + p.off_a);
        float *dH = (float *)(slot + p.off_h);
        float *dT = (float *)(slot + p.off_tau);
        void *dW = p.ws_bytes ? (void *)(slot + p.off_ws) : nullptr;
        const float *hA = A + b0 * a_bstride;
        cudaError_t e;
        if (a_bstride == (int64_t)mat_elems || cb == 1) {
            e = cudaMemcpyAsync(dA, hA, (size_t)cb * mat_bytes, cudaMemcpyHostToDevice, st);
        } else {
            // gapped batch: one strided copy, or one copy per matrix where the
            // pitch is beyond what a strided copy accepts
            e = cudaMemcpy2DAsync(dA, mat_bytes, hA, (size_t)a_bstride * sizeof(float), mat_bytes,
                                  (size_t)cb, cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) {
                cudaGetLastError();
                e = cudaSuccess;
                for (int64_t i = 0; i < cb && e == cudaSuccess; ++i)
                    e = cudaMemcpyAsync(dA + (size_t)i * mat_elems, hA + i * a_bstride, mat_bytes,
                                        cudaMemcpyHostToDevice, st);
            }
        }
        if (e != cudaSuccess) return FQR_ECUDA;
        rc = fqr::geqrf_enqueue_status(dA, cb, n, (int64_t)mat_elems, d_rs, d_cs, dH, dT, dW,
                                       p.ws_bytes, status + c, st);
        if (rc != FQR_OK) return rc;
        if (cudaMemcpyAsync(H + (size_t)b0 * mat_elems, dH, (size_t)cb * mat_bytes,
                            cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(tau + (size_t)b0 * (size_t)n, dT, (size_t)cb * (size_t)n * sizeof(float),
                            cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return FQR_ECUDA;
    }
    for (int s = 0; s < p.slots; ++s) {
        if (cudaEventRecord(d->done[s], d->st[s]) != cudaSuccess ||
            cudaStreamWaitEvent(caller, d->done[s], 0) != cudaSuccess)
            return FQR_ECUDA;
    }
    return FQR_OK;
}

int fqr_host_check_status(const void *workspace, size_t workspace_bytes, int64_t batch, int64_t n,
                          void *stream)
{
    HostPlan p;
    if (!host_plan(batch, n, &p)) return FQR_OK;
    if (!workspace || workspace_bytes < p.total) return FQR_EINVAL;
    int words[kMaxChunks + 1] = {};
    const size_t cnt = (size_t)p.nchunks;
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemcpyAsync(words, workspace, cnt * sizeof(int), cudaMemcpyDeviceToHost, st) !=
        cudaSuccess)
        return FQR_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return FQR_ECUDA;
    for (size_t i = 0; i < cnt; ++i)
        if (words[i]) return FQR_ETIMEOUT;
    return FQR_OK;
}

}  // extern "C"
