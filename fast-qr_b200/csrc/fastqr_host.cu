// fqr_geqrf_f32_host: batched QR of matrices held in HOST memory.
//
// The batch is cut into up to 16 chunks.  Each chunk is copied host->device,
// factored and copied back device->host on its own internal stream with its
// own device staging slot, so that the uploads run back to back while earlier
// chunks are factored and downloaded (the two copy directions use separate
// copy engines).  A call made
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
// The work of a call (copies, kernels, events) is captured once into a CUDA
// graph per distinct argument set and replayed by a single graph launch on
// `stream` afterwards (up to eight graphs per device, least recently used
// replaced); arguments that do not capture, such as pageable host buffers, are
// enqueued directly every time.  A caller that is capturing `stream` itself
// gets the work recorded into its own graph.
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

// Every chunk gets its own staging slot and stream: a slot reused by a later
// chunk would hold that chunk's upload until the earlier chunk's
// factorisation (a per-matrix latency chain of ~0.35 ms at n = 256, whatever
// the chunk's size) and download are done.
constexpr int kMaxSlots = 16;
constexpr int kMaxChunks = 16;
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

// One call's arguments: the key of its cached graph.
struct HostCall {
    const float *A;
    int64_t batch, n, a_bstride, a_rstride, a_cstride;
    float *H, *tau;
    void *workspace;
    size_t workspace_bytes;
    bool operator==(const HostCall &o) const
    {
        return A == o.A && batch == o.batch && n == o.n && a_bstride == o.a_bstride &&
               a_rstride == o.a_rstride && a_cstride == o.a_cstride && H == o.H && tau == o.tau &&
               workspace == o.workspace && workspace_bytes == o.workspace_bytes;
    }
};

// The work of a call is a fixed DAG of copies and kernels for fixed
// arguments; enqueueing it costs ~4.5 us of host time per launch (about 1 ms
// at C2, 4 ms at n = 1024), which the GPU would wait for.  So the DAG is
// captured once into a CUDA graph, cached per device by the call's arguments,
// and replayed with one launch.
constexpr int kGraphCache = 8;
struct CachedGraph {
    bool used = false;
    HostCall key{};
    cudaGraphExec_t exec = nullptr;  // null: these arguments do not capture (enqueue directly)
    uint64_t last = 0;
};

struct DeviceStreams {
    bool ready = false;
    cudaStream_t origin = nullptr;  // root of a captured call
    cudaStream_t st[kMaxSlots] = {};
    cudaEvent_t fork = nullptr;
    cudaEvent_t done[kMaxSlots] = {};
    CachedGraph graphs[kGraphCache];
    uint64_t tick = 0;
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
    if (cudaEventCreateWithFlags(&d.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d.origin, cudaStreamNonBlocking) != cudaSuccess)
        return FQR_ECUDA;
    for (int s = 0; s < kMaxSlots; ++s) {
        if (cudaStreamCreateWithFlags(&d.st[s], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&d.done[s], cudaEventDisableTiming) != cudaSuccess)
            return FQR_ECUDA;
    }
    d.ready = true;
    return FQR_OK;
}

// Enqueue one host-buffer call on the internal streams, forked from and
// joined back into `caller`.
int enqueue_host(const HostCall &c, const HostPlan &p, DeviceStreams *d, cudaStream_t caller)
{
    const float *A = c.A;
    const int64_t batch = c.batch, n = c.n, a_bstride = c.a_bstride;
    float *H = c.H, *tau = c.tau;
    const bool colmajor = c.a_rstride == 1 && c.a_cstride == n && n > 1;
    int rc = FQR_OK;
    unsigned char *ws = (unsigned char *)c.workspace;
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
        // Each chunk is planned as if it ran alone, so its trailing updates
        // split rows over more CTAs to shorten its chain, except for large
        // matrices (n >= 3584, rank-64 plan: one matrix per chunk, whose
        // factorisation outlasts many uploads) when the call's trailing tiles
        // together fill two CTAs per SM (296): those chunks run side by side
        // and are planned for the whole batch, which trades the last chunk's
        // longer chain for the throughput of unsplit tiles.  Measured (ms per
        // call, whole batch / alone): 16 x 4096^2 42.2 / 48.1, 24 x 4096^2
        // 56.9 / 65.0, 10 x 4096^2 32.1 / 33.2; where it lost: 4 x 4096^2
        // 19.4 / 18.7, 16 x 3072^2 27.2 / 24.2, 32 x 2048^2 17.6 / 16.8,
        // 16 x 2048^2 12.1 / 11.0, and C4's rank-32 chunks 8.0 / 7.6.
        const int64_t tiles = (n - fqr::kOuter + 127) / 128;  // trailing tiles of the first rank-64 update
        const int64_t in_flight = fqr::use_outer64(n, n) && n >= 3584 && tiles * batch >= 296 ? batch : cb;
        rc = fqr::geqrf_enqueue_status(dA, cb, n, (int64_t)mat_elems, d_rs, d_cs, dH, dT, dW,
                                       p.ws_bytes, status + c, in_flight, st);
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

    const HostCall call{A, batch, n, a_bstride, a_rstride, a_cstride, H, tau, workspace, workspace_bytes};
    cudaStream_t caller = (cudaStream_t)stream;
    // the caller is capturing a graph itself: record the work into it directly
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(caller, &cs) != cudaSuccess) return FQR_ECUDA;
    if (cs != cudaStreamCaptureStatusNone) return enqueue_host(call, p, d, caller);

    const uint64_t now = ++d->tick;
    for (CachedGraph &g : d->graphs)
        if (g.used && g.key == call) {
            g.last = now;
            if (!g.exec) return enqueue_host(call, p, d, caller);
            return cudaGraphLaunch(g.exec, caller) == cudaSuccess ? FQR_OK : FQR_ECUDA;
        }
    // capture on the internal origin stream (the caller's may be the legacy
    // default stream, which cannot capture); the graph launch then orders the
    // whole DAG after the caller's prior work and before its later work
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    if (cudaStreamBeginCapture(d->origin, cudaStreamCaptureModeRelaxed) == cudaSuccess) {
        const int crc = enqueue_host(call, p, d, d->origin);
        const cudaError_t ec = cudaStreamEndCapture(d->origin, &graph);
        if (crc == FQR_OK && ec == cudaSuccess && graph &&
            cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess)
            exec = nullptr;
        if (graph) cudaGraphDestroy(graph);
    }
    if (!exec) cudaGetLastError();  // not capturable (pageable host memory, say)
    CachedGraph *slot = &d->graphs[0];
    for (CachedGraph &g : d->graphs) {
        if (!g.used) { slot = &g; break; }
        if (g.last < slot->last) slot = &g;
    }
    if (slot->used && slot->exec) cudaGraphExecDestroy(slot->exec);
    slot->used = true;
    slot->key = call;
    slot->exec = exec;
    slot->last = now;
    if (!exec) return enqueue_host(call, p, d, caller);
    return cudaGraphLaunch(exec, caller) == cudaSuccess ? FQR_OK : FQR_ECUDA;
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
