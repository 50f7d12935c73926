// fqr_geqrf_f32_noalloc: the batched QR with no caller-provided workspace
// and no device allocation of any kind.
//
// Who needs it: callers that cannot call cudaMalloc around a call into this
// library.  Examples are a host application that owns the whole device
// memory pool and forbids plugins from allocating, a language binding (JNI,
// cgo, a database extension) whose runtime can pass buffers it already owns
// but has no clean way to create and free a scratch buffer per call, and
// latency-critical loops that cannot afford cudaMalloc/cudaFree, which may
// synchronize the whole device.
//
// How: the only scratch the QR needs (one 32 x 32 S block per matrix on the
// blocked path, n > 64, 64 x 64 for n >= 2048, plus a status block) lives in
// a file-scope __device__ array of fixed size, kNoAllocScratchBytes (16 MiB +
// 256 bytes).  Every GPU
// that loads this library keeps that array until the process exits.  Its
// device address is looked up once per device with cudaGetSymbolAddress, with
// that device current, on the first call made while it is current; make that
// first call before any stream capture begins.  Nothing in the array needs to
// start at zero: every S block is written completely before it is read, and
// the status word is cleared by the first kernel of every call.
//
// Limits: on the blocked path (n > 64) at most FQR_NOALLOC_MAX_BATCH matrices
// per call; larger batches are rejected with FQR_ENOALLOC_LIMIT before any
// work is enqueued.  All calls on one device share the array, and each call
// leaves its last S blocks in it: two calls whose kernels may overlap on the
// GPU (different streams without ordering between them) race on the array and
// give wrong results.  Issue these calls on one stream, or order them.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/fastqr.h"
#include "internal.h"

namespace {

// the largest workspace of a call with up to FQR_NOALLOC_MAX_BATCH matrices
// (64 x 64 S blocks: the rank-64 plan)
constexpr size_t kNoAllocScratchBytes = fqr::ws_total_bytes(FQR_NOALLOC_MAX_BATCH, 4096, 4096);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct ScratchAddr {
    void *ctx = nullptr;  // the CUDA context the address belongs to
    void *addr = nullptr;
};
ScratchAddr g_scratch[kMaxDevices];

// The current CUDA context (cuCtxGetCurrent through the runtime's driver
// entry point query; the library links no libcuda).  A module's __device__
// arrays belong to a context: after cudaDeviceReset, or under another
// context on the same device, the symbol's address may differ.
typedef int (*CtxGetCurrentFn)(void **);
void *current_context()
{
    static std::once_flag once;
    static CtxGetCurrentFn fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
        else
            cudaGetLastError();
    });
    void *ctx = nullptr;
    if (fn && fn(&ctx) != 0) ctx = nullptr;
    return ctx;
}

// Device address of g_noalloc_scratch in the current context, looked up
// once per (device, context).
int scratch_for_current_device(void **out)
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FQR_ECUDA;
    // (no context current yet: the symbol lookup below creates the primary
    // context, and the next call caches the address under it)
    void *ctx = current_context();
    std::lock_guard<std::mutex> lock(g_mu);
    ScratchAddr &s = g_scratch[dev];
    if (!s.addr || s.ctx != ctx || !ctx) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();  // clear the error this call left behind
            s.addr = nullptr;
            return FQR_ECUDA;
        }
        s.addr = p;
        s.ctx = ctx;
    }
    *out = s.addr;
    return FQR_OK;
}

}  // namespace

extern "C" int fqr_geqrf_f32_noalloc(const float *A, int64_t batch, int64_t n, int64_t a_bstride,
                                     int64_t a_rstride, int64_t a_cstride, float *H, float *tau,
                                     void *stream)
{
    if (batch < 0 || n < 0) return FQR_EINVAL;
    if (batch == 0 || n == 0) return FQR_OK;
    if (n > FQR_MAX_N) return FQR_EUNSUPPORTED;
    const size_t need = fqr_workspace_bytes(batch, n);
    // the documented limit (n > 64: at most FQR_NOALLOC_MAX_BATCH matrices),
    // whatever the plan's S block size
    if (need > 0 && batch > FQR_NOALLOC_MAX_BATCH) return FQR_ENOALLOC_LIMIT;
    if (need > kNoAllocScratchBytes) return FQR_ENOALLOC_LIMIT;
    void *scratch = nullptr;
    if (need > 0) {
        const int rc = scratch_for_current_device(&scratch);
        if (rc != FQR_OK) return rc;
    }
    return fqr::geqrf_enqueue(A, batch, n, a_bstride, a_rstride, a_cstride, H, tau, scratch,
                              need > 0 ? kNoAllocScratchBytes : 0, (cudaStream_t)stream);
}

extern "C" int fqr_noalloc_check_status(void *stream)
{
    // the status block is the first 256 bytes of the static array: one int
    // word per part of a batch split over streams, all cleared by every call
    int v[4] = {};
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemcpyFromSymbolAsync(v, g_noalloc_scratch, sizeof(v), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return FQR_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return FQR_ECUDA;
    int any = 0;
    for (int i = 0; i < 4; ++i) any |= v[i];
    return any ? FQR_ETIMEOUT : FQR_OK;
}
