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
// leaves its last T factors in it: two calls whose kernels may overlap on the
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
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_for_current_device(void **out)
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FQR_ECUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();  // clear the error this call left behind
            return FQR_ECUDA;
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
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
