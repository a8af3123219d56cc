// Decode attention with its scratch in a fixed device array of this module.
//
// qv_decode_attention takes a caller-provided workspace.  Some callers cannot
// provide one: host code that drives the layer through the C ABI from another
// language runtime and holds only the layer's own device pointers, with no
// device allocator of its own to call; and serving loops that must not call
// cudaMalloc/cudaFree between decode steps, because cudaFree waits for the
// whole device and a fresh allocation can fail under memory pressure in the
// middle of a step.  This entry point needs no workspace: the scratch is a
// file-scope device array of QV_NOALLOC_SCRATCH_BYTES, and the call neither
// allocates nor frees device memory.
//
// The array is shared by every call on a device, so calls that overlap in
// time (on two streams, or from two host threads without ordering between
// their streams) race on it and give wrong results.  The first call on each
// device looks up the array's address (cudaGetSymbolAddress, which may
// initialise the module on that device); make that first call before any
// stream capture or latency-critical loop begins.  The address is cached per
// device together with the CUDA context it was looked up in; a call made in
// another context (after cudaDeviceReset, or once the primary context has
// been torn down and created again) looks it up afresh.
//
// Like qv_decode_attention, the call is launched as a programmatic dependent:
// it reads the slot tables and cached K/V before the preceding kernel on the
// stream has finished, so it must directly follow qv_rope_append on the same
// stream, or a kernel that writes none of the layer's state.
#include <cudaTypedefs.h>
#include <mutex>
#include <stdio.h>

#include "common.cuh"

namespace qv {

static __device__ __align__(256) unsigned char g_decode_scratch[QV_NOALLOC_SCRATCH_BYTES];

static constexpr int kMaxDevices = 64;
static void* g_scratch_addr[kMaxDevices];
static CUcontext g_scratch_ctx[kMaxDevices];
static std::mutex g_scratch_mu;

static PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
    static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    }
    return fn;
}

// Address of g_decode_scratch on the current device, looked up once per
// device and context.
static int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_cuda_error(e);
    if (dev < 0 || dev >= kMaxDevices) return QV_EINVAL;
    auto get = ctx_get_current();
    if (!get) return QV_ECUDA;
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return QV_ECUDA;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!ctx || !g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
        // the lookup makes the device's primary context current if no context was
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return set_cuda_error(e);
        if (get(&ctx) != CUDA_SUCCESS || !ctx) return QV_ECUDA;
        g_scratch_addr[dev] = p;
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_addr[dev];
    return QV_OK;
}

int set_error_text(const char* msg);

}  // namespace qv

using namespace qv;

extern "C" int qv_decode_attention_noalloc(const qv_dims* d, const qv_layer* L, const void* q, void* out,
                                           qv_stream_t stream) {
    int rc = validate_dims(d);
    if (rc) return rc;
    if (!L || !q || !out) return QV_EINVAL;
    const size_t need = qv_decode_workspace_bytes(d);
    if (need == 0) return QV_EINVAL;
    if (need > (size_t)QV_NOALLOC_SCRATCH_BYTES) {
        char msg[200];
        snprintf(msg, sizeof(msg),
                 "qv_decode_attention_noalloc: these dims need %zu bytes of scratch, the static scratch holds %zu; "
                 "use qv_decode_attention with a workspace",
                 need, (size_t)QV_NOALLOC_SCRATCH_BYTES);
        set_error_text(msg);
        return QV_ESPACE;
    }
    void* scratch = nullptr;
    rc = scratch_address(&scratch);
    if (rc) return rc;
    // the split counters at the front of the scratch must be zero when the
    // attention kernels start; they leave them zero on a normal exit, and
    // this clear also covers a previous call that ended with an error
    const size_t tickets = ((size_t)d->batch * d->kv_heads + 1) * sizeof(int);
    cudaError_t e = cudaMemsetAsync(scratch, 0, tickets, (cudaStream_t)stream);
    if (e != cudaSuccess) return set_cuda_error(e);
    return qv_decode_attention(d, L, q, out, scratch, QV_NOALLOC_SCRATCH_BYTES, stream);
}
