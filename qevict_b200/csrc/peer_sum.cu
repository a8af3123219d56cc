// One-shot sum of a small bf16 vector across the GPUs of one node, over NVLink
// peer memory: the all-reduce of the KV-head-parallel decode (the row-parallel
// o_proj / down-projection partials, [batch, hidden] per layer).
//
// At decode batch 1 that vector is 8 KB, and a ring or tree all-reduce pays
// several dependent link crossings and a library launch for it.  Here each
// rank's buffer (cudaMalloc'd once, mapped into every other rank's process
// with CUDA IPC) holds one slot per source rank, and one CTA per call
//   1. stores this rank's vector into its slot of every rank's buffer as
//      8-byte words that carry 4 bytes of data and the low 32 bits of the
//      call's epoch (plain peer stores, no multicast): an aligned 8-byte
//      store is seen whole, so a reader that finds the epoch in a word also
//      finds its data -- no fence and no separate flag (the "low latency"
//      word format of NCCL's LL protocol);
//   2. reads its own buffer's slots in rank order, waiting (bounded) on each
//      word until it carries the epoch, and sums in fp32 with one rounding to
//      bf16, so every rank computes the same bits.
// Slots are double-buffered by epoch parity: a rank writes epoch e+2 (the
// next use of a parity) only after reading every rank's epoch-e+1 words,
// which each rank writes only after its reads of epoch e.  The epoch counter
// lives on the device, so the kernel replays unchanged inside a CUDA graph.
// A wait that gives up (about 5 s) sets the error word and goes on; the
// result of that call is not valid (qv_peer_sum_read_error).
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "ptx.cuh"

namespace qv {

constexpr int PS_MAXW = 8;
constexpr int PS_THREADS = 512;

struct PsArgs {
    unsigned char* data[PS_MAXW];      // every rank's slot area, mapped here
    unsigned char* my_data;
    unsigned long long* epoch;         // this rank's call counter
    int* err;
    int rank, world;
    long long slot_bytes;              // bytes of one slot: 8-byte words for 2 * max_bytes, 256-aligned
};

__device__ __forceinline__ void ps_store_word(unsigned char* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ps_load_word(const unsigned char* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The data half of this rank's slot-q word at wp once it carries the epoch
// (bounded: after about 5 s the error word is raised and later waits of the
// call are skipped).
__device__ __forceinline__ uint32_t ps_wait_word(const unsigned char* wp, unsigned long long tag, bool& timed_out,
                                                 int* err) {
    unsigned long long w = ps_load_word(wp);
    if ((w & 0xFFFFFFFF00000000ull) != tag && !timed_out) {
        const uint64_t t0 = global_ns();
        while ((w & 0xFFFFFFFF00000000ull) != tag) {
            w = ps_load_word(wp);
            if (global_ns() - t0 > 5000000000ull) {
                atomicOr(err, QV_DERR_TIMEOUT);
                timed_out = true;
                break;
            }
        }
    }
    return (uint32_t)w;
}

// MAX64 = false: nw words = bf16 pairs, summed.  MAX64 = true: nw / 2 int64
// values (low word first), their maximum.
template <bool MAX64>
__global__ void __launch_bounds__(PS_THREADS) peer_sum_kernel(PsArgs a, const uint32_t* __restrict__ in,
                                                              uint32_t* __restrict__ out, int nw) {
    __shared__ unsigned long long s_epoch;
    // a programmatic dependent: `in` is written by the preceding kernel; the
    // kernel after this one may be scheduled now (it waits for this grid
    // before reading the result)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) s_epoch = *a.epoch + 1;
    __syncthreads();
    const unsigned long long e = s_epoch;
    const unsigned long long tag = (e & 0xFFFFFFFFull) << 32;
    const int par = (int)(e & 1);
    const size_t slot_off = ((size_t)par * a.world + a.rank) * (size_t)a.slot_bytes;
    // 1. this rank's words into its slot at every rank (itself included)
    for (int i = threadIdx.x; i < nw; i += blockDim.x) {
        const unsigned long long w = tag | in[i];
        for (int p = 0; p < a.world; ++p) ps_store_word(a.data[p] + slot_off + 8 * (size_t)i, w);
    }
    // 2. every rank's words of this epoch, reduced in rank order
    const unsigned char* base = a.my_data + (size_t)par * a.world * (size_t)a.slot_bytes;
    bool timed_out = false;
    if (!MAX64) {
        for (int i = threadIdx.x; i < nw; i += blockDim.x) {
            float lo = 0.f, hi = 0.f;
            for (int q = 0; q < a.world; ++q) {
                const uint32_t d = ps_wait_word(base + (size_t)q * a.slot_bytes + 8 * (size_t)i, tag, timed_out, a.err);
                lo += __uint_as_float(d << 16);
                hi += __uint_as_float(d & 0xFFFF0000u);
            }
            const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
            out[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
    } else {
        for (int j = threadIdx.x; j < nw / 2; j += blockDim.x) {
            long long best = 0;
            for (int q = 0; q < a.world; ++q) {
                const unsigned char* wp = base + (size_t)q * a.slot_bytes + 16 * (size_t)j;
                const uint32_t lo = ps_wait_word(wp, tag, timed_out, a.err);
                const uint32_t hi = ps_wait_word(wp + 8, tag, timed_out, a.err);
                const long long v = (long long)(((unsigned long long)hi << 32) | lo);
                best = q == 0 || v > best ? v : best;
            }
            out[2 * j] = (uint32_t)best;
            out[2 * j + 1] = (uint32_t)((unsigned long long)best >> 32);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *a.epoch = e;
}

}  // namespace qv

using namespace qv;

static_assert(sizeof(cudaIpcMemHandle_t) == QV_PEER_HANDLE_BYTES, "IPC handle size");

struct qv_peer_sum {
    int rank, world;
    size_t slot_bytes, total;
    unsigned char* base;                 // this rank's allocation
    unsigned char* peer[PS_MAXW];        // mapped bases (own base at [rank])
    bool opened;
};

static size_t ps_al(size_t x) { return (x + 255) & ~(size_t)255; }
// [2 parities][world slots][slot_bytes] | epoch u64 | err int
static size_t ps_epoch_off(const qv_peer_sum* p) { return 2 * (size_t)p->world * p->slot_bytes; }
static size_t ps_err_off(const qv_peer_sum* p) { return ps_epoch_off(p) + 256; }

extern "C" int qv_peer_sum_create(int32_t rank, int32_t world, size_t max_bytes, qv_peer_sum** out,
                                  void* handle) {
    if (!out || !handle || world < 1 || world > PS_MAXW || rank < 0 || rank >= world || max_bytes == 0 ||
        max_bytes % 16)
        return QV_EINVAL;
    qv_peer_sum* p = new qv_peer_sum();
    p->rank = rank;
    p->world = world;
    p->slot_bytes = ps_al(2 * max_bytes);
    p->total = ps_err_off(p) + 256;
    p->opened = false;
    cudaError_t e = cudaMalloc(&p->base, p->total);
    if (e == cudaSuccess) e = cudaMemset(p->base, 0, p->total);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p->base);
    if (e != cudaSuccess) {
        if (p->base) cudaFree(p->base);
        delete p;
        return set_cuda_error(e);
    }
    memcpy(handle, &h, sizeof(h));
    for (int i = 0; i < PS_MAXW; ++i) p->peer[i] = nullptr;
    p->peer[rank] = p->base;
    *out = p;
    return QV_OK;
}

extern "C" int qv_peer_sum_open(qv_peer_sum* p, const void* handles) {
    if (!p || !handles || p->opened) return QV_EINVAL;
    for (int r = 0; r < p->world; ++r) {
        if (r == p->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + (size_t)r * QV_PEER_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != p->rank && p->peer[q]) { cudaIpcCloseMemHandle(p->peer[q]); p->peer[q] = nullptr; }
            return set_cuda_error(e);
        }
        p->peer[r] = static_cast<unsigned char*>(ptr);
    }
    p->opened = true;
    return QV_OK;
}

static PsArgs ps_args(const qv_peer_sum* p) {
    PsArgs a;
    for (int r = 0; r < PS_MAXW; ++r) a.data[r] = r < p->world ? p->peer[r] : nullptr;
    a.my_data = p->base;
    a.epoch = reinterpret_cast<unsigned long long*>(p->base + ps_epoch_off(p));
    a.err = reinterpret_cast<int*>(p->base + ps_err_off(p));
    a.rank = p->rank;
    a.world = p->world;
    a.slot_bytes = (long long)p->slot_bytes;
    return a;
}

extern "C" int qv_peer_sum_bf16(qv_peer_sum* p, const void* in, void* out, int64_t n, qv_stream_t stream) {
    if (!p || !p->opened || !in || !out || n <= 0 || n % 8 || (size_t)n * 4 > p->slot_bytes) return QV_EINVAL;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) return QV_EINVAL;
    PsArgs a = ps_args(p);
    cudaError_t e = launch_pdl(peer_sum_kernel<false>, dim3(1), dim3(PS_THREADS), 0, (cudaStream_t)stream, a,
                               static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out), (int)(n / 2));
    return e == cudaSuccess ? QV_OK : set_cuda_error(e);
}

extern "C" int qv_peer_max_i64(qv_peer_sum* p, const int64_t* in, int64_t* out, int64_t n, qv_stream_t stream) {
    if (!p || !p->opened || !in || !out || n <= 0 || (size_t)n * 16 > p->slot_bytes) return QV_EINVAL;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 7) return QV_EINVAL;
    PsArgs a = ps_args(p);
    cudaError_t e = launch_pdl(peer_sum_kernel<true>, dim3(1), dim3(PS_THREADS), 0, (cudaStream_t)stream, a,
                               reinterpret_cast<const uint32_t*>(in), reinterpret_cast<uint32_t*>(out), (int)(2 * n));
    return e == cudaSuccess ? QV_OK : set_cuda_error(e);
}

extern "C" int qv_peer_sum_read_error(qv_peer_sum* p, int32_t* host_err, qv_stream_t stream) {
    if (!p || !host_err) return QV_EINVAL;
    cudaError_t e = cudaMemcpyAsync(host_err, p->base + ps_err_off(p), sizeof(int32_t), cudaMemcpyDeviceToHost,
                                    (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    return e == cudaSuccess ? QV_OK : set_cuda_error(e);
}

extern "C" int qv_peer_sum_destroy(qv_peer_sum* p) {
    if (!p) return QV_EINVAL;
    cudaError_t first = cudaSuccess;
    for (int r = 0; r < p->world; ++r) {
        if (r == p->rank || !p->peer[r]) continue;
        cudaError_t e = cudaIpcCloseMemHandle(p->peer[r]);
        if (first == cudaSuccess) first = e;
    }
    cudaError_t e = cudaFree(p->base);
    if (first == cudaSuccess) first = e;
    delete p;
    return first == cudaSuccess ? QV_OK : set_cuda_error(first);
}
