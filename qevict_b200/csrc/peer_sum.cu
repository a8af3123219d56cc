// One-shot sum of a small bf16 vector across the GPUs of one node, over NVLink
// peer memory: the all-reduce of the KV-head-parallel decode (the row-parallel
// o_proj / down-projection partials, [batch, hidden] per layer).
//
// At decode batch 1 that vector is 8 KB, and a ring or tree all-reduce pays
// several dependent link crossings and a library launch for it.  Here each
// rank's buffer (cudaMalloc'd once, mapped into every other rank's process
// with CUDA IPC) holds one slot per source rank; one CTA per call
//   1. stores this rank's vector into its slot of every rank's buffer
//      (plain 16-byte peer stores, no multicast),
//   2. fences at system scope and publishes the call's epoch in a per-source
//      flag of every rank's buffer (st.release.sys),
//   3. waits (bounded) until every rank's flag in its own buffer has reached
//      the epoch (ld.acquire.sys), and
//   4. sums the slots in rank order in fp32 and rounds once to bf16, so every
//      rank computes the same bits.
// Slots are double-buffered by epoch parity: a rank can only reach epoch e+2
// (the next use of a parity) after every rank has published e+1, which each
// does only after finishing its reads of epoch e.  The epoch counter lives on
// the device, so the kernel replays unchanged inside a CUDA graph.  A wait
// that gives up (about 5 s) sets the error word and returns; the result of
// that call is not valid (qv_peer_sum_read_error).
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
    unsigned long long* flags[PS_MAXW];  // every rank's per-source flags, mapped here
    unsigned char* my_data;
    unsigned long long* my_flags;
    unsigned long long* epoch;         // this rank's call counter
    int* err;
    int rank, world;
    long long slot_bytes;              // bytes of one slot (max_bytes, 256-aligned)
};

__device__ __forceinline__ void ps_store_release(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ps_load_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(PS_THREADS) peer_sum_kernel(PsArgs a, const uint4* __restrict__ in,
                                                              uint4* __restrict__ out, int nvec) {
    __shared__ unsigned long long s_epoch;
    // a programmatic dependent: `in` is written by the preceding kernel; the
    // kernel after this one may be scheduled now (it waits for this grid
    // before reading the sum)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) s_epoch = *a.epoch + 1;
    __syncthreads();
    const unsigned long long e = s_epoch;
    const int par = (int)(e & 1);
    const size_t slot_off = ((size_t)par * a.world + a.rank) * (size_t)a.slot_bytes;
    // 1. this rank's vector into its slot at every rank (itself included)
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
        const uint4 v = in[i];
        for (int p = 0; p < a.world; ++p) reinterpret_cast<uint4*>(a.data[p] + slot_off)[i] = v;
    }
    // 2. the stores reach every rank before the flag that announces them
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.world) ps_store_release(a.flags[threadIdx.x] + a.rank, e);
    // 3. every rank's vector of this epoch is in this rank's buffer
    if (threadIdx.x < a.world) {
        const unsigned long long* f = a.my_flags + threadIdx.x;
        if (ps_load_acquire(f) < e) {
            const uint64_t t0 = global_ns();
            while (ps_load_acquire(f) < e) {
                if (global_ns() - t0 > 5000000000ull) {
                    atomicOr(a.err, QV_DERR_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
    // 4. the sum in rank order (L1 bypassed: peers wrote this memory)
    const uint4* base = reinterpret_cast<const uint4*>(a.my_data + (size_t)par * a.world * (size_t)a.slot_bytes);
    const size_t sv = (size_t)a.slot_bytes / 16;
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < a.world; ++q) {
            const uint4 v = __ldcg(base + (size_t)q * sv + i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc[2 * k] += __uint_as_float(w[k] << 16);
                acc[2 * k + 1] += __uint_as_float(w[k] & 0xFFFF0000u);
            }
        }
        uint32_t r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
            r[k] = *reinterpret_cast<const uint32_t*>(&h);
        }
        out[i] = make_uint4(r[0], r[1], r[2], r[3]);
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
// [2 parities][world slots][slot_bytes] | flags [world] u64 | epoch u64 | err int
static size_t ps_flags_off(const qv_peer_sum* p) { return 2 * (size_t)p->world * p->slot_bytes; }
static size_t ps_epoch_off(const qv_peer_sum* p) { return ps_flags_off(p) + ps_al((size_t)p->world * 8); }
static size_t ps_err_off(const qv_peer_sum* p) { return ps_epoch_off(p) + 256; }

extern "C" int qv_peer_sum_create(int32_t rank, int32_t world, size_t max_bytes, qv_peer_sum** out,
                                  void* handle) {
    if (!out || !handle || world < 1 || world > PS_MAXW || rank < 0 || rank >= world || max_bytes == 0 ||
        max_bytes % 16)
        return QV_EINVAL;
    qv_peer_sum* p = new qv_peer_sum();
    p->rank = rank;
    p->world = world;
    p->slot_bytes = ps_al(max_bytes);
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

extern "C" int qv_peer_sum_bf16(qv_peer_sum* p, const void* in, void* out, int64_t n, qv_stream_t stream) {
    if (!p || !p->opened || !in || !out || n <= 0 || n % 8 || (size_t)n * 2 > p->slot_bytes) return QV_EINVAL;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) return QV_EINVAL;
    PsArgs a;
    for (int r = 0; r < PS_MAXW; ++r) {
        a.data[r] = r < p->world ? p->peer[r] : nullptr;
        a.flags[r] = r < p->world ? reinterpret_cast<unsigned long long*>(p->peer[r] + ps_flags_off(p)) : nullptr;
    }
    a.my_data = p->base;
    a.my_flags = reinterpret_cast<unsigned long long*>(p->base + ps_flags_off(p));
    a.epoch = reinterpret_cast<unsigned long long*>(p->base + ps_epoch_off(p));
    a.err = reinterpret_cast<int*>(p->base + ps_err_off(p));
    a.rank = p->rank;
    a.world = p->world;
    a.slot_bytes = (long long)p->slot_bytes;
    cudaError_t e = launch_pdl(peer_sum_kernel, dim3(1), dim3(PS_THREADS), 0, (cudaStream_t)stream, a,
                               static_cast<const uint4*>(in), static_cast<uint4*>(out), (int)(n / 8));
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
