// Elementwise steps of the full-model decode driver, fused so that a decode
// step launches fewer small kernels between the cuBLAS projections:
//
//   qv_add_rmsnorm   x = x + delta (rounded to bf16), h = RMSNorm(x) * w
//                    (the residual add after a projection and the norm before
//                    the next one, one kernel instead of two)
//   qv_silu_mul      out = SiLU(g) * u of a [g | u] row (the MLP activation,
//                    one kernel instead of two)
//   qv_argmax        greedy token of each logit row in one launch
//
// bf16 in and out, fp32 arithmetic, rounded where the separate torch ops
// round (the sum, SiLU(g), the product, the norm output).  One CTA per token
// row for the norm (16-byte vector loads, block-wide sum of squares).
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace qv {

constexpr int MO_THREADS = 512;

__device__ __forceinline__ float mo_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float mo_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ uint32_t mo_pack(float a, float b) {
    const __nv_bfloat162 x = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&x);
}

__global__ void __launch_bounds__(MO_THREADS) add_rmsnorm_kernel(int K, __nv_bfloat16* __restrict__ x,
                                                                 const __nv_bfloat16* __restrict__ delta,
                                                                 const __nv_bfloat16* __restrict__ w, float eps,
                                                                 __nv_bfloat16* __restrict__ h) {
    __shared__ float red[MO_THREADS / 32];
    // the next projection (launched as a programmatic dependent) may start
    // streaming its weights now; it waits for this grid before reading h
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int b = blockIdx.x;
    uint4* xr = reinterpret_cast<uint4*>(x + (size_t)b * K);
    const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + (size_t)b * K) : nullptr;
    const int n8 = K / 8;
    constexpr int PER = 4;   // 8-element chunks per thread (K <= 8 * 4 * 512)
    uint4 xv[PER];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int c = threadIdx.x + i * MO_THREADS;
        if (c < n8) {
            uint4 v = xr[c];
            if (dr) {
                const uint4 d = dr[c];
                const uint32_t* a = reinterpret_cast<const uint32_t*>(&v);
                const uint32_t* e = reinterpret_cast<const uint32_t*>(&d);
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) o[j] = mo_pack(mo_lo(a[j]) + mo_lo(e[j]), mo_hi(a[j]) + mo_hi(e[j]));
                v = make_uint4(o[0], o[1], o[2], o[3]);
                xr[c] = v;
            }
            const uint32_t* a = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ss = fmaf(mo_lo(a[j]), mo_lo(a[j]), ss);
                ss = fmaf(mo_hi(a[j]), mo_hi(a[j]), ss);
            }
            xv[i] = v;
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < MO_THREADS / 32; ++i) t += red[i];
    const float r = rsqrtf(t / (float)K + eps);
    uint4* hr = reinterpret_cast<uint4*>(h + (size_t)b * K);
    const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int c = threadIdx.x + i * MO_THREADS;
        if (c < n8) {
            const uint4 wv = wr[c];
            const uint32_t* a = reinterpret_cast<const uint32_t*>(&xv[i]);
            const uint32_t* e = reinterpret_cast<const uint32_t*>(&wv);
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                o[j] = mo_pack(mo_lo(a[j]) * r * mo_lo(e[j]), mo_hi(a[j]) * r * mo_hi(e[j]));
            hr[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

__global__ void __launch_bounds__(256) silu_mul_kernel(int F, int rows, const __nv_bfloat16* __restrict__ gu,
                                                       __nv_bfloat16* __restrict__ out) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int n8 = F / 8;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * n8) return;
    const int b = idx / n8, c = idx % n8;
    const uint4 gv = reinterpret_cast<const uint4*>(gu + (size_t)b * 2 * F)[c];
    const uint4 uv = reinterpret_cast<const uint4*>(gu + (size_t)b * 2 * F + F)[c];
    const uint32_t* g = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&uv);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float g0 = mo_lo(g[j]), g1 = mo_hi(g[j]);
        const float s0 = __bfloat162float(__float2bfloat16_rn(g0 / (1.f + expf(-g0))));
        const float s1 = __bfloat162float(__float2bfloat16_rn(g1 / (1.f + expf(-g1))));
        o[j] = mo_pack(s0 * mo_lo(u[j]), s1 * mo_hi(u[j]));
    }
    reinterpret_cast<uint4*>(out + (size_t)b * F)[c] = make_uint4(o[0], o[1], o[2], o[3]);
}

// Greedy argmax of bf16 rows: blocks reduce slices of a row to (value, index),
// then one 64-bit atomicMax per block on a key that orders by value and, among
// equal values, by the smaller index; the last block of the row writes the
// index and resets the row's key and ticket.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    const uint32_t b = v == 0.f ? 0u : __float_as_uint(v);   // -0 ties with +0
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (uint32_t)(0x7fffffff - i);
}

__global__ void __launch_bounds__(256) argmax_kernel(int cols, const __nv_bfloat16* __restrict__ x,
                                                     unsigned long long* keys, int* tickets, int64_t* out) {
    const int b = blockIdx.y;
    const int per = (cols + gridDim.x - 1) / gridDim.x;
    const int c0 = blockIdx.x * per, c1 = min(c0 + per, cols);
    const __nv_bfloat16* row = x + (size_t)b * cols;
    unsigned long long best = 0ull;
    for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
        const unsigned long long k = argmax_key(__bfloat162float(row[c]), c);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    __shared__ unsigned long long red[8];
    __shared__ bool last;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        best = red[0] > best ? red[0] : best;
        atomicMax(keys + b, best);
        __threadfence();
        last = atomicAdd(tickets + b, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const unsigned long long k = atomicExch(keys + b, 0ull);
        out[b] = (int64_t)(0x7fffffff - (int)(uint32_t)(k & 0xffffffffull));
        tickets[b] = 0;
    }
}

}  // namespace qv

using namespace qv;

extern "C" size_t qv_argmax_workspace_bytes(int32_t rows) {
    return rows > 0 ? (size_t)rows * 16 : 0;
}

extern "C" int qv_argmax(int32_t rows, int32_t cols, const void* x, int64_t* out, void* workspace,
                         size_t workspace_bytes, qv_stream_t stream) {
    if (rows <= 0 || cols <= 0 || !x || !out || !workspace) return QV_EINVAL;
    if (workspace_bytes < qv_argmax_workspace_bytes(rows)) return QV_ESPACE;
    unsigned long long* keys = static_cast<unsigned long long*>(workspace);
    int* tickets = reinterpret_cast<int*>(keys + rows);
    int blocks = (cols + 2047) / 2048;
    if (blocks > 148) blocks = 148;
    argmax_kernel<<<dim3(blocks, rows), 256, 0, (cudaStream_t)stream>>>(cols, static_cast<const __nv_bfloat16*>(x),
                                                                         keys, tickets, out);
    return check_launch();
}

static bool mo_aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int qv_add_rmsnorm(int32_t rows, int32_t cols, void* x, const void* delta, const void* weight, float eps,
                              void* h_out, qv_stream_t stream) {
    if (rows <= 0 || cols <= 0 || cols % 8 || cols > 8 * 4 * MO_THREADS || !x || !weight || !h_out) return QV_EINVAL;
    if (!mo_aligned(x) || !mo_aligned(weight) || !mo_aligned(h_out) || (delta && !mo_aligned(delta))) return QV_EINVAL;
    add_rmsnorm_kernel<<<rows, MO_THREADS, 0, (cudaStream_t)stream>>>(
        cols, static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(delta),
        static_cast<const __nv_bfloat16*>(weight), eps, static_cast<__nv_bfloat16*>(h_out));
    return check_launch();
}

extern "C" int qv_silu_mul(int32_t rows, int32_t cols, const void* gate_up, void* out, qv_stream_t stream) {
    if (rows <= 0 || cols <= 0 || cols % 8 || !gate_up || !out) return QV_EINVAL;
    if (!mo_aligned(gate_up) || !mo_aligned(out)) return QV_EINVAL;
    const int n = rows * (cols / 8);
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(cols, rows, static_cast<const __nv_bfloat16*>(gate_up),
                                                                      static_cast<__nv_bfloat16*>(out));
    return check_launch();
}
