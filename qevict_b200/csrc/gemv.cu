// Weight-streaming GEMV of the full-model decode driver: y[b] = W . x[b] for
// a bf16 nn.Linear weight W [N][K] (row-major) and a handful of token rows x.
//
// At decode batch 1-8 a projection is a pure HBM stream of W.  Two layouts of
// the work, chosen by the row length:
//
// Rows (K <= 8192): one warp per output row at a time, 16-byte loads (8
// weights per lane), groups of U loads per lane (U KiB per warp)
// double-buffered in registers, so the next group is in flight while the
// current one is multiplied; a persistent grid sized by occupancy; each warp
// walks its rows and its groups as one stream, so the loads of the next row
// start before the current row is reduced.  U = 2 when the resident warps
// cover every row at once (one row per warp, the smallest registers), else
// U = 4 (more bytes in flight per warp).  Measured on B200 against cuBLAS back
// to back at the Llama-3-8B projection shapes: qkv 11.7 vs 15.6 us, output
// 9.2 vs 15.4, gate/up 38.7 vs 42.1, LM head 152 vs 163.
//
// K-slices (K > 8192, the MLP down projection): with rows of 28 KiB and only
// N = 4096 of them, one row per warp leaves the SMs unevenly loaded (3-4 CTAs
// each) and too few bytes in flight.  Instead each CTA (8 warps, as many per
// SM as fit) owns an equal contiguous range of rows, warp w takes K-slice w of
// every one of them, and the eight partial dot products of a row meet in
// shared memory and are added in warp order; loads are grouped U at a time
// and double-buffered like the row layout (a group is consumed as a whole, so
// its loads share one scoreboard).  Down projection: 23.7 us vs 26.1 for the
// row layout.
//
// Both: weights bypass L1 (read once; an L2 evict-first policy on them was
// measured: no gain); x (tiny, shared by every warp) is read through L1; the
// kernel is a programmatic dependent of the one before it, issues its first
// weight loads before griddepcontrol.wait (W does not depend on that kernel)
// and reads x after it.  fp32 accumulation, one rounding to bf16 per output
// (as a bf16 GEMM with fp32 compute rounds).
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace qv {

constexpr int GV_THREADS = 256;
constexpr int GV_WARPS = GV_THREADS / 32;
constexpr int GV_MAXB = 8;              // token rows
constexpr int GV_PASS = 32;             // K-slices: rows whose partials are held in shared memory at a time
constexpr int GV_KSPLIT_MIN_K = 8192;   // K above which the K-slice layout is used

__device__ __forceinline__ uint4 ld_stream16(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float gv_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float gv_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Row layout (see the top of this file).
template <int NB, int GV_U>
__global__ void __launch_bounds__(GV_THREADS) gemv_rows_kernel(int N, int K, const __nv_bfloat16* __restrict__ W,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          __nv_bfloat16* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = K >> 3;                              // 16-byte chunks per row
    const int gpr = (nc + 32 * GV_U - 1) / (32 * GV_U);  // groups per row
    const int r0 = blockIdx.x * (GV_THREADS / 32) + warp;
    const int stride = gridDim.x * (GV_THREADS / 32);
    const int nrows = r0 < N ? (N - r0 + stride - 1) / stride : 0;
    const int T = nrows * gpr;                          // this warp's groups
    uint4 wa[GV_U], wb[GV_U];

    auto load = [&](uint4* w, int t) {
        const int row = r0 + (t / gpr) * stride;
        const int c0 = (t % gpr) * 32 * GV_U + lane;
        const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)row * K);
#pragma unroll
        for (int u = 0; u < GV_U; ++u) {
            const int c = c0 + 32 * u;
            w[u] = (t < T && c < nc) ? ld_stream16(wr + c) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    auto compute = [&](const uint4* w, int t) {
        const int row = r0 + (t / gpr) * stride;
        const int grp = t % gpr;
        const int c0 = grp * 32 * GV_U + lane;
#pragma unroll
        for (int u = 0; u < GV_U; ++u) {
            const int c = c0 + 32 * u;
            if (c < nc) {
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(&w[u]);
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)b * K) + c);
                    const uint32_t* xp = reinterpret_cast<const uint32_t*>(&xv);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[b] = fmaf(gv_lo(wp[j]), gv_lo(xp[j]), acc[b]);
                        acc[b] = fmaf(gv_hi(wp[j]), gv_hi(xp[j]), acc[b]);
                    }
                }
            }
        }
        if (grp == gpr - 1) {   // the row is complete: reduce and store
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float s = warp_sum(acc[b]);
                if (lane == 0) y[(size_t)b * N + row] = __float2bfloat16_rn(s);
                acc[b] = 0.f;
            }
        }
    };

    load(wa, 0);
    // x is written by the preceding kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#pragma unroll 1
    for (int t = 0; t < T; t += 2) {
        load(wb, t + 1);
        compute(wa, t);
        if (t + 1 >= T) break;
        load(wa, t + 2);
        compute(wb, t + 1);
    }
}

// K-slice layout (see the top of this file).  CTA c owns rows
// [c*N/grid, (c+1)*N/grid); warp w of the CTA owns chunks [w*cs, (w+1)*cs) of
// each of them.
template <int NB, int U>
__global__ void __launch_bounds__(GV_THREADS, NB <= 2 ? 4 : 2)
gemv_ksplit_kernel(int N, int K, const __nv_bfloat16* __restrict__ W, const __nv_bfloat16* __restrict__ x,
                   __nv_bfloat16* __restrict__ y) {
    __shared__ float part[GV_PASS][GV_WARPS][NB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = K >> 3;                                   // 16-byte chunks per row
    const int cs = (nc + GV_WARPS - 1) / GV_WARPS;           // chunks of this warp's slice
    const int cpl = (cs + 31) >> 5;                          // chunks per lane per row slice
    const int c_lo = warp * cs;
    const int c_hi = min(c_lo + cs, nc);
    const int row0 = (int)((long long)blockIdx.x * N / gridDim.x);
    const int nrows = (int)((long long)(blockIdx.x + 1) * N / gridDim.x) - row0;
    // this warp's chunks, in order: row r = 0..nrows-1, then i = 0..cpl-1 within
    // the row's slice (chunk c_lo + lane + 32 i); loaded U at a time into one of
    // two register buffers, each buffer consumed as a whole (so a buffer's loads
    // share one scoreboard and the two buffers alternate)
    const int n_groups = (nrows * cpl + U - 1) / U;
    const uint4* __restrict__ wbase = reinterpret_cast<const uint4*>(W) + (size_t)row0 * nc;
    int lr = 0, li = 0;                                      // load cursor: row, chunk of the slice
    auto load_group = [&](uint4* buf) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c_lo + lane + 32 * li;
            buf[u] = (lr < nrows && c < c_hi) ? ld_stream16(wbase + (size_t)lr * nc + c) : make_uint4(0u, 0u, 0u, 0u);
            if (++li == cpl) { li = 0; ++lr; }
        }
    };
    uint4 bufA[U], bufB[U];
    load_group(bufA);
    // x is written by the preceding kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    const uint4* __restrict__ xg = reinterpret_cast<const uint4*>(x);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    int cr = 0, ci = 0, pr = 0;                              // consume cursor: row, chunk, row in pass
    auto consume_group = [&](const uint4* buf) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (cr < nrows) {
                const int c = c_lo + lane + 32 * ci;
                if (c < c_hi) {
                    const uint32_t* wp = reinterpret_cast<const uint32_t*>(&buf[u]);
#pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        const uint4 xv = __ldg(xg + (size_t)b * nc + c);
                        const uint32_t* xp = reinterpret_cast<const uint32_t*>(&xv);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            acc[b] = fmaf(gv_lo(wp[q]), gv_lo(xp[q]), acc[b]);
                            acc[b] = fmaf(gv_hi(wp[q]), gv_hi(xp[q]), acc[b]);
                        }
                    }
                }
                if (++ci == cpl) {              // this warp's slice of row cr is complete
                    ci = 0;
#pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        const float sum = warp_sum(acc[b]);
                        if (lane == 0) part[pr][warp][b] = sum;
                        acc[b] = 0.f;
                    }
                    // every warp reaches the end of a pass at the same point:
                    // add the slices of the pass's rows in warp order and store
                    if (++pr == GV_PASS || cr == nrows - 1) {
                        __syncthreads();
                        const int rp = cr + 1 - pr;     // first row of the pass
                        for (int i = threadIdx.x; i < pr * NB; i += GV_THREADS) {
                            const int rr = i / NB, b = i % NB;
                            float sum = 0.f;
#pragma unroll
                            for (int w2 = 0; w2 < GV_WARPS; ++w2) sum += part[rr][w2][b];
                            y[(size_t)b * N + row0 + rp + rr] = __float2bfloat16_rn(sum);
                        }
                        __syncthreads();
                        pr = 0;
                    }
                    ++cr;
                }
            }
        }
    };
#pragma unroll 1
    for (int g = 0; g < n_groups; g += 2) {
        load_group(bufB);
        consume_group(bufA);
        if (g + 1 >= n_groups) break;
        load_group(bufA);
        consume_group(bufB);
    }
}

static int gv_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
    }
    return n;
}

template <typename Kern>
static cudaError_t gv_launch(Kern kern, unsigned grid, int N, int K, const void* w, const void* x, void* y,
                             cudaStream_t s) {
    return launch_pdl(kern, dim3(grid), dim3(GV_THREADS), 0, s, N, K, static_cast<const __nv_bfloat16*>(w),
                      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y));
}

static int gv_resident(const void* kern) {
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, GV_THREADS, 0) != cudaSuccess || per < 1) per = 1;
    return per;
}

template <int NB>
static cudaError_t gemv_launch(int N, int K, const void* w, const void* x, void* y, cudaStream_t s) {
    if (K > GV_KSPLIT_MIN_K) {
        constexpr int U = NB <= 2 ? 4 : 2;
        static int per = 0;
        if (per == 0) per = gv_resident((const void*)gemv_ksplit_kernel<NB, U>);
        const long long cap = (long long)per * gv_sms();
        return gv_launch(gemv_ksplit_kernel<NB, U>, (unsigned)(N < cap ? N : cap), N, K, w, x, y, s);
    }
    static int per2 = 0, per4 = 0;
    if (per2 == 0) {
        per2 = gv_resident((const void*)gemv_rows_kernel<NB, 2>);
        per4 = gv_resident((const void*)gemv_rows_kernel<NB, 4>);
    }
    const long long need = ((long long)N + GV_WARPS - 1) / GV_WARPS;
    if ((long long)N <= (long long)per2 * gv_sms() * GV_WARPS) {
        const long long cap = (long long)per2 * gv_sms();
        return gv_launch(gemv_rows_kernel<NB, 2>, (unsigned)(need < cap ? need : cap), N, K, w, x, y, s);
    }
    const long long cap = (long long)per4 * gv_sms();
    return gv_launch(gemv_rows_kernel<NB, 4>, (unsigned)(need < cap ? need : cap), N, K, w, x, y, s);
}

}  // namespace qv

using namespace qv;

extern "C" int qv_gemv(int32_t rows, int32_t n, int32_t k, const void* w, const void* x, void* y,
                       qv_stream_t stream) {
    if (rows < 1 || rows > GV_MAXB || n <= 0 || k <= 0 || k % 8 || !w || !x || !y) return QV_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) return QV_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e;
    switch (rows) {
        case 1: e = gemv_launch<1>(n, k, w, x, y, s); break;
        case 2: e = gemv_launch<2>(n, k, w, x, y, s); break;
        case 3: e = gemv_launch<3>(n, k, w, x, y, s); break;
        case 4: e = gemv_launch<4>(n, k, w, x, y, s); break;
        case 5: e = gemv_launch<5>(n, k, w, x, y, s); break;
        case 6: e = gemv_launch<6>(n, k, w, x, y, s); break;
        case 7: e = gemv_launch<7>(n, k, w, x, y, s); break;
        default: e = gemv_launch<8>(n, k, w, x, y, s); break;
    }
    if (e != cudaSuccess) return set_cuda_error(e);
    return check_launch();
}
