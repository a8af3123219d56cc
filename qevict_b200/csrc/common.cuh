// Shared device helpers for the Sticky-KV kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qevict_b200.h"

namespace qv {

// ---------------------------------------------------------------------------
// Element types.  The reference evaluates every op of a bf16/fp16 tensor as
// "widen to fp32, compute, round to nearest even"; rnd<DT>() is that rounding.
// ---------------------------------------------------------------------------
template <int DT> struct Elt;
template <> struct Elt<QV_F32> {
    using T = float;
    static __device__ __forceinline__ float f(T x) { return x; }
    static __device__ __forceinline__ T t(float x) { return x; }
};
template <> struct Elt<QV_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float f(T x) { return __bfloat162float(x); }
    static __device__ __forceinline__ T t(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elt<QV_F16> {
    using T = __half;
    static __device__ __forceinline__ float f(T x) { return __half2float(x); }
    static __device__ __forceinline__ T t(float x) { return __float2half_rn(x); }
};

template <int DT> __device__ __forceinline__ float rnd(float x) { return Elt<DT>::f(Elt<DT>::t(x)); }

// One torch op on the KV dtype: an IEEE fp32 op (never contracted into an FMA)
// followed by the rounding to the dtype.
template <int DT> __device__ __forceinline__ float mul_r(float a, float b) { return rnd<DT>(__fmul_rn(a, b)); }
template <int DT> __device__ __forceinline__ float add_r(float a, float b) { return rnd<DT>(__fadd_rn(a, b)); }
template <int DT> __device__ __forceinline__ float sub_r(float a, float b) { return rnd<DT>(__fsub_rn(a, b)); }
template <int DT> __device__ __forceinline__ float div_r(float a, float b) { return rnd<DT>(__fdiv_rn(a, b)); }

template <int DT> __device__ __forceinline__ float ld(const void* p, size_t i) {
    return Elt<DT>::f(reinterpret_cast<const typename Elt<DT>::T*>(p)[i]);
}
template <int DT> __device__ __forceinline__ void st(void* p, size_t i, float x) {
    reinterpret_cast<typename Elt<DT>::T*>(p)[i] = Elt<DT>::t(x);
}

// ---------------------------------------------------------------------------
// Geometry of one layer, computed once on the host.
// ---------------------------------------------------------------------------
struct Geo {
    int B, H, G, D, om, sink, local, kw, qw, maxW, bits, dt, flags;
    int R;       // ring windows = local/om + 1
    int S_cap;   // sink + (kw + R) * om
    int qbytes;  // bytes of one code row: D (INT8) or D/2 (INT4)
    __host__ __device__ int ring_base() const { return sink + kw * om; }
    __host__ __device__ size_t bh(int b, int h) const { return (size_t)b * H + h; }
};

inline Geo make_geo(const qv_dims* d) {
    Geo g;
    g.B = d->batch; g.H = d->kv_heads; g.G = d->group; g.D = d->head_dim; g.om = d->omega;
    g.sink = d->sink; g.local = d->local; g.kw = d->k_windows; g.qw = d->q_windows;
    g.maxW = d->max_windows; g.bits = d->bits; g.dt = d->dtype; g.flags = d->flags;
    g.R = (d->omega > 0) ? d->local / d->omega + 1 : 0;
    g.S_cap = g.sink + (g.kw + g.R) * g.om;
    g.qbytes = g.bits == 4 ? g.D / 2 : g.D;
    return g;
}

int validate_dims(const qv_dims* d);

// Raise a kernel's dynamic shared-memory limit only when a launch needs more
// than any earlier one did, so that steady-state launches (and CUDA-graph
// captures) make no attribute calls.
template <typename K>
inline cudaError_t ensure_smem(K kernel, size_t bytes, int* cached) {
    if ((int)bytes <= *cached) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) *cached = (int)bytes;
    return e;
}
int set_cuda_error(cudaError_t e);
int check_launch();

// Launch as a programmatic dependent of the preceding kernel in the stream:
// the grid may be scheduled once every CTA of that kernel has executed
// griddepcontrol.launch_dependents, and must execute griddepcontrol.wait
// before it reads anything that kernel writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

size_t elt_size(int dt);
__host__ __device__ constexpr size_t elt_size_dev(int dt) { return dt == QV_F32 ? 4 : 2; }

// Warp reductions.
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ int warp_min_i(int x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = min(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}

// Sum of one window's omega fp32 values in the fixed order shared with the
// oracle: lane l accumulates v[l], v[l+32], v[l+64], ... sequentially, then the
// 32 lanes combine by xor-butterfly over offsets 16, 8, 4, 2, 1.
__device__ __forceinline__ float window_tree_sum(const float* v, int om, int lane) {
    float a = 0.f;
    bool first = true;
    for (int i = lane; i < om; i += 32) {
        a = first ? v[i] : a + v[i];
        first = false;
    }
    return warp_sum(a);
}

__device__ __forceinline__ void set_err(int32_t* err, int bit) { atomicOr(err, bit); }

}  // namespace qv
