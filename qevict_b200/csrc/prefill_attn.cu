// Prefill lane: causal attention + per-key column sums that seed the ledger.
// This file holds the CUDA-core kernels, used for fp32; bf16/fp16 run the
// tensor-core kernels of prefill_tc.cu (same results, within rounding).
//
// Replaces flash_attn_func + compute_chunked_prefill_scores
// (src/models/attention/ops_flash.py:22-141).  Logits are rounded the way the
// reference's scorer rounds them (q.k rounded to the KV dtype, / sqrt(D)
// rounded); each query row's softmax statistics (max, sum) come from the
// forward pass, and the column pass recomputes the probabilities, rounds them
// to the KV dtype, averages the GQA group (rounded), sums them over each
// 512-query chunk (rounded to the KV dtype) and accumulates the chunks in fp32.
//
// Pass 1 (prefill_fwd_kernel): one CTA per (64-query tile, query head, sequence).
// Pass 2 (prefill_colsum_kernel): one CTA per (64-key tile, KV head, sequence);
// each CTA owns its keys, so the column sums are deterministic.
#include <math.h>

#include "common.cuh"

namespace qv {

constexpr int PT = 64;        // tile edge (queries and keys)
constexpr int PA_THREADS = 256;
constexpr int SCORE_CHUNK = 512;

template <int DT, int D>
__global__ void __launch_bounds__(PA_THREADS)
prefill_fwd_kernel(Geo g, const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v,
                   int S, void* __restrict__ out, float* __restrict__ stats) {
    extern __shared__ __align__(16) float psm[];
    float* sQ = psm;                    // [PT][D+1]
    float* sK = sQ + PT * (D + 1);      // [PT][D+1]
    float* sV = sK + PT * (D + 1);      // [PT][D]
    float* sP = sV + PT * D;            // [PT][PT+1]
    float* sScale = sP + PT * (PT + 1); // [PT]
    const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
    const int Hq = g.H * g.G, h = hq / g.G;
    const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
    const int q0 = qt * PT;
    const float sqrt_d = sqrtf((float)D);

    for (int i = tid; i < PT * D; i += PA_THREADS) {
        const int r = i / D, d = i % D;
        const int qi = q0 + r;
        sQ[r * (D + 1) + d] = qi < S ? ld<DT>(q, (((size_t)b * S + qi) * Hq + hq) * D + d) : 0.f;
    }
    // softmax state of row r = tid / 4 (4 threads per row), output dims d = tid%4 + 4*i
    const int orow = tid / 4, oc = tid % 4;
    float m = -INFINITY, l = 0.f;
    float o[D / 4];
#pragma unroll
    for (int i = 0; i < D / 4; ++i) o[i] = 0.f;

    const int n_kt = min((q0 + PT - 1) / PT + 1, (S + PT - 1) / PT);
    for (int kt = 0; kt < n_kt; ++kt) {
        const int k0 = kt * PT;
        __syncthreads();
        for (int i = tid; i < PT * D; i += PA_THREADS) {
            const int r = i / D, d = i % D;
            const int ki = k0 + r;
            const size_t gi = (((size_t)b * S + ki) * g.H + h) * D + d;
            sK[r * (D + 1) + d] = ki < S ? ld<DT>(k, gi) : 0.f;
            sV[r * D + d] = ki < S ? ld<DT>(v, gi) : 0.f;
        }
        __syncthreads();
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        for (int d = 0; d < D; ++d) {
            float a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sQ[(ty * 4 + i) * (D + 1) + d];
#pragma unroll
            for (int j = 0; j < 4; ++j) bb[j] = sK[(tx + 16 * j) * (D + 1) + d];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int qi = q0 + ty * 4 + i, ki = k0 + tx + 16 * j;
                const float lg = div_r<DT>(rnd<DT>(acc[i][j]), sqrt_d);
                sP[(ty * 4 + i) * (PT + 1) + tx + 16 * j] = (ki <= qi && ki < S) ? lg : -INFINITY;
            }
        __syncthreads();
        // online softmax for row orow: 4 threads x 16 columns
        float mx = -INFINITY;
        for (int j = oc; j < PT; j += 4) mx = fmaxf(mx, sP[orow * (PT + 1) + j]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);
        float ps = 0.f;
        if (mn > -INFINITY) {
            for (int j = oc; j < PT; j += 4) {
                const float p = expf(sP[orow * (PT + 1) + j] - mn);
                sP[orow * (PT + 1) + j] = p;
                ps += p;
            }
        } else {
            for (int j = oc; j < PT; j += 4) sP[orow * (PT + 1) + j] = 0.f;
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        const float sc = (m > -INFINITY) ? expf(m - mn) : 0.f;
        l = l * sc + ps;
        m = mn;
        __syncwarp();
        // the 4 threads of a row are in the same warp; sP row fully written by them
        __syncthreads();
#pragma unroll
        for (int i = 0; i < D / 4; ++i) o[i] *= sc;
        for (int j = 0; j < PT; ++j) {
            const float p = sP[orow * (PT + 1) + j];
#pragma unroll
            for (int i = 0; i < D / 4; ++i) o[i] = fmaf(p, sV[j * D + oc + 4 * i], o[i]);
        }
    }
    const int qi = q0 + orow;
    if (qi < S) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int i = 0; i < D / 4; ++i)
            st<DT>(out, (((size_t)b * S + qi) * Hq + hq) * D + oc + 4 * i, o[i] * inv);
        if (oc == 0) {
            stats[(((size_t)b * Hq + hq) * S + qi) * 2 + 0] = m;
            stats[(((size_t)b * Hq + hq) * S + qi) * 2 + 1] = l;
        }
    }
    (void)sScale;
}

template <int DT, int D>
__global__ void __launch_bounds__(PA_THREADS)
prefill_colsum_kernel(Geo g, const void* __restrict__ q, const void* __restrict__ k, int S,
                      const float* __restrict__ stats, float* __restrict__ colsum) {
    extern __shared__ __align__(16) float csm[];
    float* sK = csm;                     // [PT][D+1]
    float* sQ = sK + PT * (D + 1);       // [PT][D+1]
    float* sStat = sQ + PT * (D + 1);    // [PT][2]
    float* sPart = sStat + 2 * PT;       // [16][PT]
    float* sChunk = sPart + 16 * PT;     // [PT]
    float* sAcc = sChunk + PT;           // [PT]
    const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int Hq = g.H * g.G, G = g.G;
    const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
    const int k0 = kt * PT;
    const float sqrt_d = sqrtf((float)D);

    for (int i = tid; i < PT * D; i += PA_THREADS) {
        const int r = i / D, d = i % D;
        const int ki = k0 + r;
        sK[r * (D + 1) + d] = ki < S ? ld<DT>(k, (((size_t)b * S + ki) * g.H + h) * D + d) : 0.f;
    }
    if (tid < PT) sAcc[tid] = 0.f;
    const int c_first = k0 / SCORE_CHUNK;
    const int n_chunks = (S + SCORE_CHUNK - 1) / SCORE_CHUNK;
    for (int c = c_first; c < n_chunks; ++c) {
        if (tid < PT) sChunk[tid] = 0.f;
        const int cq0 = c * SCORE_CHUNK, cq1 = min(cq0 + SCORE_CHUNK, S);
        for (int qs = max(cq0, (k0 / PT) * PT); qs < cq1; qs += PT) {
            float macc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) macc[i][j] = 0.f;
            for (int gi = 0; gi < G; ++gi) {
                const int hq = h * G + gi;
                __syncthreads();
                for (int i = tid; i < PT * D; i += PA_THREADS) {
                    const int r = i / D, d = i % D;
                    const int qi = qs + r;
                    sQ[r * (D + 1) + d] = qi < S ? ld<DT>(q, (((size_t)b * S + qi) * Hq + hq) * D + d) : 0.f;
                }
                if (tid < PT) {
                    const int qi = qs + tid;
                    sStat[2 * tid] = qi < S ? stats[(((size_t)b * Hq + hq) * S + qi) * 2] : 0.f;
                    sStat[2 * tid + 1] = qi < S ? stats[(((size_t)b * Hq + hq) * S + qi) * 2 + 1] : 1.f;
                }
                __syncthreads();
                float acc[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
                for (int d = 0; d < D; ++d) {
                    float a[4], bb[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[i] = sQ[(ty * 4 + i) * (D + 1) + d];
#pragma unroll
                    for (int j = 0; j < 4; ++j) bb[j] = sK[(tx + 16 * j) * (D + 1) + d];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int qi = qs + ty * 4 + i;
                    const float mq = sStat[2 * (ty * 4 + i)], lq = sStat[2 * (ty * 4 + i) + 1];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int ki = k0 + tx + 16 * j;
                        float p = 0.f;
                        if (qi < S && ki < S && ki <= qi) {
                            const float lg = div_r<DT>(rnd<DT>(acc[i][j]), sqrt_d);
                            p = rnd<DT>(expf(lg - mq) / lq);
                        }
                        macc[i][j] += p;
                    }
                }
            }
            // group mean (rounded), then this thread's 4 query rows, then the 16 row groups
            float colp[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float s4 = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) s4 += rnd<DT>(macc[i][j] / (float)G);
                colp[j] = s4;
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 4; ++j) sPart[ty * PT + tx + 16 * j] = colp[j];
            __syncthreads();
            if (tid < PT) {
                float s = sChunk[tid];
                for (int r = 0; r < 16; ++r) s += sPart[r * PT + tid];
                sChunk[tid] = s;
            }
        }
        __syncthreads();
        if (tid < PT) sAcc[tid] += rnd<DT>(sChunk[tid]);
        __syncthreads();
    }
    if (tid < PT && k0 + tid < S) colsum[((size_t)b * g.H + h) * S + k0 + tid] = sAcc[tid];
}

// tensor-core prefill lane (prefill_tc.cu) for bf16/fp16
bool pft_supported(const Geo& g);
size_t pft_partial_bytes(const Geo& g, int S);
int pft_launch(const Geo& g, const void* q, const void* k, const void* v, int S, void* out, float* colsum,
               float* stats, float* partial, int* err, cudaStream_t s);

static size_t fwd_smem(int D) { return (size_t)(2 * PT * (D + 1) + PT * D + PT * (PT + 1) + PT) * 4; }
static size_t col_smem(int D) { return (size_t)(2 * PT * (D + 1) + 2 * PT + 16 * PT + 2 * PT) * 4; }

template <int DT, int D>
static int launch_prefill(const Geo& g, const void* q, const void* k, const void* v, int S, void* out,
                          float* colsum, float* stats, cudaStream_t s) {
    const size_t fs = fwd_smem(D), cs = col_smem(D);
    static int c1 = 48 * 1024, c2 = 48 * 1024;
    cudaError_t e = ensure_smem(prefill_fwd_kernel<DT, D>, fs, &c1);
    if (e != cudaSuccess) return set_cuda_error(e);
    e = ensure_smem(prefill_colsum_kernel<DT, D>, cs, &c2);
    if (e != cudaSuccess) return set_cuda_error(e);
    dim3 g1((S + PT - 1) / PT, g.H * g.G, g.B);
    prefill_fwd_kernel<DT, D><<<g1, PA_THREADS, fs, s>>>(g, q, k, v, S, out, stats);
    if (colsum) {
        dim3 g2((S + PT - 1) / PT, g.H, g.B);
        prefill_colsum_kernel<DT, D><<<g2, PA_THREADS, cs, s>>>(g, q, k, S, stats, colsum);
    }
    return check_launch();
}

}  // namespace qv

using namespace qv;

// Workspace: the per-row softmax statistics; for the tensor-core lane the
// column-sum partials; then the device error word of the pipelined lane, at
// the last 256-byte boundary at least 256 bytes before the workspace's end.
static size_t err_offset(size_t workspace_bytes) { return (workspace_bytes - 256) & ~(size_t)255; }

static size_t stats_bytes(const qv_dims* d, int32_t S) {
    const size_t n = (size_t)d->batch * d->kv_heads * d->group * (size_t)S * 2 * sizeof(float);
    return (n + 255) & ~(size_t)255;
}

static size_t partial_bytes(const qv_dims* d, int32_t S) {
    const Geo g = make_geo(d);
    if (!pft_supported(g)) return 0;
    return (pft_partial_bytes(g, S) + 255) & ~(size_t)255;
}

extern "C" size_t qv_prefill_workspace_bytes(const qv_dims* d, int32_t S) {
    if (!d || S <= 0) return 0;
    return stats_bytes(d, S) + partial_bytes(d, S) + 256;
}

extern "C" int qv_prefill_read_error(const void* workspace, size_t workspace_bytes, int32_t* host_err,
                                     qv_stream_t stream) {
    if (!workspace || !host_err || workspace_bytes < 256) return QV_EINVAL;
    const int32_t* err = reinterpret_cast<const int32_t*>(static_cast<const char*>(workspace) + err_offset(workspace_bytes));
    cudaError_t e = cudaMemcpyAsync(host_err, err, sizeof(int32_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    return e == cudaSuccess ? QV_OK : set_cuda_error(e);
}

extern "C" int qv_prefill_attention(const qv_dims* d, const void* q, const void* k, const void* v, int32_t S,
                                    void* out, float* colsum, void* workspace, size_t workspace_bytes,
                                    qv_stream_t stream) {
    if (!d || !q || !k || !v || !out || S <= 0) return QV_EINVAL;
    if (d->head_dim != 64 && d->head_dim != 128) return QV_EINVAL;
    if (d->group <= 0 || d->kv_heads <= 0 || d->batch <= 0) return QV_EINVAL;
    if (workspace_bytes < qv_prefill_workspace_bytes(d, S) || !workspace) return QV_ESPACE;
    Geo g = make_geo(d);
    float* stats = reinterpret_cast<float*>(workspace);
    int* err = reinterpret_cast<int*>(static_cast<char*>(workspace) + err_offset(workspace_bytes));
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t ce = cudaMemsetAsync(err, 0, sizeof(int), s);
    if (ce != cudaSuccess) return set_cuda_error(ce);
    if (pft_supported(g)) {
        float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + stats_bytes(d, S));
        return pft_launch(g, q, k, v, S, out, colsum, stats, partial, err, s);
    }
#define QV_PA(DT)                                                                   \
    return g.D == 128 ? launch_prefill<DT, 128>(g, q, k, v, S, out, colsum, stats, s) \
                      : launch_prefill<DT, 64>(g, q, k, v, S, out, colsum, stats, s)
    switch (d->dtype) {
        case QV_F32: QV_PA(QV_F32);
        case QV_BF16: QV_PA(QV_BF16);
        default: QV_PA(QV_F16);
    }
#undef QV_PA
}
