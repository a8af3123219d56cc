// Prefill lane on the 5th-generation tensor cores (tcgen05 + TMEM), bf16/fp16.
//
// Same results as the CUDA-core kernels of prefill_attn.cu (which remain for
// fp32): causal attention output and the per-key column sums the reference's
// chunked scorer produces (src/models/attention/ops_flash.py:56-141):
// logits rounded like the reference (q.k rounded to the KV dtype, / sqrt(D)
// rounded), fp32 softmax statistics per query row, probabilities rounded to the
// KV dtype, group mean rounded, sums over each 512-query chunk rounded, chunks
// accumulated in fp32.
//
// Three kernels, each a 128-thread CTA (four warps = the four TMEM lane
// quarters, one thread per tile row); thread 0 issues the TMA loads and the
// tcgen05.mma instructions and commits them to mbarriers; every wait is
// bounded.  Operand tiles are 4-D TMA boxes (64 elements x rows) with the
// 128-byte swizzle, which is the canonical K-major / MN-major UMMA layout.
//
//   pft_stats_kernel   one CTA per (128-query tile, query head): S = Q.K^T per
//                      128-key tile into TMEM (M = queries, N = keys), running
//                      max / sum of exp of the rounded logits per row.
//   pft_out_kernel     the same S tiles; P = exp(l - max) / sum rounded to the
//                      KV dtype is written to shared memory (swizzled) and
//                      O += P.V runs on the tensor cores (V as an MN-major
//                      operand), O accumulating in TMEM across key tiles.
//   pft_colsum_kernel  one CTA per (128-key tile, KV head): S^T = K.Q^T with
//                      the keys in M and (query, group head) pairs in N
//                      (32 queries x G heads), so each thread owns one key and
//                      folds the group mean and the chunk sums on its own.
#include <cudaTypedefs.h>
#include <math.h>

#include "common.cuh"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace qv {

constexpr int PFT_ROWS = 128;        // queries (stats/out) or keys (colsum) per tile
constexpr int PFT_SLAB = 16384;      // one 64-element x 128-row swizzled slab
constexpr int PFT_QB = 32;           // queries per colsum step
constexpr int PFT_CHUNK = 512;       // queries per rounded chunk of the scorer

struct PftArgs {
    int S, B, H, G, Hq;
    float* stats;                    // [B][Hq][S][2]: max, sum
    void* out;                       // [B][S][Hq][D]
    float* colsum;                   // [B][H][S]
    int* err;                        // set to 1 when a wait gives up
};

__device__ __forceinline__ bool pft_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_wait_bounded(bar, parity)) return true;
    if (err) atomicExch(err, 1);
    return false;
}

template <int D>
__device__ __forceinline__ uint32_t pft_kmajor_step(uint32_t base, int kk) {
    // k-step kk (16 elements) of a K-major operand stored as D/64 slabs
    return base + (uint32_t)((kk >> 2) * PFT_SLAB + (kk & 3) * 32);
}

// ---------------------------------------------------------------- stats
template <int DT, int D>
__global__ void __launch_bounds__(128, 1) pft_stats_kernel(const __grid_constant__ CUtensorMap mQ,
                                                           const __grid_constant__ CUtensorMap mK, PftArgs a) {
    constexpr int NS = D / 64;                   // slabs per operand tile
    extern __shared__ unsigned char pft_raw[];
    unsigned char* sm = pft_raw + ((1024u - (smem_u32(pft_raw) & 1023u)) & 1023u);
    unsigned char* sQ = sm;                      // [NS] slabs
    unsigned char* sK = sm + NS * PFT_SLAB;      // [2][NS] slabs
    __shared__ __align__(8) uint64_t bar_k[2], bar_s;
    __shared__ uint32_t s_taddr;
    const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
    const int h = hq / a.G;
    const int warp = threadIdx.x >> 5;
    const int q0 = qt * PFT_ROWS;
    const int nkt = qt + 1;
    const float sqrt_d = sqrtf((float)D);

    if (warp == 0) { tmem_alloc(&s_taddr, 128); tmem_relinquish(); }
    if (threadIdx.x == 0) {
        mbar_init(&bar_k[0], 1); mbar_init(&bar_k[1], 1); mbar_init(&bar_s, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = s_taddr;
    const uint32_t idesc = umma_idesc_f16(DT == QV_BF16, 128, 128, 0, 0);
    if (threadIdx.x == 0) {
        prefetch_tensormap(&mQ);
        prefetch_tensormap(&mK);
        mbar_arrive_expect_tx(&bar_k[0], 2 * NS * PFT_SLAB);
        for (int s = 0; s < NS; ++s) {
            tma_load_4d(sQ + s * PFT_SLAB, &mQ, 64 * s, hq, q0, b, &bar_k[0]);
            tma_load_4d(sK + s * PFT_SLAB, &mK, 64 * s, h, 0, b, &bar_k[0]);
        }
    }
    const int qi = q0 + threadIdx.x;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int kt = 0; kt < nkt; ++kt) {
        const int st = kt & 1;
        if (threadIdx.x == 0) {
            if (kt + 1 < nkt) {
                mbar_arrive_expect_tx(&bar_k[st ^ 1], NS * PFT_SLAB);
                for (int s = 0; s < NS; ++s)
                    tma_load_4d(sK + ((st ^ 1) * NS + s) * PFT_SLAB, &mK, 64 * s, h, (kt + 1) * PFT_ROWS, b, &bar_k[st ^ 1]);
            }
            if (pft_wait(&bar_k[st], (kt >> 1) & 1, a.err)) {
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + st * NS * PFT_SLAB);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(taddr, umma_desc_sw128(pft_kmajor_step<D>(qa, kk), 16, 1024),
                             umma_desc_sw128(pft_kmajor_step<D>(ka, kk), 16, 1024), idesc, kk > 0);
            }
            umma_commit(&bar_s);
        }
        __syncwarp();
        ok = ok && pft_wait(&bar_s, kt & 1, a.err);
        ok = __all_sync(0xffffffffu, ok);   // TMEM loads are warp-collective
        tc_fence_after();
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tmem_ld32(taddr + ((uint32_t)(32 * warp) << 16) + 32 * c, v);
                tmem_wait_ld();
                const int kbase = kt * PFT_ROWS + 32 * c;
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int ki = kbase + i;
                    v[i] = (ki <= qi && ki < a.S) ? div_r<DT>(rnd<DT>(v[i]), sqrt_d) : -INFINITY;
                    mx = fmaxf(mx, v[i]);
                }
                const float mn = fmaxf(m, mx);
                if (mn > -INFINITY) {
                    float ps = 0.f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) ps += v[i] > -INFINITY ? expf(v[i] - mn) : 0.f;
                    l = (m > -INFINITY ? l * expf(m - mn) : 0.f) + ps;
                    m = mn;
                }
            }
        }
        tc_fence_before();
        __syncthreads();
    }
    if (qi < a.S) {
        float* sp = a.stats + (((size_t)b * a.Hq + hq) * a.S + qi) * 2;
        sp[0] = m;
        sp[1] = l;
    }
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, 128);
}

// ---------------------------------------------------------------- output
template <int DT, int D>
__global__ void __launch_bounds__(128, 1) pft_out_kernel(const __grid_constant__ CUtensorMap mQ,
                                                         const __grid_constant__ CUtensorMap mK,
                                                         const __grid_constant__ CUtensorMap mV, PftArgs a) {
    using T = typename Elt<DT>::T;
    constexpr int NS = D / 64;
    extern __shared__ unsigned char pft_raw[];
    unsigned char* sm = pft_raw + ((1024u - (smem_u32(pft_raw) & 1023u)) & 1023u);
    unsigned char* sQ = sm;                              // [NS]
    unsigned char* sK = sQ + NS * PFT_SLAB;              // [2][NS]
    unsigned char* sV = sK + 2 * NS * PFT_SLAB;          // [2][NS]
    unsigned char* sP = sV + 2 * NS * PFT_SLAB;          // [2] slabs: 128 queries x 128 keys
    __shared__ __align__(8) uint64_t bar_k[2], bar_s, bar_pv;
    __shared__ uint32_t s_taddr;
    const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
    const int h = hq / a.G;
    const int warp = threadIdx.x >> 5;
    const int q0 = qt * PFT_ROWS;
    const int nkt = qt + 1;
    const float sqrt_d = sqrtf((float)D);

    if (warp == 0) { tmem_alloc(&s_taddr, 256); tmem_relinquish(); }
    if (threadIdx.x == 0) {
        mbar_init(&bar_k[0], 1); mbar_init(&bar_k[1], 1); mbar_init(&bar_s, 1); mbar_init(&bar_pv, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = s_taddr;            // S: columns [0, 128); O: [128, 128 + D)
    const uint32_t id_s = umma_idesc_f16(DT == QV_BF16, 128, 128, 0, 0);
    const uint32_t id_o = umma_idesc_f16(DT == QV_BF16, 128, D, 0, 1);
    if (threadIdx.x == 0) {
        prefetch_tensormap(&mQ);
        prefetch_tensormap(&mK);
        prefetch_tensormap(&mV);
        mbar_arrive_expect_tx(&bar_k[0], 3 * NS * PFT_SLAB);
        for (int s = 0; s < NS; ++s) {
            tma_load_4d(sQ + s * PFT_SLAB, &mQ, 64 * s, hq, q0, b, &bar_k[0]);
            tma_load_4d(sK + s * PFT_SLAB, &mK, 64 * s, h, 0, b, &bar_k[0]);
            tma_load_4d(sV + s * PFT_SLAB, &mV, 64 * s, h, 0, b, &bar_k[0]);
        }
    }
    const int r = threadIdx.x;
    const int qi = q0 + r;
    float m = 0.f, linv = 0.f;
    if (qi < a.S) {
        const float* sp = a.stats + (((size_t)b * a.Hq + hq) * a.S + qi) * 2;
        m = sp[0];
        linv = sp[1] > 0.f ? 1.f / sp[1] : 0.f;
    }
    bool ok = true;
    for (int kt = 0; kt < nkt; ++kt) {
        const int st = kt & 1;
        // the previous tile's P.V has read P and its K/V stage
        if (kt > 0) ok = ok && pft_wait(&bar_pv, (kt - 1) & 1, a.err);
        if (threadIdx.x == 0) {
            if (kt + 1 < nkt) {
                mbar_arrive_expect_tx(&bar_k[st ^ 1], 2 * NS * PFT_SLAB);
                for (int s = 0; s < NS; ++s) {
                    tma_load_4d(sK + ((st ^ 1) * NS + s) * PFT_SLAB, &mK, 64 * s, h, (kt + 1) * PFT_ROWS, b, &bar_k[st ^ 1]);
                    tma_load_4d(sV + ((st ^ 1) * NS + s) * PFT_SLAB, &mV, 64 * s, h, (kt + 1) * PFT_ROWS, b, &bar_k[st ^ 1]);
                }
            }
            if (pft_wait(&bar_k[st], (kt >> 1) & 1, a.err)) {
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + st * NS * PFT_SLAB);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(taddr, umma_desc_sw128(pft_kmajor_step<D>(qa, kk), 16, 1024),
                             umma_desc_sw128(pft_kmajor_step<D>(ka, kk), 16, 1024), id_s, kk > 0);
            }
            umma_commit(&bar_s);
        }
        __syncwarp();
        ok = ok && pft_wait(&bar_s, kt & 1, a.err);
        ok = __all_sync(0xffffffffu, ok);   // TMEM loads are warp-collective
        tc_fence_after();
        // P row r: 128 keys as 16 chunks of 8, written with the 128-byte swizzle
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            float v[32];
            if (ok) {
                tmem_ld32(taddr + ((uint32_t)(32 * warp) << 16) + 32 * c, v);
                tmem_wait_ld();
            }
            const int kbase = kt * PFT_ROWS + 32 * c;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t w[4];
#pragma unroll
                for (int e2 = 0; e2 < 4; ++e2) {
                    float p2[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int i = 8 * j + 2 * e2 + u;
                        const int ki = kbase + i;
                        p2[u] = (ok && ki <= qi && ki < a.S && qi < a.S)
                                    ? expf(div_r<DT>(rnd<DT>(v[i]), sqrt_d) - m) * linv : 0.f;
                    }
                    if (DT == QV_BF16) {
                        const __nv_bfloat162 x = __floats2bfloat162_rn(p2[0], p2[1]);
                        w[e2] = *reinterpret_cast<const uint32_t*>(&x);
                    } else {
                        const __half2 x = __floats2half2_rn(p2[0], p2[1]);
                        w[e2] = *reinterpret_cast<const uint32_t*>(&x);
                    }
                }
                const int col8 = 4 * c + j;                 // 8-key chunk index 0..15
                const int slab = col8 >> 3, ch = col8 & 7;
                *reinterpret_cast<uint4*>(sP + slab * PFT_SLAB + r * 128 + ((ch ^ (r & 7)) << 4)) =
                    make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sP), va = smem_u32(sV + st * NS * PFT_SLAB);
#pragma unroll
            for (int kk = 0; kk < PFT_ROWS / 16; ++kk)
                umma_f16(taddr + 128, umma_desc_sw128(pft_kmajor_step<128>(pa, kk), 16, 1024),
                         umma_desc_sw128(va + kk * 2048, PFT_SLAB, 1024), id_o, (kt > 0 || kk > 0) ? 1 : 0);
            umma_commit(&bar_pv);
        }
        __syncwarp();
    }
    ok = ok && pft_wait(&bar_pv, (nkt - 1) & 1, a.err);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
        // every lane of the warp takes part in the (warp-collective) TMEM loads;
        // only rows inside the sequence are stored
        T* orow = reinterpret_cast<T*>(a.out) + (((size_t)b * a.S + qi) * a.Hq + hq) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
            float v[32];
            tmem_ld32(taddr + ((uint32_t)(32 * warp) << 16) + 128 + 32 * c, v);
            tmem_wait_ld();
            if (qi < a.S) {
#pragma unroll
                for (int i = 0; i < 32; ++i) orow[32 * c + i] = Elt<DT>::t(v[i]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, 256);
}

// ---------------------------------------------------------------- column sums
template <int DT, int D>
__global__ void __launch_bounds__(128, 1) pft_colsum_kernel(const __grid_constant__ CUtensorMap mK,
                                                            const __grid_constant__ CUtensorMap mQg, PftArgs a) {
    constexpr int NS = D / 64;
    extern __shared__ unsigned char pft_raw[];
    unsigned char* sm = pft_raw + ((1024u - (smem_u32(pft_raw) & 1023u)) & 1023u);
    const int G = a.G;
    const int N = PFT_QB * G;                            // (query, head) columns per step
    const int qslab = N * 128;                           // bytes of one slab of a query block
    unsigned char* sK = sm;                              // [NS]
    unsigned char* sQ = sK + NS * PFT_SLAB;              // [2][NS] slabs of N rows
    float* s_st = reinterpret_cast<float*>(sQ + 2 * NS * qslab);   // [2][N][2]
    __shared__ __align__(8) uint64_t bar_q[2], bar_s;
    __shared__ uint32_t s_taddr;
    const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5;
    const int k0 = kt * PFT_ROWS;
    const int key = k0 + threadIdx.x;
    const int qb0 = k0 / PFT_QB;
    const int nqb = (a.S + PFT_QB - 1) / PFT_QB - qb0;
    const float sqrt_d = sqrtf((float)D);

    if (warp == 0) { tmem_alloc(&s_taddr, 256); tmem_relinquish(); }
    if (threadIdx.x == 0) {
        mbar_init(&bar_q[0], 1); mbar_init(&bar_q[1], 1); mbar_init(&bar_s, 1);
        fence_barrier_init();
    }
    auto load_stats = [&](int j, int buf) {
        for (int t = threadIdx.x; t < N; t += blockDim.x) {
            const int qi = (qb0 + j) * PFT_QB + t / G, hq = h * G + t % G;
            float mv = 0.f, lv = 1.f;
            if (qi < a.S) {
                const float* sp = a.stats + (((size_t)b * a.Hq + hq) * a.S + qi) * 2;
                mv = sp[0];
                lv = sp[1];
            }
            s_st[(buf * N + t) * 2] = mv;
            s_st[(buf * N + t) * 2 + 1] = lv;
        }
    };
    load_stats(0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = s_taddr;
    const uint32_t idesc = umma_idesc_f16(DT == QV_BF16, 128, N, 0, 0);
    if (threadIdx.x == 0) {
        prefetch_tensormap(&mK);
        prefetch_tensormap(&mQg);
        mbar_arrive_expect_tx(&bar_q[0], NS * PFT_SLAB + NS * qslab);
        for (int s = 0; s < NS; ++s) {
            tma_load_4d(sK + s * PFT_SLAB, &mK, 64 * s, h, k0, b, &bar_q[0]);
            tma_load_4d(sQ + s * qslab, &mQg, 64 * s, h * G, qb0 * PFT_QB, b, &bar_q[0]);
        }
    }
    float acc = 0.f, chunk = 0.f;
    int cur = (qb0 * PFT_QB) / PFT_CHUNK;
    bool ok = true;
    for (int j = 0; j < nqb; ++j) {
        const int st = j & 1;
        if (threadIdx.x == 0) {
            if (j + 1 < nqb) {
                mbar_arrive_expect_tx(&bar_q[st ^ 1], NS * qslab);
                for (int s = 0; s < NS; ++s)
                    tma_load_4d(sQ + ((st ^ 1) * NS + s) * qslab, &mQg, 64 * s, h * G, (qb0 + j + 1) * PFT_QB, b,
                                &bar_q[st ^ 1]);
            }
            if (pft_wait(&bar_q[st], (j >> 1) & 1, a.err)) {
                tc_fence_after();
                const uint32_t ka = smem_u32(sK), qa = smem_u32(sQ + st * NS * qslab);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(taddr, umma_desc_sw128(pft_kmajor_step<D>(ka, kk), 16, 1024),
                             umma_desc_sw128(qa + (uint32_t)((kk >> 2) * qslab + (kk & 3) * 32), 16, 1024), idesc,
                             kk > 0);
            }
            umma_commit(&bar_s);
        }
        if (j + 1 < nqb) load_stats(j + 1, st ^ 1);
        __syncwarp();
        ok = ok && pft_wait(&bar_s, j & 1, a.err);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        const float* stt = s_st + st * N * 2;
        for (int c0 = 0; c0 < N; c0 += 32) {
            float v[32];
            if (ok) {
                tmem_ld32(taddr + ((uint32_t)(32 * warp) << 16) + c0, v);
                tmem_wait_ld();
            }
            // G consecutive columns are one query's heads (G divides 32)
            for (int c = 0; c < 32; c += G) {
                const int qi = (qb0 + j) * PFT_QB + (c0 + c) / G;
                if (qi >= a.S) break;
                const int ch = qi / PFT_CHUNK;
                if (ch != cur) {
                    acc += rnd<DT>(chunk);
                    chunk = 0.f;
                    cur = ch;
                }
                if (!ok || key > qi || key >= a.S) continue;
                float ps = 0.f;
                for (int gi = 0; gi < G; ++gi) {
                    const int n = c0 + c + gi;
                    const float lg = div_r<DT>(rnd<DT>(v[c + gi]), sqrt_d);
                    ps += rnd<DT>(expf(lg - stt[2 * n]) / stt[2 * n + 1]);
                }
                chunk += rnd<DT>(ps / (float)G);
            }
        }
        tc_fence_before();
        __syncthreads();
    }
    acc += rnd<DT>(chunk);
    if (key < a.S) a.colsum[((size_t)b * a.H + h) * a.S + key] = acc;
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, 256);
}

// ---------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 pft_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// [B][S][heads][D] as a 4-D tensor (D, heads, S, B); box (64, box_heads, box_rows, 1)
static bool pft_map(CUtensorMap* m, const void* base, int dt, int D, int heads, int S, int B, int box_heads,
                    int box_rows) {
    auto fn = pft_encode();
    if (!fn) return false;
    const cuuint64_t e = 2;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)S, (cuuint64_t)B};
    cuuint64_t strides[3] = {D * e, (cuuint64_t)heads * D * e, (cuuint64_t)S * heads * D * e};
    cuuint32_t box[4] = {64, (cuuint32_t)box_heads, (cuuint32_t)box_rows, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = fn(m, dt == QV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                    const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool pft_supported(const Geo& g) {
    return (g.dt == QV_BF16 || g.dt == QV_F16) && (g.D == 64 || g.D == 128) &&
           (g.G == 1 || g.G == 2 || g.G == 4 || g.G == 8);
}

template <int DT, int D>
static int pft_launch_t(const Geo& g, const void* q, const void* k, const void* v, int S, void* out, float* colsum,
                        float* stats, int* err, cudaStream_t s) {
    const int Hq = g.H * g.G;
    CUtensorMap mQ, mK, mV, mQg;
    if (!pft_map(&mQ, q, DT, D, Hq, S, g.B, 1, PFT_ROWS) || !pft_map(&mK, k, DT, D, g.H, S, g.B, 1, PFT_ROWS) ||
        !pft_map(&mV, v, DT, D, g.H, S, g.B, 1, PFT_ROWS) || !pft_map(&mQg, q, DT, D, Hq, S, g.B, g.G, PFT_QB))
        return QV_EINVAL;
    PftArgs a;
    a.S = S; a.B = g.B; a.H = g.H; a.G = g.G; a.Hq = Hq;
    a.stats = stats; a.out = out; a.colsum = colsum; a.err = err;
    constexpr int NS = D / 64;
    const size_t sm_stats = 1024 + 3 * NS * PFT_SLAB;
    const size_t sm_out = 1024 + 5 * NS * PFT_SLAB + 2 * PFT_SLAB;
    const size_t sm_col = 1024 + NS * PFT_SLAB + 2 * NS * (size_t)PFT_QB * g.G * 128 + 2 * PFT_QB * g.G * 2 * 4;
    static int c1 = 48 * 1024, c2 = 48 * 1024, c3 = 48 * 1024;
    cudaError_t e = ensure_smem(pft_stats_kernel<DT, D>, sm_stats, &c1);
    if (e == cudaSuccess) e = ensure_smem(pft_out_kernel<DT, D>, sm_out, &c2);
    if (e == cudaSuccess) e = ensure_smem(pft_colsum_kernel<DT, D>, sm_col, &c3);
    if (e != cudaSuccess) return set_cuda_error(e);
    const dim3 gq((S + PFT_ROWS - 1) / PFT_ROWS, Hq, g.B);
    pft_stats_kernel<DT, D><<<gq, 128, sm_stats, s>>>(mQ, mK, a);
    pft_out_kernel<DT, D><<<gq, 128, sm_out, s>>>(mQ, mK, mV, a);
    if (colsum) {
        const dim3 gk((S + PFT_ROWS - 1) / PFT_ROWS, g.H, g.B);
        pft_colsum_kernel<DT, D><<<gk, 128, sm_col, s>>>(mK, mQg, a);
    }
    return check_launch();
}

int pft_launch(const Geo& g, const void* q, const void* k, const void* v, int S, void* out, float* colsum,
               float* stats, int* err, cudaStream_t s) {
    if (g.dt == QV_BF16)
        return g.D == 128 ? pft_launch_t<QV_BF16, 128>(g, q, k, v, S, out, colsum, stats, err, s)
                          : pft_launch_t<QV_BF16, 64>(g, q, k, v, S, out, colsum, stats, err, s);
    return g.D == 128 ? pft_launch_t<QV_F16, 128>(g, q, k, v, S, out, colsum, stats, err, s)
                      : pft_launch_t<QV_F16, 64>(g, q, k, v, S, out, colsum, stats, err, s);
}

}  // namespace qv
