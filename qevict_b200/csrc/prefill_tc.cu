// Prefill lane on the 5th-generation tensor cores (tcgen05 + TMEM), bf16/fp16.
//
// Same results as the CUDA-core kernels of prefill_attn.cu (which remain for
// fp32): causal attention output and the per-key column sums the reference's
// chunked scorer produces (src/models/attention/ops_flash.py:56-141):
// logits rounded like the reference (q.k rounded to the KV dtype, / sqrt(D)
// rounded, src/models/attention/ops.py:23-46), fp32 softmax statistics per
// query row, probabilities rounded to the KV dtype, group mean rounded, sums
// over each 512-query chunk rounded, chunks accumulated in fp32.
//
// Warp-specialised kernels.  Each tile CTA has ten warps: eight compute warps
// (two per TMEM lane quarter, each owning half of a tile's 128 columns), one
// TMA warp and one MMA warp (one elected thread each).  The score tile S is
// double-buffered in TMEM, so the tensor cores compute tile j+1 while the
// compute warps round, exponentiate and reduce tile j; operands stream through
// multi-stage shared-memory rings guarded by mbarriers.  Every wait is bounded
// and also gives up at once when another CTA has raised the error word.
// Operand tiles are 4-D TMA boxes (64 elements x rows) with the 128-byte
// swizzle, the canonical K-major / MN-major UMMA layout.
//
//   pft_stats_kernel   one CTA per (128-query tile, query head): S = Q.K^T per
//                      128-key tile (M = queries, N = keys); running max and
//                      sum of exp of the rounded logits per row -> (max,
//                      1 / sum) in the stats buffer [B][H][S][G][2].
//   pft_attn_kernel    one CTA per (block of 128 / G queries, KV head), rows =
//                      (query, group head): the same S tiles; P rounded to the
//                      KV dtype in shared memory; O += P.V and the group sums
//                      P^T.W on the tensor cores; per (query block, key) the
//                      sum of the rounded group means -> partials.
//   pft_chunk_kernel   per key: the partials of each 512-query chunk summed and
//                      rounded, chunks accumulated in fp32 -> column sums.
//
// Arithmetic the compute warps rely on:
// * the division by sqrt(D) is a multiply by the fp32 reciprocal: for every
//   bf16 input (and every fp16 input at D = 64) round(round(x) * (1/sqrt(D)))
//   equals round(round(x) / sqrt(D)) exactly; fp16 at D = 128 adds one
//   residual correction (q' = q + (x - q*sqrt(D)) / sqrt(D), two FMAs), which
//   makes it equal in value for all 65536 inputs.  tests/test_prefill_rounding.py
//   checks both identities over every 16-bit input;
// * exp(x) is ex2.approx(x * log2(e)) on x = l - max (exact: both are values
//   of the KV dtype); its few-ulp fp32 error only moves a probability across
//   a rounding boundary of the KV dtype, which the lane's parity bounds allow.
#include <cudaTypedefs.h>
#include <math.h>

#include "common.cuh"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace qv {

constexpr int PFT_ROWS = 128;        // queries (stats/out) or keys (colsum) per tile
constexpr int PFT_SLAB = 16384;      // one 64-element x 128-row swizzled slab
constexpr int PFT_CHUNK = 512;       // queries per rounded chunk of the scorer
constexpr int PFT_CW = 8;            // compute warps
constexpr int PFT_TMA_WARP = PFT_CW;
constexpr int PFT_MMA_WARP = PFT_CW + 1;
constexpr int PFT_THREADS = 32 * (PFT_CW + 2);
constexpr int PFT_ACW = 8;           // compute warps of pft_attn_kernel (a multiple of 4)
constexpr float PFT_LOG2E = 1.4426950408889634f;

struct PftArgs {
    int S, B, H, G, Hq;
    float* stats;                    // [B][H][S][G][2]: max, 1 / sum
    void* out;                       // [B][S][Hq][D]
    float* partial;                  // [B][H] x triangle: query block j holds keys [0, (j+1) * QB)
    int* err;                        // device error word (QV_DERR_TIMEOUT)
};

// Bounded wait: false after about a second (raising the error word), or at
// once when another CTA has raised it.
__device__ __noinline__ bool pft_wait_slow(uint64_t* bar, uint32_t parity, int* err) {
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int*>(err) != 0) return false;
        if (global_ns() - t0 > 1000000000ull) {
            atomicOr(err, QV_DERR_TIMEOUT);
            return false;
        }
    }
}
__device__ __forceinline__ bool pft_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    return pft_wait_slow(bar, parity, err);
}

template <int D>
__device__ __forceinline__ uint32_t pft_kmajor_step(uint32_t base, int kk) {
    // k-step kk (16 elements) of a K-major operand stored as D/64 slabs
    return base + (uint32_t)((kk >> 2) * PFT_SLAB + (kk & 3) * 32);
}

__device__ __forceinline__ float pft_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32x2 arithmetic (sm_100): two lanes of a 64-bit register pair.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ void pft_named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Two fp32 values rounded to the KV dtype (one packed conversion), and back.
template <int DT> __device__ __forceinline__ uint32_t pft_pack(float hi, float lo) {
    uint32_t p;
    if (DT == QV_BF16)
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
    else
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
    return p;
}
template <int DT> __device__ __forceinline__ void pft_unpack(uint32_t p, float& hi, float& lo) {
    if (DT == QV_BF16) {
        hi = __uint_as_float(p & 0xFFFF0000u);
        lo = __uint_as_float(p << 16);
    } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&p);
        hi = __high2float(h);
        lo = __low2float(h);
    }
}

// Packed maximum of two KV-dtype pairs, and a packed -inf.
template <int DT> __device__ __forceinline__ uint32_t pft_max2(uint32_t a, uint32_t b) {
    uint32_t d;
    if (DT == QV_BF16)
        asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else
        asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
template <int DT> __device__ __forceinline__ uint32_t pft_ninf() { return DT == QV_BF16 ? 0xFF80u : 0xFC00u; }

// The reference's logits of an fp32 accumulator pair, round(round(x) / sqrt(D)),
// packed in the KV dtype (x0 in the low half).  inv2 = 1/sqrt(D) twice,
// nsd2 = -sqrt(D) twice (the fp16, D = 128 residual step).
template <int DT, int D>
__device__ __forceinline__ uint32_t pft_logit2(float x0, float x1, uint64_t inv2, uint64_t nsd2) {
    float r0, r1;
    pft_unpack<DT>(pft_pack<DT>(x1, x0), r1, r0);
    const uint64_t r = f2_pack(r0, r1);
    uint64_t q = f2_mul(r, inv2);
    if (DT == QV_F16 && D != 64) q = f2_fma(f2_fma(q, nsd2, r), inv2, q);
    float q0, q1;
    f2_unpack(q, q0, q1);
    return pft_pack<DT>(q1, q0);
}

// One score tile's 64 columns of a row, statistics pass: running max m and
// sum l of exp(logit - m).  DIAG: keys above the row's query are masked.
template <int DT, int D, bool DIAG>
__device__ __forceinline__ void pft_stats_tile(const float* v, int kbase, int qi, uint64_t inv2, uint64_t nsd2,
                                               float& m, float& l) {
    uint32_t lg[32];
    uint32_t mx2 = pft_ninf<DT>() * 0x10001u;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        uint32_t x = pft_logit2<DT, D>(v[2 * j], v[2 * j + 1], inv2, nsd2);
        if (DIAG) {
            if (kbase + 2 * j > qi) x = (x & 0xFFFF0000u) | pft_ninf<DT>();
            if (kbase + 2 * j + 1 > qi) x = (x & 0xFFFFu) | (pft_ninf<DT>() << 16);
        }
        lg[j] = x;
        mx2 = pft_max2<DT>(mx2, x);
    }
    float mh, ml;
    pft_unpack<DT>(mx2, mh, ml);
    const float mn = fmaxf(m, fmaxf(mh, ml));
    if (mn > -INFINITY) {
        const uint64_t mn2 = f2_pack(mn, mn), l2e = f2_pack(PFT_LOG2E, PFT_LOG2E);
        uint64_t ps2 = f2_pack(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float a, b, d0, d1;
            pft_unpack<DT>(lg[j], b, a);
            f2_unpack(f2_mul(f2_sub(f2_pack(a, b), mn2), l2e), d0, d1);
            ps2 = f2_add(ps2, f2_pack(pft_ex2(d0), pft_ex2(d1)));
        }
        float p0, p1;
        f2_unpack(ps2, p0, p1);
        l = l * pft_ex2((m - mn) * PFT_LOG2E) + (p0 + p1);
        m = mn;
    }
}

// NC columns of a row of one score tile, output pass: P = exp(logit - m) / sum
// rounded to the KV dtype, packed in pairs (w[j] = keys 2j, 2j+1).
template <int DT, int D, bool DIAG, int NC>
__device__ __forceinline__ void pft_prob_tile(const float* v, int kbase, int qi, uint64_t inv2, uint64_t nsd2,
                                              uint64_t m2, uint64_t li2, uint32_t* w) {
    const uint64_t l2e = f2_pack(PFT_LOG2E, PFT_LOG2E);
#pragma unroll
    for (int j = 0; j < NC / 2; ++j) {
        float a, b, d0, d1, p0, p1;
        pft_unpack<DT>(pft_logit2<DT, D>(v[2 * j], v[2 * j + 1], inv2, nsd2), b, a);
        f2_unpack(f2_mul(f2_sub(f2_pack(a, b), m2), l2e), d0, d1);
        f2_unpack(f2_mul(f2_pack(pft_ex2(d0), pft_ex2(d1)), li2), p0, p1);
        if (DIAG) {
            if (kbase + 2 * j > qi) p0 = 0.f;
            if (kbase + 2 * j + 1 > qi) p1 = 0.f;
        }
        w[j] = pft_pack<DT>(p1, p0);
    }
}

// ---------------------------------------------------------------- stats
template <int DT, int D>
__global__ void __launch_bounds__(PFT_THREADS, 2) pft_stats_kernel(const __grid_constant__ CUtensorMap mQ,
                                                                   const __grid_constant__ CUtensorMap mK, PftArgs a) {
    constexpr int NS = D / 64;                   // slabs per operand tile
    constexpr int KST = 2;                       // K stages (two CTAs share an SM)
    extern __shared__ unsigned char pft_raw[];
    unsigned char* sm = pft_raw + ((1024u - (smem_u32(pft_raw) & 1023u)) & 1023u);
    unsigned char* sQ = sm;                      // [NS]
    unsigned char* sK = sm + NS * PFT_SLAB;      // [KST][NS]
    __shared__ __align__(8) uint64_t bar_q, kfull[KST], kempty[KST], sfull[2], sempty[2], done;
    __shared__ float red[PFT_ROWS][2];
    __shared__ uint32_t s_taddr;
    const int qt = gridDim.x - 1 - blockIdx.x;   // longest rows first
    const int hq = blockIdx.y, b = blockIdx.z;
    const int h = hq / a.G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = qt * PFT_ROWS;
    const int nkt = qt + 1;
    int* err = a.err;

    if (warp == PFT_MMA_WARP) { tmem_alloc(&s_taddr, 256); tmem_relinquish(); }
    if (threadIdx.x == 0) {
        mbar_init(&bar_q, 1);
        for (int s = 0; s < KST; ++s) { mbar_init(&kfull[s], 1); mbar_init(&kempty[s], 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&sfull[s], 1); mbar_init(&sempty[s], PFT_CW); }
        mbar_init(&done, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = s_taddr;

    if (warp == PFT_TMA_WARP) {
        if (lane == 0) {
            prefetch_tensormap(&mQ);
            prefetch_tensormap(&mK);
            mbar_arrive_expect_tx(&bar_q, NS * PFT_SLAB);
            for (int s = 0; s < NS; ++s) tma_load_4d(sQ + s * PFT_SLAB, &mQ, 64 * s, hq, q0, b, &bar_q);
            int issued = 0;
            bool ok = true;
            for (int kt = 0; kt < nkt; ++kt) {
                const int st = kt % KST;
                if (kt >= KST) ok = ok && pft_wait(&kempty[st], (kt / KST - 1) & 1, err);
                if (!ok) break;
                mbar_arrive_expect_tx(&kfull[st], NS * PFT_SLAB);
                for (int s = 0; s < NS; ++s)
                    tma_load_4d(sK + (st * NS + s) * PFT_SLAB, &mK, 64 * s, h, kt * PFT_ROWS, b, &kfull[st]);
                issued = kt + 1;
            }
            // the copies this thread issued have landed before the CTA exits
            mbar_wait_bounded(&bar_q, 0);
            for (int kt = issued - KST > 0 ? issued - KST : 0; kt < issued; ++kt)
                mbar_wait_bounded(&kfull[kt % KST], (kt / KST) & 1);
        }
    } else if (warp == PFT_MMA_WARP) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(DT == QV_BF16, 128, 128, 0, 0);
            bool ok = pft_wait(&bar_q, 0, err);
            for (int kt = 0; kt < nkt && ok; ++kt) {
                const int st = kt % KST, bf = kt & 1;
                ok = pft_wait(&kfull[st], (kt / KST) & 1, err);
                if (ok && kt >= 2) ok = pft_wait(&sempty[bf], ((kt >> 1) - 1) & 1, err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + st * NS * PFT_SLAB);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(taddr + bf * 128, umma_desc_sw128(pft_kmajor_step<D>(qa, kk), 16, 1024),
                             umma_desc_sw128(pft_kmajor_step<D>(ka, kk), 16, 1024), idesc, kk > 0);
                umma_commit(&sfull[bf]);
                umma_commit(&kempty[st]);
            }
            // no MMA is in flight when the TMEM is released
            umma_commit(&done);
            mbar_wait_bounded(&done, 0);
        }
    } else {
        const int q4 = warp & 3, hf = warp >> 2;
        const int r = 32 * q4 + lane;
        const int qi = q0 + r;
        const int c0 = 64 * hf;
        const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
        const float sd = sqrtf((float)D), inv = 1.f / sd;
        const uint64_t inv2 = f2_pack(inv, inv), nsd2 = f2_pack(-sd, -sd);
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int kt = 0; kt < nkt; ++kt) {
            const int bf = kt & 1;
            ok = ok && pft_wait(&sfull[bf], (kt >> 1) & 1, err);
            ok = __all_sync(0xffffffffu, ok);     // TMEM loads are warp-collective
            if (!ok) break;
            tc_fence_after();
            float v[64];
            tmem_ld32(taddr + lane_off + bf * 128 + c0, v);
            tmem_ld32(taddr + lane_off + bf * 128 + c0 + 32, v + 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[bf]);
            const int kbase = kt * PFT_ROWS + c0;
            if (kt == qt) pft_stats_tile<DT, D, true>(v, kbase, qi, inv2, nsd2, m, l);
            else pft_stats_tile<DT, D, false>(v, kbase, qi, inv2, nsd2, m, l);
        }
        // the two column halves of a row combine
        if (hf == 1) { red[r][0] = m; red[r][1] = l; }
        pft_named_sync(1, 32 * PFT_CW);
        if (hf == 0 && qi < a.S) {
            const float m1 = red[r][0], l1 = red[r][1];
            const float mm = fmaxf(m, m1);
            const float ll = l * pft_ex2((m - mm) * PFT_LOG2E) + l1 * pft_ex2((m1 - mm) * PFT_LOG2E);
            float* sp = a.stats + ((((size_t)b * a.H + h) * a.S + qi) * a.G + (hq - h * a.G)) * 2;
            sp[0] = mm;
            sp[1] = ll > 0.f ? 1.f / ll : 0.f;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == PFT_MMA_WARP) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(taddr, 256);
    }
}

// ---------------------------------------------------------------- output + column-sum partials
// Row tile: QB = 128 / G queries x the G heads of KV head h (row r is query
// q0 + r / G, head h*G + r % G), so one CTA holds every head of a query and
// forms the scorer's group mean from the same rounded probabilities that feed
// P.V.  Per key tile: S = Q.K^T into TMEM (double-buffered); P = exp(l - max)
// / sum rounded to the KV dtype, written swizzled to shared memory; then two
// MMAs read P: O += P.V (V MN-major) and, for the column sums, the group sums
// Gs[key][query] = P^T.W with W[row][query] = 1 when the row belongs to the
// query (P^T as an MN-major operand).  The compute warps turn Gs into the
// rounded group means, sum them over the block's queries and store one partial
// per (query block, key); pft_chunk_kernel folds those into the 512-query
// chunk sums.
template <int DT, int D, int G, bool CS>
__global__ void __launch_bounds__(32 * (PFT_ACW + 2), 1) pft_attn_kernel(const __grid_constant__ CUtensorMap mQg,
                                                                  const __grid_constant__ CUtensorMap mK,
                                                                  const __grid_constant__ CUtensorMap mV, PftArgs a) {
    using T = typename Elt<DT>::T;
    constexpr int NS = D / 64;
    constexpr int QB = PFT_ROWS / G;                 // queries per block
    // W: N = QB columns selecting each query's G rows; with G = 1 the block's
    // partial is the plain column sum of P, one column of ones (N = 16)
    constexpr int NW = G == 1 ? 16 : QB;
    constexpr int WSLAB = NW * 128;                  // one 64-element slab of W (NW rows)
    constexpr int CW = PFT_ACW, NT = 32 * (CW + 2);  // compute warps, threads
    constexpr int TMA_W = CW, MMA_W = CW + 1;        // the TMA and MMA warps
    constexpr int NPART = CW / 4;                    // compute warps per TMEM lane quarter
    constexpr int NC = PFT_ROWS / NPART;             // score columns per compute warp
    constexpr int HCOL = G == 1 ? 1 : QB / NPART;    // Gs columns per compute warp
    constexpr int HC = D / NPART;                    // output columns per compute warp
    extern __shared__ unsigned char pft_raw[];
    unsigned char* sm = pft_raw + ((1024u - (smem_u32(pft_raw) & 1023u)) & 1023u);
    unsigned char* sQ = sm;                          // [NS]
    unsigned char* sK = sQ + NS * PFT_SLAB;          // [2][NS]
    unsigned char* sV = sK + 2 * NS * PFT_SLAB;      // [2][NS]
    unsigned char* sP = sV + 2 * NS * PFT_SLAB;      // 2 slabs: 128 rows x 128 keys
    unsigned char* sW = sP + 2 * PFT_SLAB;           // 2 slabs of NW rows (column sums only)
    __shared__ __align__(8) uint64_t bar_q, kfull[2], kempty[2], vfull[2], vempty[2], sfull[2], sempty[2];
    __shared__ __align__(8) uint64_t pfull, pempty, ofull, done;
    __shared__ float red[2][NPART - 1][PFT_ROWS];
    __shared__ uint32_t s_taddr;
    const int qb = gridDim.x - 1 - blockIdx.x;       // longest rows first
    const int h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = qb * QB;
    const int qend = min(q0 + QB, a.S);              // the block's queries: [q0, qend)
    const int nkt = (qend - 1) / PFT_ROWS + 1;       // only the last key tile crosses the diagonal
    int* err = a.err;

    if (warp == MMA_W) { tmem_alloc(&s_taddr, 512); tmem_relinquish(); }
    if (threadIdx.x == 0) {
        mbar_init(&bar_q, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kfull[s], 1); mbar_init(&kempty[s], 1);
            mbar_init(&vfull[s], 1); mbar_init(&vempty[s], 1);
            mbar_init(&sfull[s], 1); mbar_init(&sempty[s], CW);
        }
        mbar_init(&pfull, CW); mbar_init(&pempty, 1); mbar_init(&ofull, 1); mbar_init(&done, 1);
        fence_barrier_init();
    }
    if (CS) {
        // W, K-major (K = the 128 rows), 128-byte swizzle: stored 16-byte chunk sc
        // of row n holds the row's logical chunk sc ^ (n & 7)
        const uint32_t one = DT == QV_BF16 ? 0x3F80u : 0x3C00u;
        for (int i = threadIdx.x; i < 2 * WSLAB / 16; i += NT) {
            const int s = i / (WSLAB / 16), rem = i % (WSLAB / 16), n = rem >> 3, sc = rem & 7;
            const int kb = s * 64 + ((sc ^ (n & 7)) << 3);
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const bool s0 = G == 1 ? n == 0 : (kb + 2 * e) / G == n;
                const bool s1 = G == 1 ? n == 0 : (kb + 2 * e + 1) / G == n;
                w[e] = (s0 ? one : 0u) | (s1 ? one << 16 : 0u);
            }
            *reinterpret_cast<uint4*>(sW + s * WSLAB + n * 128 + sc * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = s_taddr;   // S: [0, 256) as two buffers; O: [256, 256 + D); Gs: [384, 384 + QB)

    if (warp == TMA_W) {
        if (lane == 0) {
            prefetch_tensormap(&mQg);
            prefetch_tensormap(&mK);
            prefetch_tensormap(&mV);
            mbar_arrive_expect_tx(&bar_q, NS * PFT_SLAB);
            for (int s = 0; s < NS; ++s) tma_load_4d(sQ + s * PFT_SLAB, &mQg, 64 * s, h * G, q0, b, &bar_q);
            int ik = 0, iv = 0;
            bool ok = true;
            for (int kt = 0; kt < nkt; ++kt) {
                const int st = kt & 1;
                if (kt >= 2) ok = ok && pft_wait(&kempty[st], ((kt >> 1) - 1) & 1, err);
                if (!ok) break;
                mbar_arrive_expect_tx(&kfull[st], NS * PFT_SLAB);
                for (int s = 0; s < NS; ++s)
                    tma_load_4d(sK + (st * NS + s) * PFT_SLAB, &mK, 64 * s, h, kt * PFT_ROWS, b, &kfull[st]);
                ik = kt + 1;
                if (kt >= 2) ok = ok && pft_wait(&vempty[st], ((kt >> 1) - 1) & 1, err);
                if (!ok) break;
                mbar_arrive_expect_tx(&vfull[st], NS * PFT_SLAB);
                for (int s = 0; s < NS; ++s)
                    tma_load_4d(sV + (st * NS + s) * PFT_SLAB, &mV, 64 * s, h, kt * PFT_ROWS, b, &vfull[st]);
                iv = kt + 1;
            }
            // the copies this thread issued have landed before the CTA exits
            mbar_wait_bounded(&bar_q, 0);
            for (int kt = ik - 2 > 0 ? ik - 2 : 0; kt < ik; ++kt) mbar_wait_bounded(&kfull[kt & 1], (kt >> 1) & 1);
            for (int kt = iv - 2 > 0 ? iv - 2 : 0; kt < iv; ++kt) mbar_wait_bounded(&vfull[kt & 1], (kt >> 1) & 1);
        }
    } else if (warp == MMA_W) {
        if (lane == 0) {
            const uint32_t id_s = umma_idesc_f16(DT == QV_BF16, 128, 128, 0, 0);
            const uint32_t id_o = umma_idesc_f16(DT == QV_BF16, 128, D, 0, 1);
            const uint32_t id_g = umma_idesc_f16(DT == QV_BF16, 128, NW, 1, 0);
            bool ok = pft_wait(&bar_q, 0, err);
            for (int kt = 0; kt <= nkt && ok; ++kt) {
                if (kt < nkt) {                  // S(kt) = Q.K(kt)^T
                    const int st = kt & 1;
                    ok = pft_wait(&kfull[st], (kt >> 1) & 1, err);
                    if (ok && kt >= 2) ok = pft_wait(&sempty[st], ((kt >> 1) - 1) & 1, err);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + st * NS * PFT_SLAB);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        umma_f16(taddr + st * 128, umma_desc_sw128(pft_kmajor_step<D>(qa, kk), 16, 1024),
                                 umma_desc_sw128(pft_kmajor_step<D>(ka, kk), 16, 1024), id_s, kk > 0);
                    umma_commit(&sfull[st]);
                    umma_commit(&kempty[st]);
                }
                if (kt >= 1) {                   // tile j = kt - 1: O += P.V, Gs = P^T.W
                    const int j = kt - 1, st = j & 1;
                    ok = pft_wait(&pfull, j & 1, err);
                    if (ok) ok = pft_wait(&vfull[st], (j >> 1) & 1, err);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t pa = smem_u32(sP), va = smem_u32(sV + st * NS * PFT_SLAB);
#pragma unroll
                    for (int kk = 0; kk < PFT_ROWS / 16; ++kk)
                        umma_f16(taddr + 256, umma_desc_sw128(pft_kmajor_step<128>(pa, kk), 16, 1024),
                                 umma_desc_sw128(va + kk * 2048, PFT_SLAB, 1024), id_o, (j > 0 || kk > 0) ? 1 : 0);
                    if (CS) {
                        const uint32_t wa = smem_u32(sW);
#pragma unroll
                        for (int kk = 0; kk < PFT_ROWS / 16; ++kk)
                            umma_f16(taddr + 384, umma_desc_sw128(pa + kk * 2048, PFT_SLAB, 1024),
                                     umma_desc_sw128(wa + (kk >> 2) * WSLAB + (kk & 3) * 32, 16, 1024), id_g,
                                     kk > 0);
                    }
                    umma_commit(&pempty);
                    umma_commit(&vempty[st]);
                }
            }
            if (ok) umma_commit(&ofull);
            // no MMA is in flight when the TMEM is released
            umma_commit(&done);
            mbar_wait_bounded(&done, 0);
        }
    } else {
        const int q4 = warp & 3, part_id = warp >> 2;
        const int r = 32 * q4 + lane;
        const int qi = q0 + r / G;
        const int c0 = NC * part_id;
        const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
        const float sd = sqrtf((float)D), inv = 1.f / sd;
        const uint64_t inv2 = f2_pack(inv, inv), nsd2 = f2_pack(-sd, -sd);
        float m = 0.f, linv = 0.f;                   // outside the sequence: p = 0
        if (qi < a.S) {
            const float* sp = a.stats + ((((size_t)b * a.H + h) * a.S + qi) * G + r % G) * 2;
            m = sp[0];
            linv = sp[1];
        }
        float* part_row = nullptr;                   // this block's row of column-sum partials
        if (CS) {
            const int n = (a.S + QB - 1) / QB;
            const size_t per_head = (size_t)QB * n * (n + 1) / 2;
            part_row = a.partial + ((size_t)b * a.H + h) * per_head + (size_t)QB * qb * (qb + 1) / 2;
        }
        // column-sum partials of key tile t from Gs (every compute warp calls this
        // once per tile, failed or not, so the named barrier always pairs up)
        auto cs_tile = [&](bool okk, int t) {
            const int key = t * PFT_ROWS + r;
            if constexpr (G == 1) {
                // the block's sum of P for this key, one warp per lane quarter
                if (part_id == 0 && okk) {
                    tc_fence_after();
                    float gv[4];
                    tmem_ld4(taddr + lane_off + 384, gv);
                    tmem_wait_ld();
                    if (key < qend) part_row[key] = gv[0];
                }
                tc_fence_before();
                return;
            }
            float part = 0.f;
            if (okk) {
                tc_fence_after();
                float gv[HCOL];
                const uint32_t ga = taddr + lane_off + 384 + part_id * HCOL;
                if constexpr (HCOL == 64) { tmem_ld32(ga, gv); tmem_ld32(ga + 32, gv + 32); }
                else if constexpr (HCOL == 32) tmem_ld32(ga, gv);
                else if constexpr (HCOL == 16) tmem_ld16(ga, gv);
                else if constexpr (HCOL == 8) tmem_ld8(ga, gv);
                else tmem_ld4(ga, gv);
                tmem_wait_ld();
                const uint64_t g2 = f2_pack(1.f / G, 1.f / G);
                uint64_t acc2 = f2_pack(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < HCOL; c += 2) {
                    float a0, a1, r0, r1;
                    f2_unpack(f2_mul(f2_pack(gv[c], gv[c + 1]), g2), a0, a1);
                    pft_unpack<DT>(pft_pack<DT>(a1, a0), r1, r0);
                    acc2 = f2_add(acc2, f2_pack(r0, r1));
                }
                float s0, s1;
                f2_unpack(acc2, s0, s1);
                part = s0 + s1;
            }
            tc_fence_before();
            if (part_id > 0) red[t & 1][part_id - 1][r] = part;
            pft_named_sync(1, 32 * CW);
            if (part_id == 0 && okk && key < qend) {
#pragma unroll
                for (int u = 0; u < NPART - 1; ++u) part += red[t & 1][u][r];
                part_row[key] = part;
            }
        };
        bool ok = true;
        for (int kt = 0; kt < nkt; ++kt) {
            const int bf = kt & 1;
            uint32_t w[NC / 2];
            if (ok) ok = pft_wait(&sfull[bf], (kt >> 1) & 1, err);
            ok = __all_sync(0xffffffffu, ok);       // TMEM loads are warp-collective
            if (ok) {
                tc_fence_after();
                float v[NC];
                tmem_ld32(taddr + lane_off + bf * 128 + c0, v);
                if constexpr (NC == 64) tmem_ld32(taddr + lane_off + bf * 128 + c0 + 32, v + 32);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[bf]);
                const int kbase = kt * PFT_ROWS + c0;
                const uint64_t m2 = f2_pack(m, m), li2 = f2_pack(linv, linv);
                if (kt == nkt - 1) pft_prob_tile<DT, D, true, NC>(v, kbase, qi, inv2, nsd2, m2, li2, w);
                else pft_prob_tile<DT, D, false, NC>(v, kbase, qi, inv2, nsd2, m2, li2, w);
            }
            if (kt >= 1) {
                // P(kt-1) has been read by its MMAs before P(kt) overwrites it
                if (ok) ok = pft_wait(&pempty, (kt - 1) & 1, err);
                ok = __all_sync(0xffffffffu, ok);
                if (CS) cs_tile(ok, kt - 1);
            }
            if (ok) {
                // columns c0 .. c0 + NC of row r: 16-byte chunks of its 64-key
                // slab, 128-byte swizzle
                unsigned char* prow = sP + (c0 >> 6) * PFT_SLAB + r * 128;
                const int ch0 = (c0 & 63) >> 3;
#pragma unroll
                for (int ch = 0; ch < NC / 8; ++ch)
                    *reinterpret_cast<uint4*>(prow + (((ch0 + ch) ^ (r & 7)) << 4)) =
                        make_uint4(w[4 * ch], w[4 * ch + 1], w[4 * ch + 2], w[4 * ch + 3]);
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&pfull);
            }
        }
        if (ok) ok = pft_wait(&ofull, 0, err);
        ok = __all_sync(0xffffffffu, ok);
        if (CS) cs_tile(ok, nkt - 1);
        if (ok) {
            tc_fence_after();
            constexpr int OC = HC < 32 ? HC : 32;        // columns per TMEM load
            T* orow = reinterpret_cast<T*>(a.out) + (((size_t)b * a.S + qi) * a.Hq + h * G + r % G) * D + part_id * HC;
#pragma unroll
            for (int c = 0; c < HC; c += OC) {
                float v[OC];
                if constexpr (OC == 32) tmem_ld32(taddr + lane_off + 256 + part_id * HC + c, v);
                else tmem_ld16(taddr + lane_off + 256 + part_id * HC + c, v);
                tmem_wait_ld();
                if (qi < a.S) {
#pragma unroll
                    for (int i = 0; i < OC; i += 8) {
                        uint4 u;
                        u.x = pft_pack<DT>(v[i + 1], v[i]);
                        u.y = pft_pack<DT>(v[i + 3], v[i + 2]);
                        u.z = pft_pack<DT>(v[i + 5], v[i + 4]);
                        u.w = pft_pack<DT>(v[i + 7], v[i + 6]);
                        *reinterpret_cast<uint4*>(orow + c + i) = u;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_W) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(taddr, 512);
    }
}

// Column sums from the partials: per key, the blocks of each 512-query chunk
// summed in order and rounded to the KV dtype, chunks accumulated in fp32
// (blocks that end before the key hold nothing for it and are not read).
template <int DT>
__global__ void pft_chunk_kernel(const float* __restrict__ partial, float* __restrict__ colsum, int S, int H,
                                 int QB) {
    const int key = blockIdx.x * blockDim.x + threadIdx.x;
    const int h = blockIdx.y, b = blockIdx.z;
    if (key >= S) return;
    const int n = (S + QB - 1) / QB;
    const float* base = partial + ((size_t)b * H + h) * ((size_t)QB * n * (n + 1) / 2);
    const int bpc = PFT_CHUNK / QB;
    int j = key / QB;
    float acc = 0.f;
    while (j < n) {
        const int cend = min((j / bpc + 1) * bpc, n);
        float s = 0.f;
        for (; j < cend; ++j) s += base[(size_t)QB * j * (j + 1) / 2 + key];
        acc += rnd<DT>(s);
    }
    colsum[((size_t)b * H + h) * S + key] = acc;
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

// Bytes of the column-sum partials: per (sequence, KV head) a triangle of
// n (n + 1) / 2 rows of QB keys, n = ceil(S / QB), QB = 128 / G.
size_t pft_partial_bytes(const Geo& g, int S) {
    const size_t QB = PFT_ROWS / g.G, n = (S + QB - 1) / QB;
    return (size_t)g.B * g.H * (QB * n * (n + 1) / 2) * sizeof(float);
}

template <int DT, int D, int G, bool CS>
static cudaError_t pft_attn_launch(const CUtensorMap& mQg, const CUtensorMap& mK, const CUtensorMap& mV,
                                   const PftArgs& a, cudaStream_t s) {
    constexpr int NS = D / 64;
    const size_t bytes = 1024 + 5 * NS * (size_t)PFT_SLAB + 2 * PFT_SLAB + (CS ? 2 * (G == 1 ? 16 : PFT_ROWS / G) * 128 : 0);
    static int c = 48 * 1024;
    cudaError_t e = ensure_smem(pft_attn_kernel<DT, D, G, CS>, bytes, &c);
    if (e != cudaSuccess) return e;
    const dim3 grid((a.S + PFT_ROWS / G - 1) / (PFT_ROWS / G), a.H, a.B);
    pft_attn_kernel<DT, D, G, CS><<<grid, 32 * (PFT_ACW + 2), bytes, s>>>(mQg, mK, mV, a);
    return cudaSuccess;
}

template <int DT, int D, int G>
static cudaError_t pft_attn_g(const CUtensorMap& mQg, const CUtensorMap& mK, const CUtensorMap& mV,
                              const PftArgs& a, float* colsum, cudaStream_t s) {
    if (!colsum) return pft_attn_launch<DT, D, G, false>(mQg, mK, mV, a, s);
    cudaError_t e = pft_attn_launch<DT, D, G, true>(mQg, mK, mV, a, s);
    if (e != cudaSuccess) return e;
    const dim3 grid((a.S + 255) / 256, a.H, a.B);
    pft_chunk_kernel<DT><<<grid, 256, 0, s>>>(a.partial, colsum, a.S, a.H, PFT_ROWS / G);
    return cudaSuccess;
}

template <int DT, int D>
static int pft_launch_t(const Geo& g, const void* q, const void* k, const void* v, int S, void* out, float* colsum,
                        float* stats, float* partial, int* err, cudaStream_t s) {
    const int Hq = g.H * g.G;
    CUtensorMap mQ, mK, mV, mQg;
    if (!pft_map(&mQ, q, DT, D, Hq, S, g.B, 1, PFT_ROWS) || !pft_map(&mK, k, DT, D, g.H, S, g.B, 1, PFT_ROWS) ||
        !pft_map(&mV, v, DT, D, g.H, S, g.B, 1, PFT_ROWS) ||
        !pft_map(&mQg, q, DT, D, Hq, S, g.B, g.G, PFT_ROWS / g.G))
        return QV_EINVAL;
    PftArgs a;
    a.S = S; a.B = g.B; a.H = g.H; a.G = g.G; a.Hq = Hq;
    a.stats = stats; a.out = out; a.partial = partial; a.err = err;
    constexpr int NS = D / 64;
    const size_t sm_stats = 1024 + 3 * NS * PFT_SLAB;
    static int c1 = 48 * 1024;
    cudaError_t e = ensure_smem(pft_stats_kernel<DT, D>, sm_stats, &c1);
    if (e != cudaSuccess) return set_cuda_error(e);
    const dim3 gq((S + PFT_ROWS - 1) / PFT_ROWS, Hq, g.B);
    pft_stats_kernel<DT, D><<<gq, PFT_THREADS, sm_stats, s>>>(mQ, mK, a);
    switch (g.G) {
        case 1: e = pft_attn_g<DT, D, 1>(mQg, mK, mV, a, colsum, s); break;
        case 2: e = pft_attn_g<DT, D, 2>(mQg, mK, mV, a, colsum, s); break;
        case 4: e = pft_attn_g<DT, D, 4>(mQg, mK, mV, a, colsum, s); break;
        default: e = pft_attn_g<DT, D, 8>(mQg, mK, mV, a, colsum, s); break;
    }
    if (e != cudaSuccess) return set_cuda_error(e);
    return check_launch();
}

int pft_launch(const Geo& g, const void* q, const void* k, const void* v, int S, void* out, float* colsum,
               float* stats, float* partial, int* err, cudaStream_t s) {
    if (g.dt == QV_BF16)
        return g.D == 128 ? pft_launch_t<QV_BF16, 128>(g, q, k, v, S, out, colsum, stats, partial, err, s)
                          : pft_launch_t<QV_BF16, 64>(g, q, k, v, S, out, colsum, stats, partial, err, s);
    return g.D == 128 ? pft_launch_t<QV_F16, 128>(g, q, k, v, S, out, colsum, stats, partial, err, s)
                      : pft_launch_t<QV_F16, 64>(g, q, k, v, S, out, colsum, stats, partial, err, s);
}

}  // namespace qv
