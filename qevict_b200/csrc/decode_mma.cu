// Decode attention, tensor-core version for the production shape
// (head_dim 128, omega 64, sink a multiple of 64, BF16/FP16 KV, INT8 Q-cache).
//
// Same semantics as decode_split_kernel (decode.cu) -- see that file for the
// reference citations -- restructured for B200:
//
//   * Persistent CTAs, one per SM.  The (sequence, KV head) work is flattened
//     into equal-byte items (32-token main-zone tiles, 64-token Q-cache windows)
//     split into contiguous ranges, one per CTA.
//   * One producer warp streams items through a ring of shared-memory stages
//     with 2-D TMA tiles (128-byte swizzle, no multicast) and 1-D bulk copies for
//     the Q-cache scales; every mbarrier wait is bounded.  Items holding no live
//     token (empty sticky / Q slots) are never fetched.
//   * Eight (or, for CTAs with many items, ten) consumer warps each take whole
//     items, round-robin, and run both
//     products on the tensor cores with the GQA group in the MMA's N dimension:
//     S^T[tok, head] = K[tok, :] . Q^T  and  O^T[d, head] += V^T[d, tok] . P^T,
//     P^T obtained from the S^T accumulators by movmatrix.  BF16 P is split into
//     hi + lo halves (two MMAs) so the products carry ~16 mantissa bits of P.
//   * INT8 Q-cache windows feed f16 MMAs directly: a code byte c becomes the
//     f16 value 1024 + c with one byte-permute; the per-channel K scale is
//     folded into Q, the per-token V scale into P, and the 1024 offset and the
//     zero points are added back as per-head corrections (exact fp32
//     dequantisation; see QV_FLAG_REFERENCE_ROUNDING for the reference's own).
//   * Logits are rounded like the reference's (q.k rounded to the KV dtype,
//     / sqrt(D) rounded) and written for the ledger fold; each CTA merges its
//     warps into one partial per (sequence, head, zone).  A second kernel
//     (decode_combine_kernel, chained with programmatic dependent launch)
//     merges the partials, writes the output and folds the exact probabilities
//     into the vote ledger and the Q-window scores.
#include <cudaTypedefs.h>
#include <math.h>

#include "codec.cuh"
#include "ptx.cuh"

namespace qv {

// Consumer warps per CTA: MM_CW_WIDE when a CTA holds many items (more warps
// in flight hide the per-warp latency of the MMA / conversion chains: 2.6 %
// faster at the batch-64 microbenchmark than 8 warps), MM_CW_NARROW when it
// holds few (small batch; as many warps as items).
#ifndef QV_MM_CW_WIDE
#define QV_MM_CW_WIDE 10
#endif
#ifndef QV_MM_CW_NARROW
#define QV_MM_CW_NARROW 8
#endif
constexpr int MM_CW_NARROW = QV_MM_CW_NARROW;
constexpr int MM_CW_WIDE = QV_MM_CW_WIDE;
static_assert(MM_CW_WIDE >= MM_CW_NARROW && MM_CW_WIDE <= 12, "consumer warps");
// Consumer warps that share one item: each takes an equal run of its tokens
// (main-zone tile: 2 m-tiles of 16 tokens; Q window: 4), so a stage is held
// for a fraction of an item's compute time and more stages stay in flight.
#ifndef QV_MM_SPLIT
#define QV_MM_SPLIT 2
#endif
constexpr int MM_SPLIT = QV_MM_SPLIT;
static_assert(MM_SPLIT == 1 || MM_SPLIT == 2, "warps per item");
static_assert(MM_CW_NARROW % MM_SPLIT == 0 && MM_CW_WIDE % MM_SPLIT == 0, "whole warp groups");
constexpr int MM_STAGE = 17408;                // bytes per stage (17 KB, 1024-aligned)
constexpr int MM_MAXNS = 12;                   // max pipeline stages
constexpr int MM_G = 8;                        // max GQA group
constexpr int MM_SKIPMAP = 2048;               // items whose skip flag is cached in smem
constexpr int MM_MT = 32;                      // tokens per main-zone item

struct MmPlan {
    int n_main;       // main items per (b, h): S_cap / 32
    int n_q;          // Q windows per (b, h)
    int ipb;          // items per (b, h)
    long long total;  // items overall
    int nC;           // CTAs (<= total, so every CTA owns at least one item)
    int pmax;         // partial slots per (b, h, zone)
    int ns;           // pipeline stages
    int cw;           // consumer warps per CTA
};

__host__ __device__ inline int mm_cta_of(const MmPlan& P, long long i) {
    // 32-bit division whenever the product fits (every practical size)
    if ((unsigned long long)P.total * (unsigned)P.nC < (1ull << 32))
        return (int)((unsigned)i * (unsigned)P.nC / (unsigned)P.total);
    return (int)(i * P.nC / P.total);
}
__host__ __device__ inline long long mm_first_item(const MmPlan& P, int c) {
    return ((long long)c * P.total + P.nC - 1) / P.nC;  // smallest i with i * nC / total >= c
}
__device__ inline void mm_zone_ctas(const MmPlan& P, long long bh, int zone, int* first, int* count) {
    const long long a = bh * P.ipb + (zone ? P.n_main : 0);
    const long long e = bh * P.ipb + (zone ? P.ipb : P.n_main);
    if (e <= a) { *first = 0; *count = 0; return; }
    *first = mm_cta_of(P, a);
    *count = mm_cta_of(P, e - 1) - *first + 1;
}

// Liveness of main-zone position pos (used by the combine kernel's fold).
__device__ __forceinline__ bool mm_live(const Geo& g, const int32_t* swid, int pos, int cw, int tv) {
    if (pos < g.sink) return true;
    const int r = pos - g.sink;
    const int slot = r / g.om;
    if (slot < g.kw) return swid[slot] >= 0;
    const int rs = slot - g.kw;
    const int L0 = cw - (g.R - 1);
    const int w = L0 + ((rs - (L0 % g.R)) % g.R + g.R) % g.R;
    return w < cw || (r % g.om) < tv;
}

// Liveness of a token of a fetched main item without touching memory: sink and
// sticky items are fetched only when occupied, so all their tokens are live; in
// the ring only the unwritten tail of the current window is dead.
__device__ __forceinline__ bool mm_item_live(const Geo& g, int pos, int cw, int tv) {
    const int rb = g.ring_base();
    if (pos < rb) return true;
    const int rs = (pos - rb) >> 6;
    const int L0 = cw - (g.R - 1);
    const int w = L0 + ((rs - (L0 % g.R)) % g.R + g.R) % g.R;
    return w < cw || ((pos - rb) & 63) < tv;
}

__device__ __forceinline__ bool mm_skip(const Geo& g, const qv_layer& L, const MmPlan& P, long long bh, int j) {
    if (j >= P.n_main) return L.q_wid[bh * g.qw + (j - P.n_main)] < 0;
    const int pos = j * MM_MT;
    if (pos < g.sink) return false;
    const int s = (pos - g.sink) >> 6;
    return s < g.kw && L.sticky_wid[bh * g.kw + s] < 0;
}

template <int DT> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<QV_BF16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<QV_F16>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <int DT> __device__ __forceinline__ void mma_kv(float* c, const uint32_t* a, const uint32_t* b);
template <> __device__ __forceinline__ void mma_kv<QV_BF16>(float* c, const uint32_t* a, const uint32_t* b) { mma_bf16(c, a, b); }
template <> __device__ __forceinline__ void mma_kv<QV_F16>(float* c, const uint32_t* a, const uint32_t* b) { mma_f16(c, a, b); }

__device__ __forceinline__ float f16r(float x) { return __half2float(__float2half_rn(x)); }

// byte offset of (row, 16-byte chunk) in a 128-byte-row tile written by a
// 128B-swizzled TMA box (the box starts on a 1024-byte boundary)
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return (uint32_t)(row * 128 + (((chunk ^ (row & 7)) & 7) << 4));
}

template <int CW>
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory"); }

// x / sqrt(128) correctly rounded in fp32: product with the rounded reciprocal,
// then one fused correction with the exact residual (Markstein's method).
__device__ __forceinline__ float div_sqrt128(float x) {
    const float c = 11.313708305358887f;         // fp32 nearest to sqrt(128)
    const float r = 0.0883883461356163f;         // fp32 nearest to 1/sqrt(128)
    const float q0 = __fmul_rn(x, r);
    const float res = __fmaf_rn(-q0, c, x);
    return __fmaf_rn(res, r, q0);
}

template <int DT>
__device__ __forceinline__ float logit_round(float dot) {
    return rnd<DT>(div_sqrt128(rnd<DT>(dot)));
}

// Sum over the G heads of one token's probabilities, each rounded to the KV
// dtype: sum_h rnd(exp(logit_h - M_h) / L_h).  row = the token's G rounded logits.
template <int DT>
__device__ __forceinline__ float bits_to_f(uint32_t b16);
template <> __device__ __forceinline__ float bits_to_f<QV_BF16>(uint32_t b16) { return __uint_as_float(b16 << 16); }
template <> __device__ __forceinline__ float bits_to_f<QV_F16>(uint32_t b16) {
    return __half2float(__ushort_as_half((unsigned short)b16));
}
template <int DT>
__device__ __forceinline__ float group_prob_sum(const typename Elt<DT>::T* row, int G, const float* sM, const float* sL) {
    float acc = 0.f;
    if (G == 4) {
        const uint2 u = __ldcg(reinterpret_cast<const uint2*>(row));
        acc += rnd<DT>(__expf(bits_to_f<DT>(u.x & 0xffffu) - sM[0]) / sL[0]);
        acc += rnd<DT>(__expf(bits_to_f<DT>(u.x >> 16) - sM[1]) / sL[1]);
        acc += rnd<DT>(__expf(bits_to_f<DT>(u.y & 0xffffu) - sM[2]) / sL[2]);
        acc += rnd<DT>(__expf(bits_to_f<DT>(u.y >> 16) - sM[3]) / sL[3]);
    } else {
        for (int hh = 0; hh < G; ++hh) acc += rnd<DT>(__expf(Elt<DT>::f(row[hh]) - sM[hh]) / sL[hh]);
    }
    return acc;
}

// The same for G = 4 from the token's four logits already loaded as a uint2.
template <int DT>
__device__ __forceinline__ float group_prob_sum4(uint2 u, const float* sM, const float* sL) {
    float acc = rnd<DT>(__expf(bits_to_f<DT>(u.x & 0xffffu) - sM[0]) / sL[0]);
    acc += rnd<DT>(__expf(bits_to_f<DT>(u.x >> 16) - sM[1]) / sL[1]);
    acc += rnd<DT>(__expf(bits_to_f<DT>(u.y & 0xffffu) - sM[2]) / sL[2]);
    acc += rnd<DT>(__expf(bits_to_f<DT>(u.y >> 16) - sM[3]) / sL[3]);
    return acc;
}

// Shared scratch of one combine unit, in floats: per-head partial maxima and
// weights [G][2*64], per-head totals and one liveness code per 64-token block
// of the unit.
constexpr int MM_CMB_MAXBLK = 1024;
constexpr int MM_CMB_MAXP = 128;   // partials per (sequence, head, zone): CTAs covering one zone
constexpr int MM_CMB_SMEM = 2 * MM_G * 2 * MM_CMB_MAXP + 2 * MM_G + MM_CMB_MAXBLK / 4;

// One combine unit of one (sequence, KV head) bh: the per-CTA partials'
// maxima and sums give the head totals; with OUT, this unit's slice of the
// output (each element the weighted sum of the partials in slot order --
// main zone, then Q zone -- so results do not depend on timing, rounded the
// way the reference rounds out_main, out_q and their sum, ops.py:150); with
// FOLD, the exact probabilities of this unit's 64-token blocks folded into the
// vote ledger / Q-window scores (tally_decode_scores, eviction_manager.py:198-203;
// accumulate_scores, quantize_manager.py:101-111).  Run by nthr threads
// (tid < nthr, nthr a multiple of 32 and >= 32*G) that synchronise with
// sync(); N0 is the token count the attention pass saw (new token included).
// Written for latency: a thread issues the global loads of its first round of
// work (partial maxima, partial outputs, logits, ledger entries) together
// before using any.
template <int DT, bool OUT, bool FOLD, typename Sync>
__device__ __forceinline__ void combine_unit(const Geo& g, const qv_layer& L, void* __restrict__ out,
                                             const float* __restrict__ partial, const void* __restrict__ logits,
                                             const MmPlan& P, int N0, long long bh, int chunk, int nchunks,
                                             int blocks_per_chunk, float* sm, int tid, int nthr, Sync sync) {
    constexpr int MAXP = MM_CMB_MAXP;
    constexpr int RW = 4;   // work items per thread per round
    constexpr int XP = 16;  // partial outputs of one element loaded per round
    float(*s_m)[2 * MAXP] = reinterpret_cast<float(*)[2 * MAXP]>(sm);             // maxima, then weights
    float(*s_l)[2 * MAXP] = reinterpret_cast<float(*)[2 * MAXP]>(sm + MM_G * 2 * MAXP);
    float* s_M = sm + 2 * MM_G * 2 * MAXP;
    float* s_L = s_M + MM_G;
    unsigned char* s_live = reinterpret_cast<unsigned char*>(s_L + MM_G);
    using T = typename Elt<DT>::T;
    const int n_mblk = g.S_cap / 64;              // 64-token main blocks, then one per Q window
    const int n_blk = n_mblk + g.qw;
    const int b = (int)(bh / g.H), h = (int)(bh % g.H);
    const int G = g.G;
    const int cw = (N0 - g.sink) / g.om;
    const int tv = (N0 - g.sink) % g.om + 1;
    const size_t S_tot = (size_t)g.S_cap + (size_t)g.qw * g.om;
    int f0, c0, f1, c1;
    mm_zone_ctas(P, bh, 0, &f0, &c0);
    mm_zone_ctas(P, bh, 1, &f1, &c1);
    const int np = c0 + c1;
    const float* pz0 = partial + ((size_t)bh * 2 + 0) * P.pmax * G * 130;
    const float* pz1 = partial + ((size_t)bh * 2 + 1) * P.pmax * G * 130;
    auto prow = [&](int s) { return s < c0 ? pz0 + (size_t)s * G * 130 : pz1 + (size_t)(s - c0) * G * 130; };
    const int blk0 = chunk * blocks_per_chunk;
    const int blk1 = min(blk0 + blocks_per_chunk, n_blk);
    const int ne = G * 128;
    const int per = (ne + nchunks - 1) / nchunks;
    const int e0 = min(chunk * per, ne), e1 = min(e0 + per, ne);
    const int p_beg = blk0 * 64, p_end = min(blk1, n_mblk) * 64;
    const T* lg = reinterpret_cast<const T*>(logits) + (size_t)bh * S_tot * G;
    float* votes = L.votes + bh * g.S_cap;
    const int warp = tid >> 5, lane = tid & 31;
    const int q_blk = max(blk0, n_mblk) + warp;       // this warp's first Q window block

    // ---- (A) issue every first-round load
    float pm = -INFINITY, pl = 0.f;
    const int am = tid < G * np ? tid : -1;
    if (am >= 0) {
        const float* pr = prow(am % np) + (am / np) * 130;
        pm = __ldcg(pr);
        pl = __ldcg(pr + 1);
    }
    float xo[XP];
    const int el_first = e0 + tid;
    if (OUT && el_first < e1) {
        const int hh = el_first >> 7, d = el_first & 127;
#pragma unroll
        for (int u = 0; u < XP; ++u) xo[u] = u < np ? __ldcg(prow(u) + hh * 130 + 2 + d) : 0.f;
    }
    int32_t live_src = 1;
    const int sink_blk = g.sink / 64, ring_blk = (g.sink + g.kw * g.om) / 64;
    const int lb = blk0 + tid;
    uint2 dl[RW];
    float dv[RW];
    uint2 el2[2] = {make_uint2(0, 0), make_uint2(0, 0)};
    if (FOLD) {
        if (lb < blk1) {
            if (lb >= sink_blk && lb < ring_blk) live_src = __ldcg(L.sticky_wid + bh * g.kw + (lb - sink_blk));
            else if (lb >= n_mblk) live_src = __ldcg(L.q_wid + bh * g.qw + (lb - n_mblk));
        }
#pragma unroll
        for (int u = 0; u < RW; ++u) {
            const int pos = p_beg + tid + u * nthr;
            if (pos < p_end) {
                dl[u] = G == 4 ? __ldcg(reinterpret_cast<const uint2*>(lg + (size_t)pos * G)) : make_uint2(0, 0);
                dv[u] = votes[pos];
            }
        }
        if (G == 4 && q_blk < blk1) {
            const T* wl = lg + ((size_t)g.S_cap + (size_t)(q_blk - n_mblk) * 64) * G;
            el2[0] = __ldcg(reinterpret_cast<const uint2*>(wl + (size_t)lane * G));
            el2[1] = __ldcg(reinterpret_cast<const uint2*>(wl + (size_t)(lane + 32) * G));
        }
    }
    // ---- first uses: partial maxima / sums and the block liveness codes
    //      (0 = no live token, 1 = all live, 2 = live below offset tv)
    if (am >= 0) {
        s_m[am / np][am % np] = pm;
        s_l[am / np][am % np] = pl;
    }
    // heads spread over many CTAs (few sequences x heads): more partials than threads
    for (int a2 = tid + nthr; a2 < G * np; a2 += nthr) {
        const float* pr = prow(a2 % np) + (a2 / np) * 130;
        s_m[a2 / np][a2 % np] = __ldcg(pr);
        s_l[a2 / np][a2 % np] = __ldcg(pr + 1);
    }
    if (FOLD) {
        for (int blk = lb; blk < blk1; blk += nthr) {
            if (blk != lb) {   // units with more blocks than threads
                live_src = 1;
                if (blk >= sink_blk && blk < ring_blk) live_src = L.sticky_wid[bh * g.kw + (blk - sink_blk)];
                else if (blk >= n_mblk) live_src = L.q_wid[bh * g.qw + (blk - n_mblk)];
            }
            unsigned char code;
            if (blk < sink_blk) code = 1;
            else if (blk < ring_blk || blk >= n_mblk) code = live_src >= 0;
            else code = mm_item_live(g, blk * 64 + 63, cw, 0) ? 1 : 2;
            s_live[blk - blk0] = code;
        }
    }
    sync();
    // ---- (B) one warp per head: total maximum, normaliser, per-partial weights
    if (warp < G) {
        const int hh = warp;
        float M = -INFINITY;
        for (int s2 = lane; s2 < np; s2 += 32) M = fmaxf(M, s_m[hh][s2]);
        M = warp_max(M);
        float Ls = 0.f;
        for (int s2 = lane; s2 < np; s2 += 32) {
            const float ms = s_m[hh][s2];
            const float w = ms > -INFINITY ? __expf(ms - M) : 0.f;
            Ls += s_l[hh][s2] * w;
            s_m[hh][s2] = w;
        }
        Ls = warp_sum(Ls);
        if (lane == 0) { s_M[hh] = M; s_L[hh] = Ls; }
    }
    sync();
    // ---- (C) output slice: every partial of an element added in slot order
    if (OUT) {
        const bool has_q = L.seq[b * 4 + 1] > 0;
        for (int el = el_first; el < e1; el += nthr) {
            const int hh = el >> 7, d = el & 127;
            const float* w = s_m[hh];
            float om_ = 0.f, oq = 0.f;
            for (int base = 0; base < np; base += XP) {
                if (base > 0 || el != el_first) {
#pragma unroll
                    for (int u = 0; u < XP; ++u) xo[u] = base + u < np ? __ldcg(prow(base + u) + hh * 130 + 2 + d) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < XP; ++u) {
                    const int s2 = base + u;
                    if (s2 < c0) om_ = fmaf(xo[u], w[s2], om_);
                    else if (s2 < np) oq = fmaf(xo[u], w[s2], oq);
                }
            }
            const float inv = 1.f / s_L[hh];
            const float r = has_q ? add_r<DT>(rnd<DT>(om_ * inv), rnd<DT>(oq * inv)) : rnd<DT>(om_ * inv);
            st<DT>(out, ((size_t)b * g.H * G + (size_t)h * G + hh) * 128 + d, r);
        }
    }
    if (FOLD) {
        // ---- (D) main-zone tokens: exact probabilities into the vote ledger
        for (int base = p_beg + tid; base < p_end; base += RW * nthr) {
            if (base != p_beg + tid) {
#pragma unroll
                for (int u = 0; u < RW; ++u) {
                    const int pos = base + u * nthr;
                    if (pos < p_end) {
                        dl[u] = G == 4 ? __ldcg(reinterpret_cast<const uint2*>(lg + (size_t)pos * G)) : make_uint2(0, 0);
                        dv[u] = votes[pos];
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < RW; ++u) {
                const int pos = base + u * nthr;
                if (pos >= p_end) continue;
                const int code = s_live[(pos >> 6) - blk0];
                if (!(code == 1 || (code == 2 && (pos & 63) < tv))) continue;
                const float acc = G == 4 ? group_prob_sum4<DT>(dl[u], s_M, s_L)
                                         : group_prob_sum<DT>(lg + (size_t)pos * G, G, s_M, s_L);
                votes[pos] = dv[u] + rnd<DT>(acc / (float)G);
            }
        }
        // ---- (E) Q windows: one warp per window, two tokens per lane
        for (int blk = q_blk; blk < blk1; blk += nthr >> 5) {
            const int slot = blk - n_mblk;
            const T* wl = lg + ((size_t)g.S_cap + (size_t)slot * 64) * G;
            if (blk != q_blk && G == 4) {
                el2[0] = __ldcg(reinterpret_cast<const uint2*>(wl + (size_t)lane * G));
                el2[1] = __ldcg(reinterpret_cast<const uint2*>(wl + (size_t)(lane + 32) * G));
            }
            if (!s_live[blk - blk0]) continue;
            const float a0 = G == 4 ? group_prob_sum4<DT>(el2[0], s_M, s_L)
                                    : group_prob_sum<DT>(wl + (size_t)lane * G, G, s_M, s_L);
            const float a1 = G == 4 ? group_prob_sum4<DT>(el2[1], s_M, s_L)
                                    : group_prob_sum<DT>(wl + (size_t)(lane + 32) * G, G, s_M, s_L);
            float a = rnd<DT>(a0 / (float)G) + rnd<DT>(a1 / (float)G);
            a = warp_sum(a);
            if (lane == 0) L.q_score[bh * g.qw + slot] += rnd<DT>(a);
        }
    }
    sync();   // the scratch is reused by the next unit
}

struct BlockSync {
    __device__ void operator()() const { __syncthreads(); }
};
template <int DT, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
decode_mma_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ CUtensorMap tmKQ, const __grid_constant__ CUtensorMap tmVQ,
                  Geo g, qv_layer L, const void* __restrict__ q, int* tickets, float* partial,
                  void* logits, MmPlan P) {
    using T = typename Elt<DT>::T;
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned base (128-byte-swizzled TMA boxes); offsetting the
    // shared array itself keeps every derived pointer a shared-memory pointer,
    // so the compiler emits shared (not generic) loads, stores and atomics
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int NS = P.ns;
    const int G = g.G;
    unsigned char* stages = smem;
    // per-warp segment states, double-buffered by segment parity
    float* s_wo = reinterpret_cast<float*>(smem + NS * MM_STAGE);       // [2][CW][G][128]
    float* s_wm = s_wo + 2 * CW * G * 128;                           // [2][CW][8]
    float* s_wl = s_wm + 2 * CW * MM_G;                              // [2][CW][8]
    int* s_cnt = reinterpret_cast<int*>(s_wl + 2 * CW * MM_G);       // [2] arrivals, [2] merges done
    uint64_t* full = reinterpret_cast<uint64_t*>(s_cnt + 4);
    uint64_t* empty = full + MM_MAXNS;
    unsigned char* s_skip = reinterpret_cast<unsigned char*>(empty + MM_MAXNS);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const long long i0 = mm_first_item(P, c), i1 = mm_first_item(P, c + 1);
    const size_t S_tot = (size_t)g.S_cap + (size_t)g.qw * g.om;
    const int e = (int)sizeof(T);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MM_SPLIT);
        }
        fence_barrier_init();
        s_cnt[0] = s_cnt[1] = s_cnt[2] = s_cnt[3] = 0;
    }
    // Which of this CTA's items hold no live token (the slot tables are not
    // written by the kernel that precedes this one, so read them before the wait).
    for (long long i = i0 + threadIdx.x; i < i1 && i - i0 < MM_SKIPMAP; i += blockDim.x)
        s_skip[i - i0] = mm_skip(g, L, P, i / P.ipb, (int)(i % P.ipb)) ? 1 : 0;
    __syncthreads();
    auto skipped = [&](long long i) -> bool {
        return i - i0 < MM_SKIPMAP ? s_skip[i - i0] != 0 : mm_skip(g, L, P, i / P.ipb, (int)(i % P.ipb));
    };
    // The preceding kernel (RoPE + append) writes q and one new token per
    // (sequence, KV head), at token index N0 of the ring; the token counter, the
    // slot tables and every other cached token are final before it starts.  So
    // the producer streams all other items before waiting for it, and only the
    // item holding the new token, and the consumers' read of q, wait.
    const int N0 = L.step[0];
    const int cw = (N0 - g.sink) / g.om;
    const int tv = (N0 - g.sink) % g.om + 1;
    const int j_new = (g.ring_base() + (cw % g.R) * 64 + tv - 1) / MM_MT;

    // --------------------------------------------------------------- producer
    if (warp == CW) {
        if (lane == 0 && i0 < i1) {
            prefetch_tensormap(&tmK);
            prefetch_tensormap(&tmV);
            prefetch_tensormap(&tmKQ);
            prefetch_tensormap(&tmVQ);
            bool waited = false;
            int k = 0;
            long long bh = i0 / P.ipb;
            int j = (int)(i0 % P.ipb) - 1;
#pragma unroll 1
            for (long long i = i0; i < i1; ++i, ++k) {
                // item i takes stage slot k = i - i0 (round robin), fetched or not
                if (++j == P.ipb) { j = 0; ++bh; }
                const int s = k % NS;
                if (k >= NS && !mbar_wait_bounded(&empty[s], ((k / NS) - 1) & 1)) {
                    set_err(L.err, QV_DERR_LAYOUT);
                    break;
                }
                if (skipped(i)) {
                    // no live token: the slot completes without a transfer
                    mbar_arrive(&full[s]);
                    continue;
                }
                if (j == j_new && !waited) {
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    waited = true;
                }
                unsigned char* st = stages + s * MM_STAGE;
                if (j < P.n_main) {
                    mbar_arrive_expect_tx(&full[s], 16384);
                    const int y = (int)(bh * g.S_cap + MM_MT * j);
                    tma_load_2d(st, &tmK, 0, y, &full[s]);
                    tma_load_2d(st + 4096, &tmK, 64, y, &full[s]);
                    tma_load_2d(st + 8192, &tmV, 0, y, &full[s]);
                    tma_load_2d(st + 12288, &tmV, 64, y, &full[s]);
                } else {
                    const size_t sw = (size_t)bh * g.qw + (j - P.n_main);
                    mbar_arrive_expect_tx(&full[s], 16384 + 2 * 128 * e + 2 * 64 * e);
                    tma_load_2d(st, &tmKQ, 0, (int)(sw * 64), &full[s]);
                    tma_load_2d(st + 8192, &tmVQ, 0, (int)(sw * 64), &full[s]);
                    bulk_load(st + 16384, reinterpret_cast<const char*>(L.ks) + sw * 128 * e, 128 * e, &full[s]);
                    bulk_load(st + 16384 + 256, reinterpret_cast<const char*>(L.kz) + sw * 128 * e, 128 * e, &full[s]);
                    bulk_load(st + 16384 + 512, reinterpret_cast<const char*>(L.vs) + sw * 64 * e, 64 * e, &full[s]);
                    bulk_load(st + 16384 + 640, reinterpret_cast<const char*>(L.vz) + sw * 64 * e, 64 * e, &full[s]);
                }
            }
        }
        return;
    }

    // --------------------------------------------------------------- consumers
    const int gq = lane >> 2, t4 = lane & 3, mi = lane >> 3;
    uint32_t bq[8][2];            // Q^T fragments (main zone)
    uint32_t qq[8][2];            // the same q values in the Q-cache layout (see load_q)
    float o[8][4];                // O^T accumulators: 8 d-tiles x (2 rows x 2 heads)
    float m[2], ls[2], spp[2], svz[2];
    long long cur_bh = -1;
    bool ok = true;
    T* lgp = reinterpret_cast<T*>(logits);

    auto reset_acc = [&]() {
#pragma unroll
        for (int dt = 0; dt < 8; ++dt)
#pragma unroll
            for (int r = 0; r < 4; ++r) o[dt][r] = 0.f;
        m[0] = m[1] = -INFINITY;
        ls[0] = ls[1] = spp[0] = spp[1] = svz[0] = svz[1] = 0.f;
    };

    // q is written by the preceding kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Q^T fragments straight from global memory, per warp (no CTA barrier):
    // lane (gq, t4) holds q[gq][16kk + 2t4 + {0,1}] and q[gq][16kk + 2t4 + {8,9}]
    auto load_q = [&](long long bh) {
        const int b = (int)(bh / g.H), h = (int)(bh % g.H);
        const uint32_t* qr = reinterpret_cast<const uint32_t*>(
            reinterpret_cast<const T*>(q) + ((size_t)b * g.H * G + (size_t)h * G + (gq < G ? gq : 0)) * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            bq[kk][0] = gq < G ? __ldcg(qr + 8 * kk + t4) : 0u;
            bq[kk][1] = gq < G ? __ldcg(qr + 8 * kk + t4 + 4) : 0u;
        }
        // Q-cache windows need q[gq][16kk + 4t4 + 0..3] per lane: pairs held by
        // quad lanes (2t4) & 3 and its neighbour, in register t4 >> 1
        const int srcA = (lane & ~3) | ((2 * t4) & 3);
        const bool hi_reg = (t4 >> 1) != 0;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint32_t r0 = __shfl_sync(0xffffffffu, bq[kk][0], srcA);
            const uint32_t r1 = __shfl_sync(0xffffffffu, bq[kk][1], srcA);
            const uint32_t r2 = __shfl_sync(0xffffffffu, bq[kk][0], srcA + 1);
            const uint32_t r3 = __shfl_sync(0xffffffffu, bq[kk][1], srcA + 1);
            qq[kk][0] = hi_reg ? r1 : r0;
            qq[kk][1] = hi_reg ? r3 : r2;
        }
    };

    // End of a segment (the items of one (b, h, zone) in this CTA's range) for
    // this warp: its softmax state goes to a shared slot, and the last of the
    // CTA's warps to arrive merges the slots and writes the CTA's partial.
    // No CTA-wide barrier: warps move on to the next segment at once.  Slots
    // are double-buffered by segment parity; a warp two segments ahead waits
    // (bounded) until the older segment has been merged.
    int seg = 0;
    auto flush = [&](int key, bool final_seg) {
        const long long bh = key >> 1;
        const int zone = key & 1;
        const int p = seg & 1;
        if (lane == 0) {
            volatile int* done = s_cnt + 2 + p;
            if (*done < (seg >> 1)) {
                const uint64_t t0 = global_ns();
                while (*done < (seg >> 1)) {
                    if (global_ns() - t0 > 2000000000ull) {
                        set_err(L.err, QV_DERR_LAYOUT);
                        break;
                    }
                }
            }
        }
        __syncwarp();
#pragma unroll
        for (int col = 0; col < 2; ++col) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                ls[col] += __shfl_xor_sync(0xffffffffu, ls[col], off);
                spp[col] += __shfl_xor_sync(0xffffffffu, spp[col], off);
                svz[col] += __shfl_xor_sync(0xffffffffu, svz[col], off);
            }
        }
        float* wo = s_wo + ((size_t)p * CW + warp) * G * 128;
#pragma unroll
        for (int col = 0; col < 2; ++col) {
            const int hh = 2 * t4 + col;
            if (hh < G) {
                if (gq == 0) {
                    s_wm[(p * CW + warp) * MM_G + hh] = m[col];
                    s_wl[(p * CW + warp) * MM_G + hh] = ls[col];
                }
#pragma unroll
                for (int dt = 0; dt < 8; ++dt) {
                    float va = o[dt][col], vb = o[dt][2 + col];
                    int da, db;
                    if (zone == 0) { da = 16 * dt + gq; db = da + 8; }
                    else {
                        da = 16 * dt + 2 * gq; db = da + 1;
                        va = (va - 1024.f * spp[col]) * (1.f / 1024.f) + svz[col];
                        vb = (vb - 1024.f * spp[col]) * (1.f / 1024.f) + svz[col];
                    }
                    wo[hh * 128 + da] = va;
                    wo[hh * 128 + db] = vb;
                }
            }
        }
        if (final_seg) {
            // the CTA's last segment: every warp is here, so merge with all threads
            consumer_sync<CW>();
            int first, cnt;
            mm_zone_ctas(P, bh, zone, &first, &cnt);
            float* part = partial + (((size_t)bh * 2 + zone) * P.pmax + (c - first)) * G * 130;
            const float* wm = s_wm + p * CW * MM_G;
            const float* wl = s_wl + p * CW * MM_G;
            const float* wo0 = s_wo + (size_t)p * CW * G * 128;
            for (int idx = threadIdx.x; idx < G * 128; idx += CW * 32) {
                const int hh = idx >> 7, d = idx & 127;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < CW; ++w) M = fmaxf(M, wm[w * MM_G + hh]);
                float acc = 0.f, lsum = 0.f;
#pragma unroll
                for (int w = 0; w < CW; ++w) {
                    const float mw = wm[w * MM_G + hh];
                    if (mw == -INFINITY) continue;
                    const float ew = __expf(mw - M);
                    acc += wo0[((size_t)w * G + hh) * 128 + d] * ew;
                    lsum += wl[w * MM_G + hh] * ew;
                }
                part[hh * 130 + 2 + d] = acc;
                if (d == 0) { part[hh * 130] = M; part[hh * 130 + 1] = lsum; }
            }
            ++seg;
            return;
        }
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(s_cnt + p, 1) == CW - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            int first, cnt;
            mm_zone_ctas(P, bh, zone, &first, &cnt);
            float* part = partial + (((size_t)bh * 2 + zone) * P.pmax + (c - first)) * G * 130;
            const float* wm = s_wm + p * CW * MM_G;
            const float* wl = s_wl + p * CW * MM_G;
            const float* wo0 = s_wo + (size_t)p * CW * G * 128;
            for (int hh = 0; hh < G; ++hh) {
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < CW; ++w) M = fmaxf(M, wm[w * MM_G + hh]);
                float ew[CW];
                float lsum = 0.f;
#pragma unroll
                for (int w = 0; w < CW; ++w) {
                    const float mw = wm[w * MM_G + hh];
                    ew[w] = mw == -INFINITY ? 0.f : __expf(mw - M);
                    lsum += wl[w * MM_G + hh] * ew[w];
                }
#pragma unroll
                for (int d = lane; d < 128; d += 32) {
                    float acc = 0.f;
#pragma unroll
                    for (int w = 0; w < CW; ++w)
                        if (ew[w] != 0.f) acc += wo0[((size_t)w * G + hh) * 128 + d] * ew[w];
                    part[hh * 130 + 2 + d] = acc;
                }
                if (lane == 0) { part[hh * 130] = M; part[hh * 130 + 1] = lsum; }
            }
            __syncwarp();
            if (lane == 0) {
                s_cnt[p] = 0;
                __threadfence_block();
                atomicAdd(s_cnt + 2 + p, 1);
            }
        }
        ++seg;
    };

    // online-softmax update for one column from this lane's NV logits
    auto softmax_update = [&](int col, const float* lgv, float* pv, int nv) {
        float mx = -INFINITY;
        for (int x = 0; x < nv; ++x) mx = fmaxf(mx, lgv[x]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[col], mx);
        if (mn == -INFINITY) {
            for (int x = 0; x < nv; ++x) pv[x] = 0.f;
            return;
        }
        if (mn > m[col]) {
            const float scl = __expf(m[col] - mn);
            ls[col] *= scl;
            spp[col] *= scl;
            svz[col] *= scl;
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
                o[dt][col] *= scl;
                o[dt][2 + col] *= scl;
            }
            m[col] = mn;
        }
        float sum = 0.f;
        for (int x = 0; x < nv; ++x) {
            pv[x] = __expf(lgv[x] - mn);
            sum += pv[x];
        }
        ls[col] += sum;
    };

    // Segment by segment (the items of one (sequence, head, zone) in this
    // CTA's range): the warp group of this warp takes items i0 + grp,
    // i0 + grp + NG, ...; item i is in stage slot (i - i0) mod NS.  Every
    // warp closes every segment (flush), so the segment merge sees all warps.
    constexpr int NG = CW / MM_SPLIT;
    const int grp = warp / MM_SPLIT, part = warp % MM_SPLIT;
#pragma unroll 1
    for (long long sa = i0; sa < i1;) {
        const long long bh = sa / P.ipb;
        const int zone = (int)(sa - bh * P.ipb) >= P.n_main ? 1 : 0;
        const long long sb = min(i1, bh * P.ipb + (zone ? P.ipb : P.n_main));
        if (bh != cur_bh) { load_q(bh); cur_bh = bh; }
        reset_acc();
        const long long rel = sa - i0;
        const long long first = sa + (((long long)grp - rel) % NG + NG) % NG;
#pragma unroll 1
        for (long long i = first; i < sb; i += NG) {
        const int j = (int)(i - bh * P.ipb);
        const int kk_item = (int)(i - i0);
        const int s = kk_item % NS;
        // A warp that gives up waiting keeps walking the items (and joins every
        // named barrier) without computing, so no barrier is left unmatched.
        if (ok && !mbar_wait_bounded(&full[s], (kk_item / NS) & 1)) {
            set_err(L.err, QV_DERR_LAYOUT);
            ok = false;
        }
        if (!ok || skipped(i)) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            continue;
        }
        const uint32_t st = smem_u32(stages + s * MM_STAGE);
        const unsigned char* stp = stages + s * MM_STAGE;
        if (zone == 0) {
            // ---------------- main zone: 32 tokens = 2 m-tiles, MMT per warp ----
            // two accumulators per m-tile (d < 64 and d >= 64) halve the chain
            // of dependent MMAs
            constexpr int MMT = 2 / MM_SPLIT;
            const int mt0 = part * MMT;
            float sc[MMT][4], sc2[MMT][4];
#pragma unroll
            for (int i = 0; i < MMT; ++i)
#pragma unroll
                for (int r = 0; r < 4; ++r) sc[i][r] = sc2[i][r] = 0.f;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int d = 16 * kk + 8 * (mi >> 1);
#pragma unroll
                for (int i = 0; i < MMT; ++i) {
                    const int row = 16 * (mt0 + i) + (lane & 7) + 8 * (mi & 1);
                    uint32_t a[4], a2[4];
                    ldsm_x4(st + swz(row, d >> 3), a[0], a[1], a[2], a[3]);
                    ldsm_x4(st + 4096 + swz(row, d >> 3), a2[0], a2[1], a2[2], a2[3]);
                    mma_kv<DT>(sc[i], a, bq[kk]);
                    mma_kv<DT>(sc2[i], a2, bq[kk + 4]);
                }
            }
#pragma unroll
            for (int i = 0; i < MMT; ++i)
#pragma unroll
                for (int r = 0; r < 4; ++r) sc[i][r] += sc2[i][r];
            float lg[2][2 * MMT];   // per column: [i*2 + rowhalf]
            const int pos0 = MM_MT * j;
            // token t of this item is live iff off0 + t < lim: only the current
            // ring window has an unwritten tail
            int off0 = 0, lim = 64;
            if (pos0 >= g.ring_base()) {
                off0 = (pos0 - g.ring_base()) & 63;
                if (!mm_item_live(g, pos0 + 63 - off0, cw, 0)) lim = tv;
            }
#pragma unroll
            for (int i = 0; i < MMT; ++i) {
                const int tA = 16 * (mt0 + i) + gq, tB = tA + 8;
                const bool la = off0 + tA < lim, lb = off0 + tB < lim;
                const float v0 = la ? logit_round<DT>(sc[i][0]) : -INFINITY;
                const float v1 = la ? logit_round<DT>(sc[i][1]) : -INFINITY;
                const float v2 = lb ? logit_round<DT>(sc[i][2]) : -INFINITY;
                const float v3 = lb ? logit_round<DT>(sc[i][3]) : -INFINITY;
                lg[0][2 * i] = v0; lg[1][2 * i] = v1; lg[0][2 * i + 1] = v2; lg[1][2 * i + 1] = v3;
                const int h0 = 2 * t4;
                const size_t ia = ((size_t)bh * S_tot + pos0 + tA) * G + h0, ib = ((size_t)bh * S_tot + pos0 + tB) * G + h0;
                if (h0 + 1 < G) {
                    if (la) *reinterpret_cast<uint32_t*>(lgp + ia) = pack2<DT>(v0, v1);
                    if (lb) *reinterpret_cast<uint32_t*>(lgp + ib) = pack2<DT>(v2, v3);
                } else if (h0 < G) {
                    if (la) lgp[ia] = Elt<DT>::t(v0);
                    if (lb) lgp[ib] = Elt<DT>::t(v2);
                }
            }
            float p[2][2 * MMT];
            softmax_update(0, lg[0], p[0], 2 * MMT);
            softmax_update(1, lg[1], p[1], 2 * MMT);
            // P^T fragments per 16-token k-step (hi + lo halves for BF16)
#pragma unroll
            for (int i = 0; i < MMT; ++i) {
                uint32_t bp[2], bl[2];
                bp[0] = movm_t(pack2<DT>(p[0][2 * i], p[1][2 * i]));
                bp[1] = movm_t(pack2<DT>(p[0][2 * i + 1], p[1][2 * i + 1]));
                if (DT == QV_BF16) {
                    const float r0 = p[0][2 * i] - rnd<QV_BF16>(p[0][2 * i]);
                    const float r1 = p[1][2 * i] - rnd<QV_BF16>(p[1][2 * i]);
                    const float r2 = p[0][2 * i + 1] - rnd<QV_BF16>(p[0][2 * i + 1]);
                    const float r3 = p[1][2 * i + 1] - rnd<QV_BF16>(p[1][2 * i + 1]);
                    bl[0] = movm_t(pack2<DT>(r0, r1));
                    bl[1] = movm_t(pack2<DT>(r2, r3));
                }
#pragma unroll
                for (int dt = 0; dt < 8; ++dt) {
                    const int row = 16 * (mt0 + i) + (lane & 7) + 8 * (mi >> 1);
                    const int d = 16 * dt + 8 * (mi & 1);
                    uint32_t a[4];
                    ldsm_x4_t(st + 8192 + (d >= 64 ? 4096 : 0) + swz(row, (d & 63) >> 3), a[0], a[1], a[2], a[3]);
                    mma_kv<DT>(o[dt], a, bp);
                    if (DT == QV_BF16) mma_kv<DT>(o[dt], a, bl);
                }
            }
        } else {
            // ---------------- Q-cache window: 64 tokens = 4 m-tiles ------------
            const T* ks = reinterpret_cast<const T*>(stp + 16384);
            const T* kz = reinterpret_cast<const T*>(stp + 16384 + 256);
            const T* vs = reinterpret_cast<const T*>(stp + 16384 + 512);
            const T* vz = reinterpret_cast<const T*>(stp + 16384 + 640);
            uint32_t bk[8][2];
            float zsum = 0.f, ssum = 0.f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                // lane (gq, t4): d = 16kk + 4t4 + 0..3; scales and zero points in
                // one 8-byte load each
                const int d0 = 16 * kk + 4 * t4;
                const uint2 ksv = *reinterpret_cast<const uint2*>(ks + d0);
                const uint2 kzv = *reinterpret_cast<const uint2*>(kz + d0);
                const float q0 = bits_to_f<DT>(qq[kk][0] & 0xffffu), q1 = bits_to_f<DT>(qq[kk][0] >> 16);
                const float q2 = bits_to_f<DT>(qq[kk][1] & 0xffffu), q3 = bits_to_f<DT>(qq[kk][1] >> 16);
                // q * K scale rounded once to f16 (two values per conversion)
                const __half2 h01 = __floats2half2_rn(q0 * bits_to_f<DT>(ksv.x & 0xffffu), q1 * bits_to_f<DT>(ksv.x >> 16));
                const __half2 h23 = __floats2half2_rn(q2 * bits_to_f<DT>(ksv.y & 0xffffu), q3 * bits_to_f<DT>(ksv.y >> 16));
                bk[kk][0] = *reinterpret_cast<const uint32_t*>(&h01);
                bk[kk][1] = *reinterpret_cast<const uint32_t*>(&h23);
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                zsum = fmaf(q0, bits_to_f<DT>(kzv.x & 0xffffu), zsum);
                zsum = fmaf(q1, bits_to_f<DT>(kzv.x >> 16), zsum);
                zsum = fmaf(q2, bits_to_f<DT>(kzv.y & 0xffffu), zsum);
                zsum = fmaf(q3, bits_to_f<DT>(kzv.y >> 16), zsum);
                ssum += f01.x;
                ssum += f01.y;
                ssum += f23.x;
                ssum += f23.y;
            }
            zsum += __shfl_xor_sync(0xffffffffu, zsum, 1);
            zsum += __shfl_xor_sync(0xffffffffu, zsum, 2);
            ssum += __shfl_xor_sync(0xffffffffu, ssum, 1);
            ssum += __shfl_xor_sync(0xffffffffu, ssum, 2);
            const float cr = zsum - 1024.f * ssum;
            const float corr0 = __shfl_sync(0xffffffffu, cr, 8 * t4);
            const float corr1 = __shfl_sync(0xffffffffu, cr, 8 * t4 + 4);
            constexpr int QMT = 4 / MM_SPLIT;   // m-tiles of this warp
            const int qt0 = part * QMT;
            float sc[QMT][4];
#pragma unroll
            for (int i = 0; i < QMT; ++i)
#pragma unroll
                for (int r = 0; r < 4; ++r) sc[i][r] = 0.f;
#pragma unroll
            for (int kk2 = 0; kk2 < 4; ++kk2) {
                const int chunk = 2 * kk2 + (mi >> 1);
#pragma unroll
                for (int i = 0; i < QMT; ++i) {
                    const int row = 16 * (qt0 + i) + (lane & 7) + 8 * (mi & 1);
                    uint32_t r[4];
                    ldsm_x4(st + swz(row, chunk), r[0], r[1], r[2], r[3]);
                    const uint32_t a0[4] = {__byte_perm(r[0], 0x64646464u, 0x5140), __byte_perm(r[1], 0x64646464u, 0x5140),
                                            __byte_perm(r[0], 0x64646464u, 0x5342), __byte_perm(r[1], 0x64646464u, 0x5342)};
                    const uint32_t a1[4] = {__byte_perm(r[2], 0x64646464u, 0x5140), __byte_perm(r[3], 0x64646464u, 0x5140),
                                            __byte_perm(r[2], 0x64646464u, 0x5342), __byte_perm(r[3], 0x64646464u, 0x5342)};
                    mma_f16(sc[i], a0, bk[2 * kk2]);
                    mma_f16(sc[i], a1, bk[2 * kk2 + 1]);
                }
            }
            const int slot = j - P.n_main;
            float lg[2][2 * QMT];
#pragma unroll
            for (int i = 0; i < QMT; ++i) {
                const int tA = 16 * (qt0 + i) + gq;
                const float v0 = logit_round<DT>(sc[i][0] + corr0);
                const float v1 = logit_round<DT>(sc[i][1] + corr1);
                const float v2 = logit_round<DT>(sc[i][2] + corr0);
                const float v3 = logit_round<DT>(sc[i][3] + corr1);
                lg[0][2 * i] = v0; lg[1][2 * i] = v1; lg[0][2 * i + 1] = v2; lg[1][2 * i + 1] = v3;
                const int h0 = 2 * t4;
                const size_t ia = ((size_t)bh * S_tot + g.S_cap + (size_t)slot * 64 + tA) * G + h0;
                const size_t ib = ia + 8 * (size_t)G;
                if (h0 + 1 < G) {
                    *reinterpret_cast<uint32_t*>(lgp + ia) = pack2<DT>(v0, v1);
                    *reinterpret_cast<uint32_t*>(lgp + ib) = pack2<DT>(v2, v3);
                } else if (h0 < G) {
                    lgp[ia] = Elt<DT>::t(v0);
                    lgp[ib] = Elt<DT>::t(v2);
                }
            }
            float p[2][2 * QMT];
            softmax_update(0, lg[0], p[0], 2 * QMT);
            softmax_update(1, lg[1], p[1], 2 * QMT);
            uint32_t bp[QMT][2];
#pragma unroll
            for (int i = 0; i < QMT; ++i) {
                const int tA = 16 * (qt0 + i) + gq, tB = tA + 8;
                const float vsA = Elt<DT>::f(vs[tA]) * 1024.f, vsB = Elt<DT>::f(vs[tB]) * 1024.f;
                const float vzA = Elt<DT>::f(vz[tA]), vzB = Elt<DT>::f(vz[tB]);
                // P'' = p * v_scale * 1024 in f16; corrections use the rounded values
                const float pa0 = f16r(p[0][2 * i] * vsA), pa1 = f16r(p[1][2 * i] * vsA);
                const float pb0 = f16r(p[0][2 * i + 1] * vsB), pb1 = f16r(p[1][2 * i + 1] * vsB);
                spp[0] += pa0 + pb0;
                spp[1] += pa1 + pb1;
                svz[0] += p[0][2 * i] * vzA + p[0][2 * i + 1] * vzB;
                svz[1] += p[1][2 * i] * vzA + p[1][2 * i + 1] * vzB;
                bp[i][0] = movm_t(pack2<QV_F16>(pa0, pa1));
                bp[i][1] = movm_t(pack2<QV_F16>(pb0, pb1));
            }
#pragma unroll
            for (int dt2 = 0; dt2 < 4; ++dt2) {
                const int chunk = 2 * dt2 + (mi >> 1);
#pragma unroll
                for (int i = 0; i < QMT; ++i) {
                    const int row = 16 * (qt0 + i) + (lane & 7) + 8 * (mi & 1);
                    uint32_t r[4];
                    ldsm_x4_t(st + 8192 + swz(row, chunk), r[0], r[1], r[2], r[3]);
                    const uint32_t a0[4] = {__byte_perm(r[0], 0x64646464u, 0x5240), __byte_perm(r[0], 0x64646464u, 0x5341),
                                            __byte_perm(r[1], 0x64646464u, 0x5240), __byte_perm(r[1], 0x64646464u, 0x5341)};
                    const uint32_t a1[4] = {__byte_perm(r[2], 0x64646464u, 0x5240), __byte_perm(r[2], 0x64646464u, 0x5341),
                                            __byte_perm(r[3], 0x64646464u, 0x5240), __byte_perm(r[3], 0x64646464u, 0x5341)};
                    mma_f16(o[2 * dt2], a0, bp[i]);
                    mma_f16(o[2 * dt2 + 1], a1, bp[i]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        }
        flush((int)(bh * 2 + zone), sb == i1);
        sa = sb;
    }
    // let the combine grid get scheduled while this grid drains (it waits for
    // this grid's completion before reading anything).  Triggering at the
    // start instead, with fewer stages at batch 1 so that a combine block fits
    // beside each CTA, was measured: 0.08 ms slower per 32-layer decode step.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // every CTA has read the token counter at its start; the last one to finish
    // advances it (the combine kernel reads the advanced value)
    __threadfence();
    consumer_sync<CW>();
    if (threadIdx.x == 0) {
        if (atomicAdd(tickets, 1) == (int)gridDim.x - 1) {
            tickets[0] = 0;
            L.step[0] = N0 + 1;
        }
    }
}

// Combine kernel: a grid of many small blocks, chained to the attention
// kernel with programmatic dependent launch.  grid = (chunks, B*H).
template <int DT, bool OUT, bool FOLD>
__global__ void __launch_bounds__(256) decode_combine_kernel(Geo g, qv_layer L, void* __restrict__ out,
                                                             const float* __restrict__ partial,
                                                             const void* __restrict__ logits, MmPlan P,
                                                             int blocks_per_chunk) {
    __shared__ float sm[MM_CMB_SMEM];
    // wait for the streaming kernel (programmatic dependent launch; a no-op
    // when launched after an event on another stream)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // a programmatic dependent (the output projection) may start streaming
    // its weights; it waits for this grid before reading the output
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int N0 = L.step[0] - 1;
    combine_unit<DT, OUT, FOLD>(g, L, out, partial, logits, P, N0, blockIdx.y, blockIdx.x, gridDim.x,
                                blocks_per_chunk, sm, threadIdx.x, blockDim.x, BlockSync{});
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

static bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
    }
    return n;
}

bool mm_supported(const Geo& g) {
    return !(g.flags & QV_FLAG_REFERENCE_ROUNDING) && (g.dt == QV_BF16 || g.dt == QV_F16) && g.D == 128 &&
           g.om == 64 && g.sink % 64 == 0 && g.bits == 8 && g.G <= MM_G && g.S_cap % 64 == 0;
}

static size_t mm_fixed_smem(const Geo& g, int cw) {
    return 1024 + (size_t)(2 * cw * g.G * 128 + 4 * cw * MM_G) * 4 + 16 + 2 * MM_MAXNS * 8 + MM_SKIPMAP;
}

MmPlan mm_plan(const Geo& g) {
    MmPlan P;
    P.n_main = g.S_cap / MM_MT;
    P.n_q = g.qw;
    P.ipb = P.n_main + P.n_q;
    P.total = (long long)P.ipb * g.B * g.H;
    long long nc = sm_count();
    if (nc > P.total) nc = P.total;
    P.nC = (int)(nc < 1 ? 1 : nc);
    const long long wz = P.n_main > P.n_q ? P.n_main : P.n_q;
    P.pmax = (int)((wz * P.nC + P.total - 1) / P.total + 2);
    // items of the fullest CTA: with many per CTA more consumer warps hide latency
    const long long per_cta = (P.total + P.nC - 1) / P.nC;
    P.cw = per_cta >= 2 * MM_CW_WIDE ? MM_CW_WIDE : MM_CW_NARROW;
    const int ns = (int)((232448 - mm_fixed_smem(g, P.cw)) / MM_STAGE);
    P.ns = ns > MM_MAXNS ? MM_MAXNS : ns;
    return P;
}

size_t mm_ws_bytes(const Geo& g, size_t* off_part, size_t* off_logits) {
    MmPlan P = mm_plan(g);
    const size_t BH = (size_t)g.B * g.H;
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t o = al((BH + 1) * sizeof(int));
    *off_part = o;
    o += al(BH * 2 * P.pmax * g.G * 130 * sizeof(float));
    *off_logits = o;
    o += al(BH * (size_t)(g.S_cap + g.qw * g.om) * g.G * elt_size(g.dt));
    return o;
}

// mode: 0 = attention, output and ledger fold; 1 = attention and output (the
// fold left pending); 2 = the pending fold of the attention launched last with
// this workspace
int mm_launch(const Geo& g, const qv_layer& L, const void* q, void* out, void* ws, cudaStream_t s, int mode) {
    MmPlan P = mm_plan(g);
    // a warp group may wait on a stage only one fill ahead of it: stages >= groups
    if (P.pmax > MM_CMB_MAXP || P.ns < P.cw / MM_SPLIT) return QV_EINVAL;
    size_t op, ol;
    mm_ws_bytes(g, &op, &ol);
    char* base = reinterpret_cast<char*>(ws);
    CUtensorMap mk, mv, mkq, mvq;
    const CUtensorMapDataType kt = g.dt == QV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t rows = (uint64_t)g.B * g.H * g.S_cap;
    const uint64_t qrows = (uint64_t)g.B * g.H * (g.qw > 0 ? g.qw : 1) * 64;
    if (mode != 2) {
        bool okm = make_map(&mk, L.k, kt, 128, rows, 256, 64, MM_MT) && make_map(&mv, L.v, kt, 128, rows, 256, 64, MM_MT);
        const void* kqb = g.qw > 0 ? (const void*)L.kq : (const void*)L.k;
        const void* vqb = g.qw > 0 ? (const void*)L.vq : (const void*)L.v;
        okm = okm && make_map(&mkq, kqb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, qrows, 128, 128, 64) &&
              make_map(&mvq, vqb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, qrows, 128, 128, 64);
        if (!okm) return QV_EINVAL;
    }
    const size_t smem = mm_fixed_smem(g, P.cw) + (size_t)P.ns * MM_STAGE;
    static int cached[2][2] = {{48 * 1024, 48 * 1024}, {48 * 1024, 48 * 1024}};
    int* tickets = reinterpret_cast<int*>(base);
    float* part = reinterpret_cast<float*>(base + op);
    void* lgt = base + ol;
    const int BH = g.B * g.H;
    const int n_blk = g.S_cap / 64 + g.qw;
    int chunks = (2 * sm_count() + BH - 1) / BH;
    if (chunks > n_blk) chunks = n_blk;
    if (chunks < (n_blk + MM_CMB_MAXBLK - 1) / MM_CMB_MAXBLK) chunks = (n_blk + MM_CMB_MAXBLK - 1) / MM_CMB_MAXBLK;
    if (chunks < 1) chunks = 1;
    const int bpc = (n_blk + chunks - 1) / chunks;
    chunks = (n_blk + bpc - 1) / bpc;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg1 = {};
    cfg1.gridDim = dim3(P.nC);
    cfg1.blockDim = dim3((P.cw + 1) * 32);
    cfg1.dynamicSmemBytes = smem;
    cfg1.stream = s;
    cfg1.attrs = attr;
    cfg1.numAttrs = 1;
    cudaLaunchConfig_t cfg2 = cfg1;
    cfg2.gridDim = dim3(chunks, BH);
    cfg2.blockDim = dim3(256);
    cfg2.dynamicSmemBytes = 0;
    const bool wide = P.cw == MM_CW_WIDE;
    auto kern = g.dt == QV_BF16 ? (wide ? decode_mma_kernel<QV_BF16, MM_CW_WIDE> : decode_mma_kernel<QV_BF16, MM_CW_NARROW>)
                                : (wide ? decode_mma_kernel<QV_F16, MM_CW_WIDE> : decode_mma_kernel<QV_F16, MM_CW_NARROW>);
    const bool bf = g.dt == QV_BF16;
    auto comb = mode == 0 ? (bf ? decode_combine_kernel<QV_BF16, true, true> : decode_combine_kernel<QV_F16, true, true>)
              : mode == 1 ? (bf ? decode_combine_kernel<QV_BF16, true, false> : decode_combine_kernel<QV_F16, true, false>)
                          : (bf ? decode_combine_kernel<QV_BF16, false, true> : decode_combine_kernel<QV_F16, false, true>);
    cudaError_t e = cudaSuccess;
    if (mode != 2) {
        e = ensure_smem(kern, smem, &cached[bf ? 0 : 1][wide ? 1 : 0]);
        if (e != cudaSuccess) return set_cuda_error(e);
        e = cudaLaunchKernelEx(&cfg1, kern, mk, mv, mkq, mvq, g, L, q, tickets, part, lgt, P);
        if (e != cudaSuccess) return set_cuda_error(e);
    }
    e = cudaLaunchKernelEx(&cfg2, comb, g, L, out, (const float*)part, (const void*)lgt, P, bpc);
    if (e != cudaSuccess) return set_cuda_error(e);
    return check_launch();
}

}  // namespace qv
