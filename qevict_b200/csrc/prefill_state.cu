// Prefill: build one layer's Sticky-KV state from the prompt.
//
// Follows the prefill branch of STICKYKVCache_LayerWise.__call__
// (src/models/kv_cache/cache.py:269-355):
//   tally_prefill_scores      eviction_manager.py:115-173  window sums of the
//                             per-key column scores, local-history seeding
//   evict_from_window_scores  eviction.py:102-156  top-k winners (kept in id
//                             order) and top-q losers (top-k order)
//   store_windows             quantize_manager.py:91-98  losers -> Q-cache
//   create_mask_and_evict_from_kv_cache_prompt_stage  eviction.py:163-240
//                             sinks + winners + local zone
// The compacted cache is written straight into the slot layout: winner i (in
// id order) to sticky slot i, local window w to ring slot w % ring_windows,
// loser j to Q slot j.
#include <math.h>

#include "codec.cuh"

namespace qv {

constexpr int PF_THREADS = 256;

template <int SD>
__device__ __forceinline__ float window_score(const void* colsum, size_t base, int om, int lane) {
    float a = 0.f;
    bool first = true;
    for (int i = lane; i < om; i += 32) {
        const float v = ld<SD>(colsum, base + i);
        a = first ? v : a + v;
        first = false;
    }
    a = warp_sum(a);
    return rnd<SD>(a);  // the reference sums in the scores' dtype (identity for fp32)
}

// One CTA per (sequence, KV head).  smem: scores[nw], rank[nw].
template <int SD>
__global__ void __launch_bounds__(PF_THREADS) prefill_select_kernel(Geo g, qv_layer L, const void* colsum,
                                                                   int S) {
    extern __shared__ __align__(16) unsigned char smem[];
    const size_t bh = blockIdx.x;
    const int b = (int)(bh / g.H);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = PF_THREADS / 32;
    const int nw = (S - g.local - g.sink) / g.om;   // scored windows
    const int tpw = (S - g.sink) / g.om;            // all prompt windows
    float* sc = reinterpret_cast<float*>(smem);
    int* rk = reinterpret_cast<int*>(sc + nw);
    float* lhist = L.local_hist + bh * g.maxW;

    for (int w = threadIdx.x; w < g.maxW; w += PF_THREADS) {
        lhist[w] = 0.f;
        L.arch_valid[bh * g.maxW + w] = 0;
    }
    for (int p = threadIdx.x; p < g.S_cap; p += PF_THREADS) L.votes[bh * g.S_cap + p] = 0.f;
    __syncthreads();
    // window scores / local history from the column sums
    for (int w = warp; w < tpw; w += nwarp) {
        const float v = window_score<SD>(colsum, bh * (size_t)S + g.sink + (size_t)w * g.om, g.om, lane);
        if (lane == 0) {
            if (w < g.maxW) lhist[w] = v;
            else set_err(L.err, QV_DERR_TABLE);
            if (w < nw) sc[w] = v;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nw; i += PF_THREADS) {
        const float si = sc[i];
        int r = 0;
        for (int j = 0; j < nw; ++j) {
            const float sj = sc[j];
            r += (sj > si) || (sj == si && j < i);
        }
        rk[i] = r;
    }
    __syncthreads();
    const int curr_k = min(g.kw, nw);
    const int q_cnt = (g.qw > 0 && nw - curr_k > 0) ? min(g.qw, nw - curr_k) : 0;
    int32_t* swid = L.sticky_wid + bh * g.kw;
    float* sscore = L.sticky_score + bh * g.kw;
    int32_t* sorder = L.sticky_order + bh * g.kw;
    int32_t* qwid = L.q_wid + bh * g.qw;
    float* qscore = L.q_score + bh * g.qw;
    int32_t* qorder = L.q_order + bh * g.qw;
    for (int s = threadIdx.x; s < g.kw; s += PF_THREADS) { swid[s] = -1; sscore[s] = 0.f; sorder[s] = s; }
    for (int s = threadIdx.x; s < g.qw; s += PF_THREADS) { qwid[s] = -1; qscore[s] = 0.f; qorder[s] = s; }
    __syncthreads();
    // winners in id order: ids are candidate indices, so position = #winners with smaller index
    for (int i = threadIdx.x; i < nw; i += PF_THREADS) {
        if (rk[i] < curr_k) {
            int pos = 0;
            for (int j = 0; j < i; ++j) pos += rk[j] < curr_k;
            swid[pos] = i;
            sscore[pos] = sc[i];
        } else if (rk[i] - curr_k < q_cnt) {
            const int j = rk[i] - curr_k;
            qwid[j] = i;
            qscore[j] = sc[i];
        }
    }
    if (threadIdx.x == 0 && bh % g.H == 0) {
        L.seq[b * 4 + 0] = curr_k;
        L.seq[b * 4 + 1] = q_cnt;
        L.seq[b * 4 + 2] = 0;
        L.seq[b * 4 + 3] = 0;
        if (b == 0) { L.step[0] = S; L.step[1] = S; }
    }
}

// Copy / quantise one window per CTA.  Tasks: 0 sinks, [1, 1+kw) sticky slots,
// [1+kw, kw+R) local windows, [kw+R, kw+R+qw) Q slots.
template <int DT>
__global__ void __launch_bounds__(128) prefill_fill_kernel(Geo g, qv_layer L, const void* kp, const void* vp, int S) {
    __shared__ float sm[256];
    const size_t bh = blockIdx.x;
    const int task = blockIdx.y;
    const int om = g.om, D = g.D;
    const int nw = (S - g.local - g.sink) / om;
    const size_t src0 = bh * (size_t)S * D;
    const size_t dst0 = bh * (size_t)g.S_cap * D;
    auto copy_rows = [&](int from, int to, int n) {
        for (int i = threadIdx.x; i < n * D; i += blockDim.x) {
            st<DT>(L.k, dst0 + (size_t)to * D + i, ld<DT>(kp, src0 + (size_t)from * D + i));
            st<DT>(L.v, dst0 + (size_t)to * D + i, ld<DT>(vp, src0 + (size_t)from * D + i));
        }
    };
    if (task == 0) {
        copy_rows(0, 0, g.sink);
    } else if (task < 1 + g.kw) {
        const int s = task - 1;
        const int wid = L.sticky_wid[bh * g.kw + s];
        if (wid >= 0) copy_rows(g.sink + wid * om, g.sink + s * om, om);
    } else if (task < g.kw + g.R) {
        const int w = nw + (task - 1 - g.kw);
        copy_rows(g.sink + w * om, g.ring_base() + (w % g.R) * om, om);
    } else {
        const int j = task - g.kw - g.R;
        const int wid = L.q_wid[bh * g.qw + j];
        if (wid < 0) return;
        const int qb = g.bits == 4 ? D / 2 : D;
        const size_t sw = bh * g.qw + j;
        const size_t xb = src0 + (size_t)(g.sink + wid * om) * D;
        quantize_k_window<DT>(kp, xb, om, D, g.bits, false, L.kq, sw * om * qb, L.ks, L.kz, sw * D,
                              false, nullptr, nullptr, 0, sm);
        quantize_v_window<DT>(vp, xb, om, D, g.bits, false, L.vq, sw * om * qb, L.vs, L.vz, sw * om,
                              false, nullptr, nullptr, 0, sm);
    }
}

}  // namespace qv

using namespace qv;

extern "C" int qv_prefill_build(const qv_dims* d, const qv_layer* L, const void* k_prompt, const void* v_prompt,
                                int32_t S, const void* colsum, int32_t score_dtype, qv_stream_t stream) {
    int rc = validate_dims(d);
    if (rc) return rc;
    if (!L || !k_prompt || !v_prompt || !colsum) return QV_EINVAL;
    if (score_dtype != QV_F32 && score_dtype != d->dtype) return QV_EINVAL;
    Geo g = make_geo(d);
    if (S < g.sink + g.local || (S - g.sink) % g.om) return QV_ENOTALIGNED;
    if ((S - g.sink) / g.om > g.maxW) return QV_EINVAL;
    const int nw = (S - g.local - g.sink) / g.om;
    const size_t smem = (size_t)nw * 8 + 16;
    if (smem > 220 * 1024) return QV_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    const int BH = g.B * g.H;
#define QV_PF_SEL(SD)                                                                                  \
    do {                                                                                               \
        static int cached = 48 * 1024;                                                                 \
        cudaError_t e = ensure_smem(prefill_select_kernel<SD>, smem, &cached);                         \
        if (e != cudaSuccess) return set_cuda_error(e);                                                \
        prefill_select_kernel<SD><<<BH, PF_THREADS, smem, s>>>(g, *L, colsum, S);                      \
    } while (0)
    switch (score_dtype) {
        case QV_F32: QV_PF_SEL(QV_F32); break;
        case QV_BF16: QV_PF_SEL(QV_BF16); break;
        default: QV_PF_SEL(QV_F16); break;
    }
#undef QV_PF_SEL
    dim3 grid(BH, g.kw + g.R + g.qw);
    switch (g.dt) {
        case QV_F32: prefill_fill_kernel<QV_F32><<<grid, 128, 0, s>>>(g, *L, k_prompt, v_prompt, S); break;
        case QV_BF16: prefill_fill_kernel<QV_BF16><<<grid, 128, 0, s>>>(g, *L, k_prompt, v_prompt, S); break;
        default: prefill_fill_kernel<QV_F16><<<grid, 128, 0, s>>>(g, *L, k_prompt, v_prompt, S); break;
    }
    return check_launch();
}
