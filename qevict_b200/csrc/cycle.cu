// Eviction cycle (every omega decode tokens), device-side, no host sync.
//
// Semantics follow EvictionManager.run_decode_cycle / update_local_history /
// commit_decode_result / reset_decode_counters
// (src/models/kv_cache/eviction_manager.py:205-417), QuantizationManager.
// get_promoted_windows / rebuild (src/models/kv_cache/quantize_manager.py:114-327)
// and STICKYKVCache_LayerWise._build_physical_cache (src/models/kv_cache/cache.py:433-575).
//
// Kernels (one stream, in order):
//   cycle_select   one CTA per sequence, one warp per KV head: scoreboard over
//                  slots, candidate list [old sticky (id order) | challenger |
//                  Q (top-k order)], rank-based top-k (ties -> lower candidate
//                  index), cross-head min for the loser count, local-history
//                  update, new slot tables and a move plan.
//   cycle_up_gather   promoted Q windows (dequantised) and the winning
//                  challenger (copied from its ring slot) -> staging; archives
//                  the promoted windows' scales for path C.
//   cycle_demote   new Q entries: quantise fresh (path B) or with the archived
//                  scale/zp (path C) from their sticky slot, or from zeros when
//                  the window is not in a sticky slot (the reference's
//                  zero-filled gather, quantize_manager.py:256-258).
//   cycle_up_scatter  staging -> freed sticky slots.
// Windows that keep their tier do not move.
#include <limits.h>
#include <math.h>

#include "codec.cuh"

namespace qv {

struct CycleWs {
    int* plan;      // [BH][plan_stride]
    void* staging;  // [BH][max_up][2][om][D]
    int max_up, max_down, plan_stride;
};

enum { UP_PROMOTE = 0, UP_RING = 1, UP_ZERO = 2 };

static inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

static void cycle_ws_layout(const Geo& g, CycleWs* w, size_t* off_stage, size_t* total) {
    w->max_up = max(1, min(g.kw, g.qw + 1));
    w->max_down = max(1, min(g.qw, g.kw + 1));
    w->plan_stride = 2 + 4 * w->max_up + 4 * w->max_down;
    const size_t BH = (size_t)g.B * g.H;
    size_t o = a256(BH * w->plan_stride * sizeof(int));
    *off_stage = o;
    o += a256(BH * (size_t)w->max_up * 2 * g.om * g.D * elt_size(g.dt));
    *total = o;
}

static size_t select_smem_per_warp(const Geo& g) {
    const int NC = g.kw + 1 + g.qw;
    return (size_t)NC * 14 * 4 + (size_t)(g.kw + g.R) * 4 + 64;
}

// nrem_out != nullptr: counting pass only -- write, per sequence, the minimum
// over this launch's KV heads of the loser count and change nothing else.
// nrem_in != nullptr: the minimum over KV heads held elsewhere (other ranks of
// a head-sharded layer), folded into this launch's own minimum.
__global__ void __launch_bounds__(1024) cycle_select_kernel(Geo g, qv_layer L, CycleWs ws, int per_warp_bytes,
                                                            int32_t* nrem_out, const int32_t* nrem_in) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_nrem;
    const int b = blockIdx.x;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t bh = (size_t)b * g.H + h;
    const int NC = g.kw + 1 + g.qw;
    int* base = reinterpret_cast<int*>(smem + (size_t)h * per_warp_bytes);
    int* c_id = base;               // candidate window id
    float* c_sc = reinterpret_cast<float*>(base + NC);  // candidate score
    int* c_rank = base + 2 * NC;    // top-k rank
    int* c_src = base + 3 * NC;     // old sticky slot / ring slot / Q slot
    int* c_pos = base + 4 * NC;     // winner position in id order, else -1
    int* p_cand = base + 5 * NC;    // id-order position -> candidate
    int* p_old = base + 6 * NC;     // old sticky slot holding the winner's id, else -1
    int* p_q = base + 7 * NC;       // Q slot holding the winner's id, else -1
    int* p_slot = base + 8 * NC;    // new sticky slot of the winner
    int* l_cand = base + 9 * NC;    // loser rank -> candidate
    int* l_ret = base + 10 * NC;    // retained old Q slot, else -1
    int* l_src = base + 11 * NC;    // old sticky slot holding the loser's id, else -1
    int* l_path = base + 12 * NC;   // 1 = path C (archived scale/zp)
    int* l_slot = base + 13 * NC;   // new Q slot
    float* sb_st = reinterpret_cast<float*>(base + 14 * NC);
    float* sb_ring = sb_st + g.kw;

    if (threadIdx.x == 0) s_nrem = INT_MAX;

    const int N = L.step[0];                 // tokens incl. the current one
    const int cw = (N - 1 - g.sink) / g.om;  // the window just completed
    const int L0 = cw - (g.R - 1);           // oldest ring window (the challenger)
    const int curr_prev = L.seq[b * 4 + 0];
    const int q_prev = L.seq[b * 4 + 1];

    int32_t* swid = L.sticky_wid + bh * g.kw;
    float* sscore = L.sticky_score + bh * g.kw;
    int32_t* sorder = L.sticky_order + bh * g.kw;
    int32_t* qwid = L.q_wid + bh * g.qw;
    float* qscore = L.q_score + bh * g.qw;
    int32_t* qorder = L.q_order + bh * g.qw;
    float* votes = L.votes + bh * g.S_cap;
    float* lhist = L.local_hist + bh * g.maxW;
    uint8_t* arch = L.arch_valid + bh * g.maxW;

    // 1. scoreboard over slots (eviction_manager.py:229-255): every window's votes
    //    summed in the fixed warp order, 8 windows' loads in flight at a time
    {
        const int nslot = g.kw + g.R;
        for (int s0 = 0; s0 < nslot; s0 += 8) {
            float a[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int s = s0 + u;
                a[u] = 0.f;
                if (s < nslot && (s >= g.kw || swid[s] >= 0)) {
                    const float* v = votes + g.sink + s * g.om;   // ring slots follow the sticky slots
                    bool first = true;
                    for (int i = lane; i < g.om; i += 32) {
                        a[u] = first ? v[i] : a[u] + v[i];
                        first = false;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float t = warp_sum(a[u]);
                const int s = s0 + u;
                if (lane == 0 && s < nslot) {
                    if (s < g.kw) sb_st[s] = t;
                    else sb_ring[s - g.kw] = t;
                }
            }
        }
    }
    __syncwarp();
    auto sbv = [&](int w) -> float {
        if (w >= L0 && w <= cw) return sb_ring[w % g.R];
        for (int s = 0; s < g.kw; ++s)
            if (swid[s] == w) return sb_st[s];
        return 0.f;
    };

    // 2. candidates [old sticky in id order | challenger | Q in top-k order] (eviction_manager.py:257-325)
    const int vo = min(g.kw, curr_prev);
    for (int i = lane; i < vo; i += 32) {
        const int slot = sorder[i];
        c_id[i] = swid[slot];
        c_sc[i] = sscore[slot] + sb_st[slot];
        c_src[i] = slot;
    }
    __syncwarp();
    const int lnum = N - g.sink - g.local;
    int last = lnum >= 0 ? lnum / g.om - 1 : -1 - ((-lnum + g.om - 1) / g.om);
    last = min(last, g.maxW - 1);
    const bool has = last >= 0;
    const int qbase = vo + (has ? 1 : 0);
    if (has && lane == 0) {
        bool already = false;
        for (int i = 0; i < vo; ++i) already |= (c_id[i] == last);
        const float gen = sbv(last);
        const float hist = lhist[last];
        if (!already && !nrem_out) lhist[last] = 0.f;
        c_id[vo] = last;
        c_sc[vo] = already ? -INFINITY : gen + hist;
        c_src[vo] = (last >= L0 && last <= cw) ? last % g.R : -1;
    }
    const int qn = (g.qw > 0 && q_prev > 0) ? q_prev : 0;
    for (int j = lane; j < qn; j += 32) {
        const int slot = qorder[j];
        c_id[qbase + j] = qwid[slot];
        c_sc[qbase + j] = qscore[slot];
        c_src[qbase + j] = slot;
    }
    const int nc = qbase + qn;
    __syncwarp();

    // 3. ranks: descending score, ties -> lower candidate index
    const int curr_k = min(g.kw, nc);
    for (int i = lane; i < nc; i += 32) {
        const float si = c_sc[i];
        int r = 0;
        for (int j = 0; j < nc; ++j) {
            const float sj = c_sc[j];
            r += (sj > si) || (sj == si && j < i);
        }
        c_rank[i] = r;
    }
    __syncwarp();
    // winners ordered by (id, rank): argsort of the surviving ids (eviction_manager.py:330-333)
    for (int i = lane; i < nc; i += 32) {
        int pos = -1;
        if (c_rank[i] < curr_k) {
            pos = 0;
            for (int j = 0; j < nc; ++j)
                if (c_rank[j] < curr_k)
                    pos += (c_id[j] < c_id[i]) || (c_id[j] == c_id[i] && c_rank[j] < c_rank[i]);
            p_cand[pos] = i;
        }
        c_pos[i] = pos;
    }
    int nrem = 0;
    for (int i = lane; i < nc; i += 32) nrem += (c_rank[i] >= curr_k && c_sc[i] > -INFINITY);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) nrem += __shfl_xor_sync(0xffffffffu, nrem, o);
    __syncthreads();
    if (lane == 0) atomicMin(&s_nrem, nrem);
    __syncthreads();
    if (nrem_out) {
        if (threadIdx.x == 0) nrem_out[b] = s_nrem;
        return;
    }
    if (nrem_in && threadIdx.x == 0) s_nrem = min(s_nrem, nrem_in[b]);
    __syncthreads();
    const int q_new = (g.qw > 0 && s_nrem > 0) ? min(g.qw, s_nrem) : 0;

    // 4. per-winner sources by id: old sticky slot, then Q slot (cache.py:458-559)
    for (int p = lane; p < curr_k; p += 32) {
        const int wid = c_id[p_cand[p]];
        int old = -1, qs = -1;
        for (int r = 0; r < vo; ++r)
            if (c_id[r] == wid) { old = c_src[r]; break; }
        for (int r = 0; r < qn; ++r)
            if (c_id[qbase + r] == wid) { qs = c_src[qbase + r]; break; }
        p_old[p] = old;
        p_q[p] = qs;
    }
    // archive every Q window whose id is among the winners (quantize_manager.py:120-143)
    for (int r = lane; r < qn; r += 32) {
        const int wid = c_id[qbase + r];
        bool win = false;
        for (int j = 0; j < nc; ++j) win |= (c_rank[j] < curr_k && c_id[j] == wid);
        if (win) {
            if (wid >= 0 && wid < g.maxW) arch[wid] = 1;
            else set_err(L.err, QV_DERR_TABLE);
        }
    }
    // losers in top-k order (eviction_manager.py:335-345)
    for (int i = lane; i < nc; i += 32) {
        const int r = c_rank[i] - curr_k;
        if (r >= 0 && r < q_new) l_cand[r] = i;
    }
    __syncwarp();
    // per-loser routing: path A (retained), else from an old sticky slot or zeros,
    // path C when the window's scale/zp are archived (quantize_manager.py:168-318)
    for (int j = lane; j < q_new; j += 32) {
        const int wid = c_id[l_cand[j]];
        int ret = -1, src = -1;
        for (int r = 0; r < qn; ++r)
            if (c_id[qbase + r] == wid) { ret = c_src[qbase + r]; break; }
        for (int r = 0; r < vo; ++r)
            if (c_id[r] == wid) { src = c_src[r]; break; }
        l_ret[j] = ret;
        l_src[j] = src;
        l_path[j] = (wid >= 0 && wid < g.maxW && arch[wid]) ? 1 : 0;
    }
    __syncwarp();

    int* plan = ws.plan + bh * ws.plan_stride;
    if (lane == 0) {
        unsigned int keep[16];
        for (int i = 0; i < 16; ++i) keep[i] = 0u;
        // winners that stay in their old slot
        for (int p = 0; p < curr_k; ++p) {
            const int old = p_old[p];
            if (old >= 0 && !(keep[old >> 5] & (1u << (old & 31)))) {
                keep[old >> 5] |= 1u << (old & 31);
                p_slot[p] = old;
            } else {
                p_slot[p] = -1;
            }
        }
        int n_up = 0, n_down = 0, nf = 0;
        for (int p = 0; p < curr_k; ++p) {
            if (p_slot[p] >= 0) continue;
            while (nf < g.kw && (keep[nf >> 5] & (1u << (nf & 31)))) ++nf;
            if (nf >= g.kw) { set_err(L.err, QV_DERR_CAPACITY); p_slot[p] = -1; continue; }
            keep[nf >> 5] |= 1u << (nf & 31);
            p_slot[p] = nf;
            const int wid = c_id[p_cand[p]];
            int kind = UP_ZERO, src = -1;
            if (p_q[p] >= 0) { kind = UP_PROMOTE; src = p_q[p]; }
            else if (wid >= L0 && wid <= cw) { kind = UP_RING; src = wid % g.R; }
            if (n_up < ws.max_up) {
                int* e = plan + 2 + 4 * n_up;
                e[0] = kind; e[1] = src; e[2] = nf; e[3] = wid;
                ++n_up;
            } else {
                set_err(L.err, QV_DERR_CAPACITY);
            }
        }
        unsigned int qkeep[16];
        for (int i = 0; i < 16; ++i) qkeep[i] = 0u;
        for (int j = 0; j < q_new; ++j) {
            const int r = l_ret[j];
            if (r >= 0 && !(qkeep[r >> 5] & (1u << (r & 31)))) {
                qkeep[r >> 5] |= 1u << (r & 31);
                l_slot[j] = r;
            } else {
                l_slot[j] = -1;
            }
        }
        int qf = 0;
        for (int j = 0; j < q_new; ++j) {
            if (l_slot[j] >= 0) continue;
            while (qf < g.qw && (qkeep[qf >> 5] & (1u << (qf & 31)))) ++qf;
            if (qf >= g.qw) { set_err(L.err, QV_DERR_CAPACITY); continue; }
            qkeep[qf >> 5] |= 1u << (qf & 31);
            l_slot[j] = qf;
            if (n_down < ws.max_down) {
                int* e = plan + 2 + 4 * ws.max_up + 4 * n_down;
                e[0] = l_src[j]; e[1] = qf; e[2] = l_path[j]; e[3] = c_id[l_cand[j]];
                ++n_down;
            } else {
                set_err(L.err, QV_DERR_CAPACITY);
            }
        }
        plan[0] = n_up;
        plan[1] = n_down;
    }
    __syncwarp();
    // local history (eviction_manager.py:347-356, 398-412), one window per lane
    {
        const int start = has ? last + 1 : max(0, lnum / g.om);
        for (int w = start + lane; w < start + (g.R - 1); w += 32)
            if (w >= 0 && w < g.maxW) lhist[w] += sbv(w);
    }
    __syncwarp();
    // 5. commit tables (eviction_manager.py:385-396)
    for (int s = lane; s < g.kw; s += 32) swid[s] = -1;
    for (int s = lane; s < g.qw; s += 32) qwid[s] = -1;
    __syncwarp();
    for (int p = lane; p < curr_k; p += 32) {
        const int s = p_slot[p];
        if (s < 0) continue;
        swid[s] = c_id[p_cand[p]];
        sscore[s] = c_sc[p_cand[p]];
        sorder[p] = s;
    }
    for (int j = lane; j < q_new; j += 32) {
        const int s = l_slot[j];
        if (s < 0) continue;
        qwid[s] = c_id[l_cand[j]];
        qscore[s] = c_sc[l_cand[j]];
        qorder[j] = s;
    }
    // 6. reset votes (eviction_manager.py:414-417)
    for (int p = lane; p < g.S_cap; p += 32) votes[p] = 0.f;
    __syncthreads();
    if (threadIdx.x == 0) {
        L.seq[b * 4 + 0] = curr_k;
        L.seq[b * 4 + 1] = q_new;
    }
}

// 16-byte vector copy of n bytes (n a multiple of 16, both pointers 16-byte aligned)
__device__ __forceinline__ void copy16(void* dst, const void* src, size_t n) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    const size_t n4 = n / 16;
#pragma unroll 4
    for (size_t i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = s4[i];
}

template <int DT>
__global__ void __launch_bounds__(128) cycle_up_gather_kernel(Geo g, qv_layer L, CycleWs ws) {
    const size_t bh = blockIdx.x;
    const int i = blockIdx.y;
    const int* plan = ws.plan + bh * ws.plan_stride;
    if (i >= plan[0]) return;
    const int* e = plan + 2 + 4 * i;
    const int kind = e[0], src = e[1], wid = e[3];
    const int om = g.om, D = g.D;
    const size_t es = elt_size_dev(DT);
    char* stage = reinterpret_cast<char*>(ws.staging);
    char* stK = stage + ((bh * ws.max_up + i) * 2 + 0) * (size_t)om * D * es;
    char* stV = stK + (size_t)om * D * es;
    const int qb = g.bits == 4 ? D / 2 : D;
    if (kind == UP_RING) {
        const size_t row = (bh * g.S_cap + g.ring_base() + (size_t)src * om) * D * es;
        copy16(stK, reinterpret_cast<const char*>(L.k) + row, (size_t)om * D * es);
        copy16(stV, reinterpret_cast<const char*>(L.v) + row, (size_t)om * D * es);
    } else if (kind == UP_PROMOTE) {
        const size_t sw = bh * g.qw + src;
#pragma unroll 4
        for (int idx = threadIdx.x; idx < om * D; idx += blockDim.x) {
            const int t = idx / D, d = idx % D;
            st<DT>(stK, idx, dequant1<DT>(code_at(L.kq + (sw * om + t) * qb, d, g.bits), ld<DT>(L.ks, sw * D + d), ld<DT>(L.kz, sw * D + d)));
            st<DT>(stV, idx, dequant1<DT>(code_at(L.vq + (sw * om + t) * qb, d, g.bits), ld<DT>(L.vs, sw * om + t), ld<DT>(L.vz, sw * om + t)));
        }
    } else {
        for (int idx = threadIdx.x; idx < om * D; idx += blockDim.x) {
            st<DT>(stK, idx, 0.f);
            st<DT>(stV, idx, 0.f);
        }
    }
    if (kind == UP_PROMOTE && wid >= 0 && wid < g.maxW) {
        const size_t sw = bh * g.qw + src;
        const size_t aw = bh * g.maxW + wid;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            st<DT>(L.arch_ks, aw * D + d, ld<DT>(L.ks, sw * D + d));
            st<DT>(L.arch_kz, aw * D + d, ld<DT>(L.kz, sw * D + d));
        }
        for (int t = threadIdx.x; t < om; t += blockDim.x) {
            st<DT>(L.arch_vs, aw * om + t, ld<DT>(L.vs, sw * om + t));
            st<DT>(L.arch_vz, aw * om + t, ld<DT>(L.vz, sw * om + t));
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(128) cycle_demote_kernel(Geo g, qv_layer L, CycleWs ws) {
    __shared__ float sm[256];
    const size_t bh = blockIdx.x;
    const int i = blockIdx.y;
    const int* plan = ws.plan + bh * ws.plan_stride;
    if (i >= plan[1]) return;
    const int* e = plan + 2 + 4 * ws.max_up + 4 * i;
    const int src = e[0], dst = e[1], path = e[2], wid = e[3];
    const int om = g.om, D = g.D;
    const int qb = g.bits == 4 ? D / 2 : D;
    const bool zero = src < 0;
    const size_t xbase = zero ? 0 : (bh * g.S_cap + g.sink + (size_t)src * om) * D;
    const size_t sw = bh * g.qw + dst;
    const bool meta = path == 1 && wid >= 0 && wid < g.maxW;
    const size_t aw = bh * g.maxW + (meta ? wid : 0);
    quantize_k_window<DT>(L.k, xbase, om, D, g.bits, zero, L.kq, sw * om * qb, L.ks, L.kz, sw * D,
                          meta, L.arch_ks, L.arch_kz, aw * D, sm);
    quantize_v_window<DT>(L.v, xbase, om, D, g.bits, zero, L.vq, sw * om * qb, L.vs, L.vz, sw * om,
                          meta, L.arch_vs, L.arch_vz, aw * om, sm);
}

template <int DT>
__global__ void __launch_bounds__(128) cycle_up_scatter_kernel(Geo g, qv_layer L, CycleWs ws) {
    const size_t bh = blockIdx.x;
    const int i = blockIdx.y;
    const int* plan = ws.plan + bh * ws.plan_stride;
    if (i >= plan[0]) return;
    const int* e = plan + 2 + 4 * i;
    const int dst = e[2];
    const int om = g.om, D = g.D;
    const size_t es = elt_size_dev(DT);
    const char* stage = reinterpret_cast<const char*>(ws.staging);
    const char* stK = stage + ((bh * ws.max_up + i) * 2 + 0) * (size_t)om * D * es;
    const char* stV = stK + (size_t)om * D * es;
    const size_t row0 = (bh * g.S_cap + g.sink + (size_t)dst * om) * D * es;
    copy16(reinterpret_cast<char*>(L.k) + row0, stK, (size_t)om * D * es);
    copy16(reinterpret_cast<char*>(L.v) + row0, stV, (size_t)om * D * es);
}

}  // namespace qv

using namespace qv;

extern "C" size_t qv_cycle_workspace_bytes(const qv_dims* d) {
    if (validate_dims(d)) return 0;
    Geo g = make_geo(d);
    CycleWs w;
    size_t os, tot;
    cycle_ws_layout(g, &w, &os, &tot);
    return tot;
}

template <int DT>
static void launch_cycle_moves(const Geo& g, const qv_layer& L, const CycleWs& w, cudaStream_t s) {
    dim3 gu(g.B * g.H, w.max_up), gd(g.B * g.H, w.max_down);
    cycle_up_gather_kernel<DT><<<gu, 128, 0, s>>>(g, L, w);
    cycle_demote_kernel<DT><<<gd, 128, 0, s>>>(g, L, w);
    cycle_up_scatter_kernel<DT><<<gu, 128, 0, s>>>(g, L, w);
}

static int cycle_launch(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                        int32_t* nrem_out, const int32_t* nrem_in, qv_stream_t stream) {
    int rc = validate_dims(d);
    if (rc) return rc;
    if (!L || !workspace || !L->step || !L->seq || !L->err) return QV_EINVAL;
    Geo g = make_geo(d);
    CycleWs w;
    size_t os, tot;
    cycle_ws_layout(g, &w, &os, &tot);
    if (workspace_bytes < tot) return QV_ESPACE;
    w.plan = reinterpret_cast<int*>(workspace);
    w.staging = reinterpret_cast<char*>(workspace) + os;
    const size_t per_warp = (select_smem_per_warp(g) + 15) & ~(size_t)15;
    const size_t smem = per_warp * g.H;
    if (smem > 220 * 1024) return QV_EINVAL;
    static int cached = 48 * 1024;
    cudaError_t e = ensure_smem(cycle_select_kernel, smem, &cached);
    if (e != cudaSuccess) return set_cuda_error(e);
    cudaStream_t s = (cudaStream_t)stream;
    cycle_select_kernel<<<g.B, 32 * g.H, smem, s>>>(g, *L, w, (int)per_warp, nrem_out, nrem_in);
    if (!nrem_out) {
        switch (g.dt) {
            case QV_F32: launch_cycle_moves<QV_F32>(g, *L, w, s); break;
            case QV_BF16: launch_cycle_moves<QV_BF16>(g, *L, w, s); break;
            default: launch_cycle_moves<QV_F16>(g, *L, w, s); break;
        }
    }
    return check_launch();
}

extern "C" int qv_evict_cycle(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                              qv_stream_t stream) {
    return cycle_launch(d, L, workspace, workspace_bytes, nullptr, nullptr, stream);
}

extern "C" int qv_evict_cycle_count(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                                    int32_t* loser_count, qv_stream_t stream) {
    if (!loser_count) return QV_EINVAL;
    return cycle_launch(d, L, workspace, workspace_bytes, loser_count, nullptr, stream);
}

extern "C" int qv_evict_cycle_ext(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                                  const int32_t* loser_count, qv_stream_t stream) {
    if (!loser_count) return QV_EINVAL;
    return cycle_launch(d, L, workspace, workspace_bytes, nullptr, loser_count, stream);
}
