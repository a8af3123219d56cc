// Decode step: RoPE + in-place append, and the fused split-K attention over the
// mixed BF16/FP16/FP32 main zone and the INT8/INT4 Q-cache with the ledger fold.
//
// Attention semantics follow src/models/attention/ops.py:23-212: logits are the
// q.k products rounded to the KV dtype and divided by sqrt(D) (rounded), the
// softmax is fp32 over [main | Q], probabilities are rounded to the KV dtype
// and averaged over the GQA group (rounded) before being added to the fp32
// vote ledger (eviction_manager.py:198-203) or summed per Q window
// (quantize_manager.py:101-111).
//
// Split-K: every CTA owns a token range of one (sequence, KV head) and writes a
// partial (max, sum, unnormalised output) per query head plus the rounded
// logits of its tokens.  The last CTA of a (sequence, head) -- elected with an
// atomic ticket after a __threadfence, no spinning -- merges the partials,
// writes the output and folds the exact probabilities into the ledger.  The
// last of all merges advances the token counter.
#include <math.h>
#include <stdlib.h>

#include "codec.cuh"

namespace qv {

constexpr int MAXG = 8;
constexpr int DEC_THREADS = 256;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int CH_MAIN = 256;   // main-zone tokens per split
constexpr int CH_Q = 512;      // Q-zone tokens per split

struct DecodeWs {
    int* tickets;    // [BH + 1]
    float* partial;  // [BH][nsplit][G][D + 2]
    void* logits;    // [BH][S_cap + qw*om][G]  (kv dtype)
    int n_main, n_q;
};

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static void decode_ws_layout(const Geo& g, size_t* off_partial, size_t* off_logits, size_t* total,
                             int* n_main, int* n_q) {
    const size_t BH = (size_t)g.B * g.H;
    *n_main = (g.S_cap + CH_MAIN - 1) / CH_MAIN;
    *n_q = (g.qw * g.om + CH_Q - 1) / CH_Q;
    const int ns = *n_main + *n_q;
    size_t o = align256((BH + 1) * sizeof(int));
    *off_partial = o;
    o += align256(BH * ns * g.G * (g.D + 2) * sizeof(float));
    *off_logits = o;
    o += align256(BH * (size_t)(g.S_cap + g.qw * g.om) * g.G * elt_size(g.dt));
    *total = o;
}

// Is main-zone position pos of (b, h) a live token?  Sinks always; sticky slots
// when occupied; ring slots except the not-yet-written tail of the current window.
__device__ __forceinline__ bool main_live(const Geo& g, const int32_t* swid, int pos, int cw, int tv) {
    if (pos < g.sink) return true;
    const int r = pos - g.sink;
    const int slot = r / g.om;
    if (slot < g.kw) return swid[slot] >= 0;
    const int rs = slot - g.kw;
    const int L0 = cw - (g.R - 1);
    const int w = L0 + ((rs - (L0 % g.R)) % g.R + g.R) % g.R;
    return w < cw || (r % g.om) < tv;
}

template <int DT>
__device__ __forceinline__ float ldcg_elt(const void* p, size_t i);
template <> __device__ __forceinline__ float ldcg_elt<QV_F32>(const void* p, size_t i) {
    return __ldcg(reinterpret_cast<const float*>(p) + i);
}
template <> __device__ __forceinline__ float ldcg_elt<QV_BF16>(const void* p, size_t i) {
    unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p) + i);
    return __uint_as_float(((uint32_t)u) << 16);
}
template <> __device__ __forceinline__ float ldcg_elt<QV_F16>(const void* p, size_t i) {
    unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p) + i);
    return __half2float(__ushort_as_half(u));
}

template <int DT>
__device__ __forceinline__ float logit_of(float dot, float inv_sqrt_unused, float sqrt_d) {
    // (q @ k^T) rounded to the KV dtype, then / sqrt(D) rounded (ops.py:38-40)
    return div_r<DT>(rnd<DT>(dot), sqrt_d);
}

template <int DT, int D, int BITS>
__global__ void __launch_bounds__(DEC_THREADS)
decode_split_kernel(Geo g, qv_layer L, const void* __restrict__ q, DecodeWs ws, void* __restrict__ out) {
    constexpr int VPL = D / 32;
    const int bh = blockIdx.y;
    const int b = bh / g.H, h = bh % g.H;
    const int split = blockIdx.x;
    const int nsplit = ws.n_main + ws.n_q;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = g.G;
    const float sqrt_d = sqrtf((float)D);
    const int N0 = L.step[0];
    const int cw = (N0 - g.sink) / g.om;
    const int tv = (N0 - g.sink) % g.om + 1;
    const size_t S_tot = (size_t)g.S_cap + (size_t)g.qw * g.om;

    float qr[MAXG][VPL];
#pragma unroll
    for (int gi = 0; gi < MAXG; ++gi)
#pragma unroll
        for (int i = 0; i < VPL; ++i)
            qr[gi][i] = gi < G ? ld<DT>(q, ((size_t)b * g.H * G + (size_t)h * G + gi) * D + lane * VPL + i) : 0.f;

    float m[MAXG], l[MAXG], o[MAXG][VPL];
#pragma unroll
    for (int gi = 0; gi < MAXG; ++gi) {
        m[gi] = -INFINITY; l[gi] = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) o[gi][i] = 0.f;
    }

    auto consume = [&](const float* kf, const float* vf, size_t lidx) {
#pragma unroll
        for (int gi = 0; gi < MAXG; ++gi) {
            if (gi >= G) break;
            float dot = 0.f;
#pragma unroll
            for (int i = 0; i < VPL; ++i) dot = fmaf(qr[gi][i], kf[i], dot);
            dot = warp_sum(dot);
            const float lg = logit_of<DT>(dot, 0.f, sqrt_d);
            if (lane == gi) st<DT>(ws.logits, lidx * G + gi, lg);
            const float mn = fmaxf(m[gi], lg);
            const float sc = expf(m[gi] - mn);
            const float pe = expf(lg - mn);
            l[gi] = l[gi] * sc + pe;
#pragma unroll
            for (int i = 0; i < VPL; ++i) o[gi][i] = o[gi][i] * sc + pe * vf[i];
            m[gi] = mn;
        }
    };

    if (split < ws.n_main) {
        const int32_t* swid = L.sticky_wid + (size_t)bh * g.kw;
        const int p0 = split * CH_MAIN;
        const int p1 = min(p0 + CH_MAIN, g.S_cap);
        const size_t base = (size_t)bh * g.S_cap;
        for (int pos = p0 + warp; pos < p1; pos += DEC_WARPS) {
            if (!main_live(g, swid, pos, cw, tv)) continue;
            float kf[VPL], vf[VPL];
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                kf[i] = ld<DT>(L.k, (base + pos) * D + lane * VPL + i);
                vf[i] = ld<DT>(L.v, (base + pos) * D + lane * VPL + i);
            }
            consume(kf, vf, (size_t)bh * S_tot + pos);
        }
    } else {
        const int t0 = (split - ws.n_main) * CH_Q;
        const int t1 = min(t0 + CH_Q, g.qw * g.om);
        const int32_t* qwid = L.q_wid + (size_t)bh * g.qw;
        const int qb = BITS == 4 ? D / 2 : D;
        for (int tok = t0 + warp; tok < t1; tok += DEC_WARPS) {
            const int slot = tok / g.om, t = tok % g.om;
            if (qwid[slot] < 0) continue;
            const size_t sw = (size_t)bh * g.qw + slot;
            const uint8_t* krow = L.kq + (sw * g.om + t) * qb;
            const uint8_t* vrow = L.vq + (sw * g.om + t) * qb;
            const float vsc = ld<DT>(L.vs, sw * g.om + t), vzp = ld<DT>(L.vz, sw * g.om + t);
            float kf[VPL], vf[VPL];
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                const int d = lane * VPL + i;
                kf[i] = dequant1<DT>(code_at(krow, d, BITS), ld<DT>(L.ks, sw * D + d), ld<DT>(L.kz, sw * D + d));
                vf[i] = dequant1<DT>(code_at(vrow, d, BITS), vsc, vzp);
            }
            consume(kf, vf, (size_t)bh * S_tot + g.S_cap + tok);
        }
    }

    // ---- merge the warps of this CTA into one partial --------------------------
    __shared__ float s_m[DEC_WARPS][MAXG], s_l[DEC_WARPS][MAXG];
    __shared__ float s_o[DEC_WARPS][MAXG][D];
    __shared__ int s_last;
#pragma unroll
    for (int gi = 0; gi < MAXG; ++gi) {
        if (gi >= G) break;
        if (lane == 0) { s_m[warp][gi] = m[gi]; s_l[warp][gi] = l[gi]; }
#pragma unroll
        for (int i = 0; i < VPL; ++i) s_o[warp][gi][lane * VPL + i] = o[gi][i];
    }
    __syncthreads();
    float* part = ws.partial + ((size_t)bh * nsplit + split) * G * (D + 2);
    for (int idx = threadIdx.x; idx < G * D; idx += DEC_THREADS) {
        const int gi = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, s_m[w][gi]);
        float acc = 0.f, ls = 0.f;
        if (M > -INFINITY) {
            for (int w = 0; w < DEC_WARPS; ++w) {
                const float e = expf(s_m[w][gi] - M);
                acc += s_o[w][gi][d] * e;
                ls += s_l[w][gi] * e;
            }
        }
        part[gi * (D + 2) + 2 + d] = acc;
        if (d == 0) { part[gi * (D + 2)] = M; part[gi * (D + 2) + 1] = ls; }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(ws.tickets + bh, 1) == nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---- last CTA of (b, h): merge splits, write output, fold the ledger --------
    __shared__ float s_M[MAXG], s_L[MAXG];
    const float* parts = ws.partial + (size_t)bh * nsplit * G * (D + 2);
    if (threadIdx.x < G) {
        const int gi = threadIdx.x;
        float M = -INFINITY;
        for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(parts + (size_t)s * G * (D + 2) + gi * (D + 2)));
        float Ls = 0.f;
        if (M > -INFINITY)
            for (int s = 0; s < nsplit; ++s) {
                const float* pr = parts + (size_t)s * G * (D + 2) + gi * (D + 2);
                const float ms = __ldcg(pr);
                if (ms > -INFINITY) Ls += __ldcg(pr + 1) * expf(ms - M);
            }
        s_M[gi] = M; s_L[gi] = Ls;
    }
    __syncthreads();
    const bool has_q = L.seq[b * 4 + 1] > 0;
    for (int idx = threadIdx.x; idx < G * D; idx += DEC_THREADS) {
        const int gi = idx / D, d = idx % D;
        float om_ = 0.f, oq = 0.f;
        for (int s = 0; s < nsplit; ++s) {
            const float* pr = parts + (size_t)s * G * (D + 2) + gi * (D + 2);
            const float ms = __ldcg(pr);
            if (ms == -INFINITY) continue;
            const float c = __ldcg(pr + 2 + d) * expf(ms - s_M[gi]);
            if (s < ws.n_main) om_ += c; else oq += c;
        }
        const float inv = 1.f / s_L[gi];
        float r = has_q ? add_r<DT>(rnd<DT>(om_ * inv), rnd<DT>(oq * inv)) : rnd<DT>(om_ * inv);
        st<DT>(out, ((size_t)b * g.H * G + (size_t)h * G + gi) * D + d, r);
    }
    // main-zone votes
    const int32_t* swid = L.sticky_wid + (size_t)bh * g.kw;
    for (int pos = threadIdx.x; pos < g.S_cap; pos += DEC_THREADS) {
        if (!main_live(g, swid, pos, cw, tv)) continue;
        float acc = 0.f;
        for (int gi = 0; gi < G; ++gi) {
            const float lg = ldcg_elt<DT>(ws.logits, ((size_t)bh * S_tot + pos) * G + gi);
            acc += rnd<DT>(expf(lg - s_M[gi]) / s_L[gi]);
        }
        L.votes[(size_t)bh * g.S_cap + pos] += rnd<DT>(acc / (float)G);
    }
    // Q-window scores: sum of the window's group-mean probabilities, rounded once
    const int32_t* qwid = L.q_wid + (size_t)bh * g.qw;
    for (int slot = warp; slot < g.qw; slot += DEC_WARPS) {
        if (qwid[slot] < 0) continue;
        float a = 0.f;
        bool first = true;
        for (int t = lane; t < g.om; t += 32) {
            const size_t li = (size_t)bh * S_tot + g.S_cap + (size_t)slot * g.om + t;
            float acc = 0.f;
            for (int gi = 0; gi < G; ++gi)
                acc += rnd<DT>(expf(ldcg_elt<DT>(ws.logits, li * G + gi) - s_M[gi]) / s_L[gi]);
            const float mean = rnd<DT>(acc / (float)G);
            a = first ? mean : a + mean;
            first = false;
        }
        a = warp_sum(a);
        if (lane == 0) L.q_score[(size_t)bh * g.qw + slot] += rnd<DT>(a);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        ws.tickets[bh] = 0;
        __threadfence();
        const int BH = g.B * g.H;
        if (atomicAdd(ws.tickets + BH, 1) == BH - 1) {
            ws.tickets[BH] = 0;
            L.step[0] = N0 + 1;
        }
    }
}

// ---- RoPE + append ----------------------------------------------------------
// One CTA per (sequence, row): rows are the G*H query heads, then the H new keys,
// then the H new values.  blockDim = D.
template <int DT>
__global__ void rope_append_kernel(Geo g, qv_layer L, const void* __restrict__ q_in, const void* __restrict__ k_in,
                                   const void* __restrict__ v_in, const void* __restrict__ cos_t,
                                   const void* __restrict__ sin_t, void* __restrict__ q_out) {
    // the attention kernel may start its prologue now (it waits for this grid)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int b = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
    const int N0 = L.step[0];
    const int D = g.D, half = D / 2;
    const int nq = g.H * g.G;
    const void* src;
    size_t si;
    if (r < nq) { src = q_in; si = ((size_t)b * nq + r) * D; }
    else if (r < nq + g.H) { src = k_in; si = ((size_t)b * g.H + (r - nq)) * D; }
    else { src = v_in; si = ((size_t)b * g.H + (r - nq - g.H)) * D; }
    float x = ld<DT>(src, si + d);
    if (cos_t != nullptr && r < nq + g.H) {
        // (x * cos) + (rotate_half(x) * sin)   (helpers.py:56-62)
        const float xr = d < half ? -ld<DT>(src, si + d + half) : ld<DT>(src, si + d - half);
        const float c = ld<DT>(cos_t, (size_t)N0 * D + d), sn = ld<DT>(sin_t, (size_t)N0 * D + d);
        x = add_r<DT>(mul_r<DT>(x, c), mul_r<DT>(xr, sn));
    }
    if (r < nq) {
        st<DT>(q_out, si + d, x);
    } else {
        const int w = (N0 - g.sink) / g.om;
        const int off = (N0 - g.sink) % g.om;
        const int ppos = g.ring_base() + (w % g.R) * g.om + off;
        const int hh = r < nq + g.H ? r - nq : r - nq - g.H;
        void* dst = r < nq + g.H ? L.k : L.v;
        st<DT>(dst, (((size_t)b * g.H + hh) * g.S_cap + ppos) * D + d, x);
    }
}

// RoPE of a token-major block x[b][s][head][d] at positions pos0 + s (in place).
template <int DT>
__global__ void rope_tokens_kernel(int heads, int D, void* __restrict__ x, const void* __restrict__ cos_t,
                                   const void* __restrict__ sin_t, int S, int pos0) {
    const size_t row = blockIdx.x;  // (b * S + s) * heads + head
    const int s = (int)((row / heads) % S);
    const int pos = pos0 + s;
    const int half = D / 2;
    extern __shared__ float rrow[];
    for (int d = threadIdx.x; d < D; d += blockDim.x) rrow[d] = ld<DT>(x, row * D + d);
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float xv = rrow[d];
        const float xr = d < half ? -rrow[d + half] : rrow[d - half];
        const float c = ld<DT>(cos_t, (size_t)pos * D + d), sn = ld<DT>(sin_t, (size_t)pos * D + d);
        st<DT>(x, row * D + d, add_r<DT>(mul_r<DT>(xv, c), mul_r<DT>(xr, sn)));
    }
}

// tensor-core kernel for the production shape (decode_mma.cu)
bool mm_supported(const Geo& g);
size_t mm_ws_bytes(const Geo& g, size_t* off_part, size_t* off_logits);
int mm_launch(const Geo& g, const qv_layer& L, const void* q, void* out, void* ws, cudaStream_t s, int mode);

}  // namespace qv

using namespace qv;

extern "C" int qv_rope(int32_t batch, int32_t seq, int32_t heads, int32_t head_dim, int32_t dtype, void* x,
                       const void* cos_tab, const void* sin_tab, int32_t pos0, qv_stream_t stream) {
    if (batch <= 0 || seq <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 2 || !x || !cos_tab || !sin_tab || pos0 < 0)
        return QV_EINVAL;
    const size_t rows = (size_t)batch * seq * heads;
    const size_t sm = head_dim * sizeof(float);
    cudaStream_t s = (cudaStream_t)stream;
    switch (dtype) {
        case QV_F32: rope_tokens_kernel<QV_F32><<<rows, 128, sm, s>>>(heads, head_dim, x, cos_tab, sin_tab, seq, pos0); break;
        case QV_BF16: rope_tokens_kernel<QV_BF16><<<rows, 128, sm, s>>>(heads, head_dim, x, cos_tab, sin_tab, seq, pos0); break;
        case QV_F16: rope_tokens_kernel<QV_F16><<<rows, 128, sm, s>>>(heads, head_dim, x, cos_tab, sin_tab, seq, pos0); break;
        default: return QV_EINVAL;
    }
    return check_launch();
}

extern "C" int32_t qv_decode_path(const qv_dims* d) {
    if (validate_dims(d)) return -1;
    return mm_supported(make_geo(d)) ? 1 : 0;
}

extern "C" size_t qv_decode_logits_offset(const qv_dims* d) {
    if (validate_dims(d)) return 0;
    Geo g = make_geo(d);
    size_t a, b, t;
    if (mm_supported(g)) {
        mm_ws_bytes(g, &a, &b);
        return b;
    }
    int nm, nq;
    decode_ws_layout(g, &a, &b, &t, &nm, &nq);
    return b;
}

extern "C" size_t qv_decode_workspace_bytes(const qv_dims* d) {
    if (validate_dims(d)) return 0;
    Geo g = make_geo(d);
    size_t a, b, t;
    int nm, nq;
    decode_ws_layout(g, &a, &b, &t, &nm, &nq);
    if (mm_supported(g)) {
        const size_t t2 = mm_ws_bytes(g, &a, &b);
        if (t2 > t) t = t2;
    }
    return t;
}

extern "C" int qv_rope_append(const qv_dims* d, const qv_layer* L, const void* q_in, const void* k_in,
                              const void* v_in, const void* cos_tab, const void* sin_tab, void* q_out,
                              qv_stream_t stream) {
    int rc = validate_dims(d);
    if (rc) return rc;
    if (!L || !q_in || !k_in || !v_in || !q_out || !L->k || !L->v || !L->step) return QV_EINVAL;
    if ((cos_tab == nullptr) != (sin_tab == nullptr)) return QV_EINVAL;
    Geo g = make_geo(d);
    cudaStream_t s = (cudaStream_t)stream;
    const dim3 grid(g.B, g.H * g.G + 2 * g.H);
    switch (g.dt) {
        case QV_F32: rope_append_kernel<QV_F32><<<grid, g.D, 0, s>>>(g, *L, q_in, k_in, v_in, cos_tab, sin_tab, q_out); break;
        case QV_BF16: rope_append_kernel<QV_BF16><<<grid, g.D, 0, s>>>(g, *L, q_in, k_in, v_in, cos_tab, sin_tab, q_out); break;
        default: rope_append_kernel<QV_F16><<<grid, g.D, 0, s>>>(g, *L, q_in, k_in, v_in, cos_tab, sin_tab, q_out); break;
    }
    return check_launch();
}

template <int DT, int D>
static void launch_decode(const Geo& g, const qv_layer& L, const void* q, DecodeWs ws, void* out, cudaStream_t s) {
    dim3 grid(ws.n_main + ws.n_q, g.B * g.H);
    if (g.bits == 8) decode_split_kernel<DT, D, 8><<<grid, DEC_THREADS, 0, s>>>(g, L, q, ws, out);
    else decode_split_kernel<DT, D, 4><<<grid, DEC_THREADS, 0, s>>>(g, L, q, ws, out);
}

// mode: 0 = attention + ledger fold, 1 = attention (fold pending), 2 = the pending fold
static int decode_attention_mode(const qv_dims* d, const qv_layer* L, const void* q, void* out, void* workspace,
                                 size_t workspace_bytes, qv_stream_t stream, int mode) {
    int rc = validate_dims(d);
    if (rc) return rc;
    if (!L || !workspace || (mode != 2 && (!q || !out))) return QV_EINVAL;
    Geo g = make_geo(d);
    size_t op, ol, tot;
    DecodeWs ws;
    decode_ws_layout(g, &op, &ol, &tot, &ws.n_main, &ws.n_q);
    if (workspace_bytes < tot) return QV_ESPACE;
    cudaStream_t s = (cudaStream_t)stream;
    if (mm_supported(g)) {
        size_t a2, b2;
        if (workspace_bytes < mm_ws_bytes(g, &a2, &b2)) return QV_ESPACE;
        return mm_launch(g, *L, q, out, workspace, s, mode);
    }
    // the CUDA-core kernel folds the ledger inside the attention launch
    if (mode == 2) return QV_OK;
    char* base = reinterpret_cast<char*>(workspace);
    ws.tickets = reinterpret_cast<int*>(base);
    ws.partial = reinterpret_cast<float*>(base + op);
    ws.logits = base + ol;
    switch (g.dt) {
        case QV_F32: if (g.D == 128) launch_decode<QV_F32, 128>(g, *L, q, ws, out, s); else launch_decode<QV_F32, 64>(g, *L, q, ws, out, s); break;
        case QV_BF16: if (g.D == 128) launch_decode<QV_BF16, 128>(g, *L, q, ws, out, s); else launch_decode<QV_BF16, 64>(g, *L, q, ws, out, s); break;
        default: if (g.D == 128) launch_decode<QV_F16, 128>(g, *L, q, ws, out, s); else launch_decode<QV_F16, 64>(g, *L, q, ws, out, s); break;
    }
    return check_launch();
}

extern "C" int qv_decode_attention(const qv_dims* d, const qv_layer* L, const void* q, void* out,
                                   void* workspace, size_t workspace_bytes, qv_stream_t stream) {
    return decode_attention_mode(d, L, q, out, workspace, workspace_bytes, stream, 0);
}

extern "C" int qv_decode_attention_nofold(const qv_dims* d, const qv_layer* L, const void* q, void* out,
                                          void* workspace, size_t workspace_bytes, qv_stream_t stream) {
    return decode_attention_mode(d, L, q, out, workspace, workspace_bytes, stream, 1);
}

extern "C" int qv_decode_fold(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                              qv_stream_t stream) {
    return decode_attention_mode(d, L, nullptr, nullptr, workspace, workspace_bytes, stream, 2);
}
