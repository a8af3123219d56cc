// Research token ledger on the device: the three updates of the reference's
// TrackingManager (src/models/kv_cache/tracking_manager.py:27-204).
//
// One sequence per call.  ledger [C][2 + 2H] float32 rows of (global id,
// layer id, physical position per head, cumulative importance per head) and
// history [C][H] float32, C = max_context; positions index the reference's
// physical cache order.  Every value written is the reference's float32
// arithmetic on the same operands, so the tables match bit for bit.
//
// One thread per ledger row (rows are independent in all three updates); a
// row is 2 + 2H floats, so the threads of a warp sweep one contiguous span of
// the table.
#include <stdint.h>

#include "common.cuh"

namespace qv {

constexpr int TK_THREADS = 256;

// record_prefill, first half (tracking_manager.py:77-101 and the reset of the
// position columns at :112): fill the rows of the new tokens, copy the
// pre-eviction importance into live rows, clear every row's positions.
__global__ void __launch_bounds__(TK_THREADS) track_prefill_rows(int C, int H, int seq_len, int q_len, int layer,
                                                                 long long g0, int num_new,
                                                                 const float* __restrict__ imp, int kv,
                                                                 float* __restrict__ ledger,
                                                                 float* __restrict__ hist) {
    const long long g = (long long)blockIdx.x * TK_THREADS + threadIdx.x;
    if (g >= C) return;
    float* row = ledger + g * (2 + 2 * H);
    if (g >= g0 && g < g0 + num_new) {
        row[0] = (float)g;
        row[1] = (float)layer;
        const float p = (float)(seq_len - q_len + (g - g0));
        for (int h = 0; h < H; ++h) row[2 + h] = p;
    }
    if (g < (long long)min(seq_len, C)) {
        bool live = false;
        for (int h = 0; h < H; ++h) live |= row[2 + h] >= 0.f;
        if (live && row[0] >= 0.f) {
            const long long p = (long long)row[2];   // head 0's position picks the column (:92)
            if (p >= 0 && p < kv)
                for (int h = 0; h < H; ++h) {
                    const float v = imp[(size_t)h * kv + p];
                    row[2 + H + h] = v;
                    hist[g * H + h] = v;
                }
        }
    }
    for (int h = 0; h < H; ++h) row[2 + h] = -1.f;
}

// record_prefill, second half (:113-124): survivors get their compressed
// position and their importance.  One thread per (head, survivor).
__global__ void __launch_bounds__(TK_THREADS) track_prefill_survivors(int C, int H, int seq_len, long long g0,
                                                                      int num_new, const float* __restrict__ imp,
                                                                      int kv, const int64_t* __restrict__ surv,
                                                                      int n_surv, float* __restrict__ ledger) {
    const long long t = (long long)blockIdx.x * TK_THREADS + threadIdx.x;
    if (t >= (long long)H * n_surv) return;
    const int h = (int)(t / n_surv), j = (int)(t % n_surv);
    const long long s = surv[t];
    const long long g = g0 + s - (seq_len - num_new);
    if (g < 0 || g >= C) return;
    float* row = ledger + g * (2 + 2 * H);
    row[2 + h] = (float)j;
    if (s < kv) {
        const long long i = s < 0 ? s + kv : s;   // torch's negative indexing
        if (i >= 0) row[2 + H + h] = imp[(size_t)h * kv + i];
    }
}

// record_decode (:126-160): the new token's row, then every live row adds its
// score at its position (0 where the position is outside the score row).
__global__ void __launch_bounds__(TK_THREADS) track_decode_rows(int C, int H, long long n_active, long long g_new,
                                                                int seq_len, int layer,
                                                                const float* __restrict__ sc, int kv,
                                                                float* __restrict__ ledger,
                                                                float* __restrict__ hist) {
    const long long g = (long long)blockIdx.x * TK_THREADS + threadIdx.x;
    if (g >= C) return;
    float* row = ledger + g * (2 + 2 * H);
    if (g == g_new) {
        row[0] = (float)g;
        row[1] = (float)layer;
        for (int h = 0; h < H; ++h) {
            row[2 + h] = (float)(seq_len - 1);
            row[2 + H + h] = 0.f;
            hist[g * H + h] = 0.f;
        }
    }
    if (g >= n_active) return;
    bool live = false;
    for (int h = 0; h < H; ++h) live |= row[2 + h] >= 0.f;
    if (!live) return;
    for (int h = 0; h < H; ++h) {
        const long long p = (long long)row[2 + h];
        const bool in = p >= 0 && p < kv;
        const long long q = p < 0 ? 0 : (p > kv - 1 ? kv - 1 : p);
        const float v = sc[(size_t)h * kv + q] * (in ? 1.f : 0.f);
        row[2 + H + h] += v;
        hist[g * H + h] += v;
    }
}

// update_physical_positions (:162-191): move live rows to their new
// positions; a token that leaves the cache adds the cycle's vote at its old
// position once more.
__global__ void __launch_bounds__(TK_THREADS) track_position_rows(int C, int H, long long n_active, int seq_len,
                                                                  const float* __restrict__ mapping,
                                                                  const float* __restrict__ votes, int vstride,
                                                                  float* __restrict__ ledger,
                                                                  float* __restrict__ hist) {
    const long long g = (long long)blockIdx.x * TK_THREADS + threadIdx.x;
    if (g >= n_active) return;
    float* row = ledger + g * (2 + 2 * H);
    bool live = false;
    for (int h = 0; h < H; ++h) live |= row[2 + h] >= 0.f;
    if (!live) return;
    for (int h = 0; h < H; ++h) {
        const long long p = (long long)row[2 + h];
        const bool valid = p >= 0 && p < seq_len;
        const long long q = p < 0 ? 0 : (p > seq_len - 1 ? seq_len - 1 : p);
        const float nm = valid ? mapping[(size_t)h * seq_len + q] : -1.f;
        const bool evicted = nm < 0.f && valid;
        const float v = votes[(size_t)h * vstride + q] * (evicted ? 1.f : 0.f);
        row[2 + H + h] += v;
        hist[g * H + h] += v;
        row[2 + h] = nm;
    }
}

static unsigned tk_blocks(long long rows) { return (unsigned)((rows + TK_THREADS - 1) / TK_THREADS); }

}  // namespace qv

using namespace qv;

extern "C" int qv_track_prefill(int32_t max_context, int32_t heads, int32_t seq_len, int32_t q_len, int32_t layer_idx,
                                int64_t global_start, int32_t num_new, const float* importance, int32_t kv_len,
                                const int64_t* survivors, int32_t n_surv, float* ledger, float* history,
                                qv_stream_t stream) {
    if (max_context <= 0 || heads <= 0 || seq_len <= 0 || q_len < 0 || num_new < 0 || global_start < 0 ||
        kv_len <= 0 || n_surv < 0 || !importance || !ledger || !history || (n_surv > 0 && !survivors))
        return QV_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    track_prefill_rows<<<tk_blocks(max_context), TK_THREADS, 0, s>>>(max_context, heads, seq_len, q_len, layer_idx,
                                                                     global_start, num_new, importance, kv_len,
                                                                     ledger, history);
    if (n_surv > 0)
        track_prefill_survivors<<<tk_blocks((long long)heads * n_surv), TK_THREADS, 0, s>>>(
            max_context, heads, seq_len, global_start, num_new, importance, kv_len, survivors, n_surv, ledger);
    return check_launch();
}

extern "C" int qv_track_decode(int32_t max_context, int32_t heads, int64_t counter, int64_t global_start,
                               int32_t seq_len, int32_t layer_idx, const float* scores, int32_t kv_len, float* ledger,
                               float* history, qv_stream_t stream) {
    if (max_context <= 0 || heads <= 0 || counter < 0 || global_start < 0 || seq_len <= 0 || kv_len <= 0 ||
        !scores || !ledger || !history)
        return QV_EINVAL;
    const long long n_active = counter < max_context ? counter : max_context;
    const long long rows = global_start < max_context ? (global_start + 1 > n_active ? global_start + 1 : n_active)
                                                      : n_active;
    if (rows == 0) return QV_OK;
    track_decode_rows<<<tk_blocks(rows), TK_THREADS, 0, (cudaStream_t)stream>>>(
        max_context, heads, n_active, global_start, seq_len, layer_idx, scores, kv_len, ledger, history);
    return check_launch();
}

extern "C" int qv_track_positions(int32_t max_context, int32_t heads, int64_t counter, int32_t seq_len,
                                  const float* mapping, const float* votes, int32_t votes_stride, float* ledger,
                                  float* history, qv_stream_t stream) {
    if (max_context <= 0 || heads <= 0 || counter < 0 || seq_len <= 0 || votes_stride < seq_len || !mapping ||
        !votes || !ledger || !history)
        return QV_EINVAL;
    const long long n_active = counter < max_context ? counter : max_context;
    if (n_active == 0) return QV_OK;
    track_position_rows<<<tk_blocks(n_active), TK_THREADS, 0, (cudaStream_t)stream>>>(
        max_context, heads, n_active, seq_len, mapping, votes, votes_stride, ledger, history);
    return check_launch();
}
