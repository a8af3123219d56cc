/*
 * qevict_b200.h -- C ABI of the B200 (sm_100a) Sticky-KV hot path.
 *
 * Plain device pointers and sizes; no framework types.  Every entry point is
 * stream-ordered, never synchronises the host, never allocates, and returns
 * QV_OK (0) or a negative QV_E* code for invalid arguments.  Problems that can
 * only be seen on the device (an index outside a table, a window that is not
 * where the layout says it is) set bits in the layer's device error word,
 * which qv_read_error() copies out on demand.
 *
 * Layout of one layer's state in HBM ("slot layout").  For sequence b, KV head h:
 *
 *   main zone  K,V  [B][H][S_cap][D]  (kv dtype), S_cap = sink + k_windows*omega + ring_windows*omega
 *       [0, sink)                                   attention sinks
 *       [sink + s*omega, +omega)      s < k_windows  sticky slot s, holding window sticky_wid[b][h][s]
 *       [sink + (k_windows + r)*omega, +omega)      ring slot r = w % ring_windows holds local window w
 *   Q zone     kq,vq [B][H][q_windows][omega][D or D/2] u8, ks,kz [B][H][q_windows][D],
 *              vs,vz [B][H][q_windows][omega]  (kv dtype); slot j holds window q_wid[b][h][j]
 *
 * Sticky and Q slots are unordered; sticky_order / q_order give the slot of
 * each logical rank (sticky: ascending window id, as the reference keeps
 * window_scores; Q: the reference's top-k order).  Only windows that change
 * tier move during an eviction cycle.
 *
 * The reference (shaswata965-coder/Qevict) is Python/PyTorch; the entry points
 * below replace the torch-op groups cited beside each one.  A ctypes binding
 * is in qevict_b200/_native.py.
 */
#ifndef QEVICT_B200_H
#define QEVICT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qv_stream_t; /* a cudaStream_t */

enum {
    QV_OK = 0,
    QV_EINVAL = -1,     /* bad dimension / null pointer / unsupported combination */
    QV_ENOTALIGNED = -2,/* prompt or local zone not a whole number of windows */
    QV_ESPACE = -3,     /* workspace too small */
    QV_ECUDA = -4,      /* a CUDA launch failed (see qv_last_cuda_error) */
};

enum { QV_F32 = 0, QV_BF16 = 1, QV_F16 = 2 };

/* device error word bits (qv_read_error) */
enum {
    QV_DERR_TABLE = 1 << 0,    /* window id outside [0, max_windows) */
    QV_DERR_LAYOUT = 1 << 1,   /* a window was not found where the layout says it is */
    QV_DERR_CAPACITY = 1 << 2, /* more movers than free slots */
    QV_DERR_TIMEOUT = 1 << 3,  /* a bounded wait of a pipelined kernel gave up (the output is not valid) */
};

typedef struct qv_dims {
    int32_t batch;        /* sequences decoded in lockstep */
    int32_t kv_heads;     /* H */
    int32_t group;        /* query heads per KV head (G) */
    int32_t head_dim;     /* D: 64 or 128 */
    int32_t omega;        /* window length, multiple of 16, <= 128 */
    int32_t sink;         /* attention-sink tokens */
    int32_t local;        /* local-zone tokens, multiple of omega */
    int32_t k_windows;    /* sticky capacity (windows) */
    int32_t q_windows;    /* Q-cache capacity (windows), may be 0 */
    int32_t max_windows;  /* window-id table size */
    int32_t bits;         /* 8 or 4 */
    int32_t dtype;        /* QV_F32 / QV_BF16 / QV_F16 */
    int32_t flags;        /* QV_FLAG_* */
} qv_dims;

/* qv_dims.flags */
enum {
    /* Decode attention dequantises Q-cache codes with the reference's own
     * rounding, rnd(rnd(code*scale) + zp) in the KV dtype (quantize.py:62-71),
     * on the CUDA-core kernel.  Without the flag, head_dim-128 / omega-64 /
     * INT8 / BF16-or-FP16 layers use the tensor-core kernel, which applies the
     * scale and zero point exactly in fp32 instead. */
    QV_FLAG_REFERENCE_ROUNDING = 1,
};

typedef struct qv_layer {
    void* k;                 /* [B][H][S_cap][D] */
    void* v;
    uint8_t* kq;             /* [B][H][q_windows][omega][qbytes] */
    uint8_t* vq;
    void* ks;                /* [B][H][q_windows][D] */
    void* kz;
    void* vs;                /* [B][H][q_windows][omega] */
    void* vz;
    int32_t* sticky_wid;     /* [B][H][k_windows]  -1 = empty */
    float* sticky_score;     /* [B][H][k_windows] */
    int32_t* sticky_order;   /* [B][H][k_windows]  rank (ascending id) -> slot */
    int32_t* q_wid;          /* [B][H][q_windows]  -1 = empty */
    float* q_score;          /* [B][H][q_windows] */
    int32_t* q_order;        /* [B][H][q_windows]  rank (top-k order) -> slot */
    float* votes;            /* [B][H][S_cap] running attention votes (fp32) */
    float* local_hist;       /* [B][H][max_windows] */
    uint8_t* arch_valid;     /* [B][H][max_windows] path-C archive flags */
    void* arch_ks;           /* [B][H][max_windows][D] */
    void* arch_kz;
    void* arch_vs;           /* [B][H][max_windows][omega] */
    void* arch_vz;
    int32_t* seq;            /* [B][4]: curr_k, q_count, reserved, reserved */
    int32_t* step;           /* [4]: tokens in cache (incl. prompt), prompt length, reserved */
    int32_t* err;            /* [1] device error word */
} qv_layer;

/* ---- sizes -------------------------------------------------------------- */
int32_t qv_ring_windows(const qv_dims* d);            /* local/omega + 1 */
int32_t qv_main_capacity(const qv_dims* d);           /* S_cap */
size_t qv_decode_workspace_bytes(const qv_dims* d);
/* Which decode-attention kernel qv_decode_attention runs for these dims:
 * 0 = CUDA-core kernel with the reference's dequantisation rounding,
 * 1 = tensor-core kernel (TMA pipeline, exact fp32 dequantisation). */
int32_t qv_decode_path(const qv_dims* d);
/* Byte offset, inside the decode workspace, of the rounded logits the last
 * qv_decode_attention wrote: [B*H][S_cap + q_windows*omega][group] in the KV
 * dtype, main-zone positions in slot layout followed by the Q slots (used by
 * the parity tests to separate accumulation-order effects from the rest). */
size_t qv_decode_logits_offset(const qv_dims* d);
size_t qv_cycle_workspace_bytes(const qv_dims* d);

/* ---- decode step ------------------------------------------------------- */

/* RoPE on the new query/key (HF rotate_half form) and in-place append of the
 * new K/V token at its ring slot.  Replaces apply_rotary_pos_emb_single
 * (src/models/kv_cache/helpers.py:56-62) applied at module.py:188-189 and the
 * O(S) torch.cat append (src/models/attention/module.py:198-200).
 * q_in [B][G*H][D], k_in/v_in [B][H][D]; cos/sin [max_pos][D] (kv dtype);
 * q_out [B][G*H][D].  cos/sin may be NULL when the inputs are already rotated. */
int qv_rope_append(const qv_dims* d, const qv_layer* L, const void* q_in, const void* k_in,
                   const void* v_in, const void* cos_tab, const void* sin_tab, void* q_out,
                   qv_stream_t stream);

/* RoPE of a token-major block x[batch][seq][heads][head_dim] at positions
 * pos0 .. pos0+seq-1, in place, HF rotate_half form with the reference's
 * rounding: (x*cos) + (rotate_half(x)*sin), each op rounded to the dtype
 * (src/models/kv_cache/helpers.py:56-62, applied at module.py:188-189 for the
 * prompt).  cos/sin [max_pos][head_dim] in the same dtype. */
int qv_rope(int32_t batch, int32_t seq, int32_t heads, int32_t head_dim, int32_t dtype, void* x,
            const void* cos_tab, const void* sin_tab, int32_t pos0, qv_stream_t stream);

/* Fused split-K decode attention over [sinks | sticky slots | ring] plus the
 * INT8/INT4 Q-cache, with the ledger fold.  Replaces compute_main_logits +
 * compute_qcache_joint_softmax / compute_standard_softmax
 * (src/models/attention/ops.py:23-46, 74-169, 176-212), the vote tally
 * EvictionManager.tally_decode_scores (src/models/kv_cache/eviction_manager.py:198-203)
 * and QuantizationManager.accumulate_scores (src/models/kv_cache/quantize_manager.py:101-111).
 * q [B][G*H][D] rotated; out [B][G*H][D].  Advances step[0] by one token.
 * Launched as a programmatic dependent of the preceding kernel on the stream:
 * it reads step[0], the slot tables and every cached token except the new one
 * before that kernel has finished (only the new token and q are read after
 * it), so the call must directly follow qv_rope_append on the same stream, or
 * follow a kernel that writes none of this layer's state. */
int qv_decode_attention(const qv_dims* d, const qv_layer* L, const void* q, void* out,
                        void* workspace, size_t workspace_bytes, qv_stream_t stream);

/* qv_decode_attention in two launches, so that the vote-ledger fold can run
 * off the critical path (on another stream, beside the next projections).
 * No counterpart in the reference (its tally follows its attention in one
 * Python call, eviction_manager.py:198-203).
 * qv_decode_attention_nofold writes out and advances step[0]; the fold of this
 * step's probabilities into votes / q_score is left pending.
 * qv_decode_fold performs the pending fold.  It must be ordered after the
 * nofold call (same stream, or an event) and before the next qv_rope_append,
 * qv_decode_attention* or qv_evict_cycle on this layer, and before the
 * workspace is used again.  On the CUDA-core path (qv_decode_path() == 0) the
 * nofold call folds the ledger itself and qv_decode_fold does nothing. */
int qv_decode_attention_nofold(const qv_dims* d, const qv_layer* L, const void* q, void* out,
                               void* workspace, size_t workspace_bytes, qv_stream_t stream);
int qv_decode_fold(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                   qv_stream_t stream);

/* qv_decode_attention without a workspace argument; no counterpart in the
 * reference.  For callers that cannot allocate device memory between decode
 * steps (a foreign-language host holding only the layer's pointers, or a
 * serving loop that must not call cudaMalloc/cudaFree).  Its scratch is a
 * fixed device array of QV_NOALLOC_SCRATCH_BYTES inside this library (8 MiB:
 * batch 8 at the Llama-3-8B layer shape, 32 sticky + 32 Q windows of 64,
 * local 512, fits); dims whose qv_decode_workspace_bytes exceeds it return
 * QV_ESPACE with a message in qv_last_cuda_error().  The scratch is shared per
 * device, so calls that overlap in time race on it; the first call on a
 * device looks up the scratch address and should come before any capture or
 * timed loop.  The address is cached per device and CUDA context: after a
 * device reset the next call looks it up again (outside any capture).
 * Ordering as qv_decode_attention (a programmatic dependent: directly after
 * qv_rope_append on the same stream).  Results are those of
 * qv_decode_attention, except that the logits are not exposed. */
#define QV_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int qv_decode_attention_noalloc(const qv_dims* d, const qv_layer* L, const void* q, void* out,
                                qv_stream_t stream);

/* One eviction cycle (every omega tokens): scoreboard, window competition,
 * segmented top-k, promotion, Q-cache rebuild (paths A/B/C) and slot moves.
 * Replaces EvictionManager.run_decode_cycle / update_local_history /
 * commit_decode_result / reset_decode_counters (eviction_manager.py:205-417),
 * QuantizationManager.get_promoted_windows / rebuild (quantize_manager.py:114-327)
 * and STICKYKVCache_LayerWise._build_physical_cache (src/models/kv_cache/cache.py:433-575). */
int qv_evict_cycle(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                   qv_stream_t stream);

/* The eviction cycle of a layer whose KV heads are split over several devices
 * (one qv_layer per device, dims.kv_heads = the local heads).  The cycle's one
 * coupling between heads -- the number of Q-cache losers is the minimum over
 * all heads of the candidates left after the top-k (eviction_manager.py:335-345)
 * -- needs the heads of every device: qv_evict_cycle_count writes the local
 * minimum per sequence (int32 [batch]) and changes nothing else; after a MIN
 * reduction of those counts over the devices, qv_evict_cycle_ext runs the cycle
 * with the global minimum.  On one device qv_evict_cycle is the same as
 * count + ext with the local counts.  No counterpart in the reference, which
 * keeps all heads of a layer on one device. */
int qv_evict_cycle_count(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                         int32_t* loser_count, qv_stream_t stream);
int qv_evict_cycle_ext(const qv_dims* d, const qv_layer* L, void* workspace, size_t workspace_bytes,
                       const int32_t* loser_count, qv_stream_t stream);

/* ---- prefill ----------------------------------------------------------- */

/* Build the layer state from a prompt: window tally, top-k/top-q selection,
 * Q-cache store, compaction into the slot layout.  Replaces the prefill branch
 * of STICKYKVCache_LayerWise.__call__ (cache.py:269-355): tally_prefill_scores
 * (eviction_manager.py:115-173), evict_from_window_scores (eviction.py:102-156),
 * store_windows (quantize_manager.py:91-98),
 * create_mask_and_evict_from_kv_cache_prompt_stage (eviction.py:163-240).
 * k_prompt/v_prompt [B][H][S][D] rotated; colsum [B][H][S] per-key column sums
 * (score_dtype QV_F32 for the flash path, or the kv dtype for the SDPA path,
 * whose window sums the reference rounds to that dtype). */
int qv_prefill_build(const qv_dims* d, const qv_layer* L, const void* k_prompt, const void* v_prompt,
                     int32_t prompt_len, const void* colsum, int32_t score_dtype, qv_stream_t stream);

/* Causal prefill attention that also emits the per-key column sums of the
 * GQA-group-mean softmax (512-query chunks rounded to the kv dtype, fp32
 * across chunks).  Replaces flash_attn_func + compute_chunked_prefill_scores
 * (src/models/attention/ops_flash.py:22-141).
 * q [B][S][G*H][D], k,v [B][S][H][D] (rotated); out [B][S][G*H][D]; colsum [B][H][S] fp32.
 * Workspace (qv_prefill_workspace_bytes): per-row softmax statistics, and for
 * bf16/fp16 the column-sum partials, a triangle of about S*S*G/256 fp32 values
 * per sequence and KV head (0.54 GB for 8 KV heads, G = 4, S = 32768). */
int qv_prefill_attention(const qv_dims* d, const void* q, const void* k, const void* v, int32_t seq_len,
                         void* out, float* colsum, void* workspace, size_t workspace_bytes,
                         qv_stream_t stream);
size_t qv_prefill_workspace_bytes(const qv_dims* d, int32_t seq_len);
/* The device error word of the last qv_prefill_attention on this workspace
 * (0, or QV_DERR_TIMEOUT when a pipelined kernel gave up waiting and its
 * outputs are not valid); pass the workspace and size given to
 * qv_prefill_attention.  Synchronises the stream. */
int qv_prefill_read_error(const void* workspace, size_t workspace_bytes, int32_t* host_err, qv_stream_t stream);

/* ---- codec (the reference's static methods) ----------------------------- */

/* quantize_k_per_window / quantize_v_per_window / dequantize_from_quant
 * (src/models/kv_cache/quantize.py:19-71), for n windows of [omega][D]:
 * x [n][omega][D]; codes [n][omega][D or D/2]; K: scale/zp [n][D]; V: scale/zp [n][omega]. */
int qv_quantize_k(int32_t n, int32_t omega, int32_t head_dim, int32_t bits, int32_t dtype,
                  const void* x, uint8_t* codes, void* scale, void* zp, qv_stream_t stream);
int qv_quantize_v(int32_t n, int32_t omega, int32_t head_dim, int32_t bits, int32_t dtype,
                  const void* x, uint8_t* codes, void* scale, void* zp, qv_stream_t stream);
/* per_token = 0: scale/zp [n][D] (K); 1: scale/zp [n][omega] (V) */
int qv_dequantize(int32_t n, int32_t omega, int32_t head_dim, int32_t bits, int32_t dtype,
                  int32_t per_token, const uint8_t* codes, const void* scale, const void* zp,
                  void* out, qv_stream_t stream);

/* ---- elementwise steps of the full-model decode driver --------------------
 * Not part of the reference's Sticky-KV path (its Llama layer uses HF
 * modules); fused so that a decode step launches fewer small kernels.
 * bf16, cols a multiple of 8, 16-byte aligned rows.
 * qv_add_rmsnorm: x[r] = bf16(x[r] + delta[r]) (skipped when delta is NULL),
 *                 h_out[r] = bf16(x[r] * rsqrt(mean(x[r]^2) + eps) * weight); cols <= 16384.
 * qv_silu_mul:    out[r] = bf16(bf16(SiLU(g)) * u) with g = gate_up[r][0:cols],
 *                 u = gate_up[r][cols:2*cols]. */
int qv_add_rmsnorm(int32_t rows, int32_t cols, void* x, const void* delta, const void* weight, float eps,
                   void* h_out, qv_stream_t stream);
int qv_silu_mul(int32_t rows, int32_t cols, const void* gate_up, void* out, qv_stream_t stream);
/* qv_gemv: y[r] = bf16(W . x[r]) for r < rows (1..8), W [n][k] bf16 row-major
 * (an nn.Linear weight), x [rows][k], y [rows][n]; fp32 accumulation; k a
 * multiple of 8, W and x 16-byte aligned.  The summation order is fixed, so
 * repeated calls give identical results.  Launched as a programmatic
 * dependent of the preceding kernel (its weight stream starts before that
 * kernel ends; x is read after it). */
int qv_gemv(int32_t rows, int32_t n, int32_t k, const void* w, const void* x, void* y, qv_stream_t stream);
/* qv_argmax: out[r] = the index of the largest bf16 value of x[r] (smallest
 * index among equal values), one launch.  The workspace
 * (qv_argmax_workspace_bytes) must be zero before the first call; each call
 * leaves it zero. */
size_t qv_argmax_workspace_bytes(int32_t rows);
int qv_argmax(int32_t rows, int32_t cols, const void* x, int64_t* out, void* workspace, size_t workspace_bytes,
              qv_stream_t stream);

/* ---- research token ledger (TrackingManager, kv_cache/tracking_manager.py:27-204)
 * One sequence per call.  ledger [max_context][2 + 2*heads] float32 rows of
 * (global id, layer id, physical position per head, cumulative importance per
 * head), history [max_context][heads] float32 (the reference's
 * _global_score_history), both -1 when fresh.  Positions index the
 * reference's physical cache order.  Bit-identical to the reference's float32
 * updates.
 * qv_track_prefill replaces TrackingManager.record_prefill (tracking_manager.py:61-124):
 *   importance [heads][kv_len] = attn_score_cache[0, :, :seq_len, :].sum(dim=1)
 *   as float32; survivors [heads][n_surv] = the kept physical indices in
 *   compressed order (eviction.py:225-229).
 * qv_track_decode replaces TrackingManager.record_decode (tracking_manager.py:126-160):
 *   scores [heads][kv_len] = attn_score_cache[0, :, 0, :] as float32; counter
 *   is the global token counter after this token's increment.
 * qv_track_positions replaces TrackingManager.update_physical_positions
 *   (tracking_manager.py:162-191): mapping [heads][seq_len] old -> new
 *   position (-1 = left the cache, cache.py:456-573), votes [heads][votes_stride]
 *   the vote ledger the cycle consumed. */
int qv_track_prefill(int32_t max_context, int32_t heads, int32_t seq_len, int32_t q_len, int32_t layer_idx,
                     int64_t global_start, int32_t num_new, const float* importance, int32_t kv_len,
                     const int64_t* survivors, int32_t n_surv, float* ledger, float* history, qv_stream_t stream);
int qv_track_decode(int32_t max_context, int32_t heads, int64_t counter, int64_t global_start, int32_t seq_len,
                    int32_t layer_idx, const float* scores, int32_t kv_len, float* ledger, float* history,
                    qv_stream_t stream);
int qv_track_positions(int32_t max_context, int32_t heads, int64_t counter, int32_t seq_len, const float* mapping,
                       const float* votes, int32_t votes_stride, float* ledger, float* history, qv_stream_t stream);

/* ---- diagnostics ------------------------------------------------------- */
int qv_read_error(const qv_layer* L, int32_t* host_err, qv_stream_t stream); /* synchronises the stream */
/* ---- one-shot sum across the GPUs of a node (KV-head tensor parallelism) ---
 * Not part of the reference, which runs one GPU: the all-reduce of the
 * row-parallel decode partials ([batch, hidden] bf16 per layer) when the
 * decoder is split by KV head over up to 8 GPUs of one node.  Each rank
 * allocates one buffer (create), publishes its CUDA IPC handle, maps every
 * other rank's buffer (open), then each call stores its vector into every
 * rank's buffer over NVLink as 8-byte words tagged with the call's epoch,
 * waits (bounded) until every rank's words of the epoch are in its own
 * buffer and sums the vectors in rank order in fp32, rounded once to bf16:
 * the same bits on every rank.  Every rank must make the same calls in
 * the same order on one stream each (the call is capturable like any kernel);
 * in and out may alias; n a multiple of 8, n*2 <= max_bytes, 16-byte aligned.
 * A wait that gives up sets QV_DERR_TIMEOUT (qv_peer_sum_read_error). */
#define QV_PEER_HANDLE_BYTES 64
typedef struct qv_peer_sum qv_peer_sum;
int qv_peer_sum_create(int32_t rank, int32_t world, size_t max_bytes, qv_peer_sum** out,
                       void* handle /* QV_PEER_HANDLE_BYTES, to publish */);
int qv_peer_sum_open(qv_peer_sum* ps, const void* handles /* world x QV_PEER_HANDLE_BYTES, rank order */);
int qv_peer_sum_bf16(qv_peer_sum* ps, const void* in, void* out, int64_t n, qv_stream_t stream);
/* The same hand-off for n int64 values, their maximum over the ranks (the
 * greedy token's packed (value, index) key); n*16 <= 2*max_bytes, 8-byte aligned. */
int qv_peer_max_i64(qv_peer_sum* ps, const int64_t* in, int64_t* out, int64_t n, qv_stream_t stream);
int qv_peer_sum_read_error(qv_peer_sum* ps, int32_t* host_err, qv_stream_t stream); /* synchronises */
int qv_peer_sum_destroy(qv_peer_sum* ps); /* after every rank's last call has completed */

const char* qv_last_cuda_error(void);
const char* qv_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QEVICT_B200_H */
