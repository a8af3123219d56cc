"""Per-layer Sticky-KV state machine restated in numpy (test infrastructure only).

One sequence (the reference is batch-1), all KV heads of one layer, in the
reference's own physical layout.  Mirrors, function by function:

  STICKYKVCache_LayerWise.__call__            src/models/kv_cache/cache.py:234-427
  STICKYKVCache_LayerWise._build_physical_cache   cache.py:433-575 (with its
                                              old -> new position mapping)
  EvictionManager.tally_prefill_scores        src/models/kv_cache/eviction_manager.py:115-173
  EvictionManager.commit_prefill_result       eviction_manager.py:184-192
  EvictionManager.tally_decode_scores         eviction_manager.py:198-203
  EvictionManager.run_decode_cycle            eviction_manager.py:205-383
  EvictionManager.commit_decode_result        eviction_manager.py:385-396
  EvictionManager.update_local_history        eviction_manager.py:398-412
  EvictionManager.reset_decode_counters       eviction_manager.py:414-417
  evict_from_window_scores                    src/models/kv_cache/eviction.py:102-156
  create_mask_and_evict_from_kv_cache_prompt_stage   eviction.py:163-240
  find_logical_window_span                    eviction.py:26-60
  QuantizationManager.store_windows / accumulate_scores / get_promoted_windows / rebuild
                                              src/models/kv_cache/quantize_manager.py:91-327

Deliberate, documented difference: ``torch.topk`` on CPU returns tied values
in an order that depends on its quickselect; here (and in the CUDA kernels)
ties are broken by candidate index, lowest first.  On inputs without ties the
selected sets and their order are identical to the reference's.

``window_sum`` selects the fp32 summation order of the per-window scoreboard:
"sequential" follows the reference's scatter_add, "tree" follows the CUDA
kernel's warp reduction (see ``numerics.tree_sum32``) so that both sides see
bit-identical window scores when they consume the same vote ledger.
"""

import math

import numpy as np

from .codec import (
    dequantize_from_quant,
    quantize_k_per_window,
    quantize_v_per_window,
    requantize_with_meta,
)
from .numerics import f32, rnd, sum_round, tree_sum32

NEG_INF = np.float32(-np.inf)


def topk_desc(scores, k):
    """Row-wise top-k, values descending, ties broken by lower index (see module doc):
    the torch.topk(..., largest=True) of eviction_manager.py:329,343 and
    eviction.py:132,147, whose order among equal scores torch leaves unspecified."""
    scores = f32(scores)
    order = np.argsort(-scores.astype(np.float64), axis=1, kind="stable")[:, :k]
    return np.take_along_axis(scores, order, axis=1), order


def compute_budget(total_cache_ratio, sink_tokens, use_fixed_local_tokens, local_num_tokens,
                   local_cache_ratio, q_ratio, quant_bit_width, head_dim, omega, new_tokens,
                   max_tokens):
    """CFO budget carve (src/models/kv_cache/allocator.py:24-107)."""
    total = (new_tokens + max_tokens) * total_cache_ratio // 100
    remaining = max(0, total - sink_tokens)
    target_local = local_num_tokens if use_fixed_local_tokens else (total * local_cache_ratio) // 100
    local_num = min(target_local, remaining)
    remaining = max(0, remaining - local_num)
    bf16_bytes = 2 * head_dim
    quant_bytes = head_dim if quant_bit_width == 8 else head_dim / 2.0
    ratio = bf16_bytes / quant_bytes
    bf16_target = (remaining * (100 - q_ratio)) // 100
    q_mem_target = remaining - bf16_target
    q_target = int(q_mem_target * ratio)
    k_windows = -(-bf16_target // omega)
    q_windows = -(-q_target // omega)
    q_num = int((q_windows * omega) / ratio)
    return dict(local_num=local_num, k_windows=k_windows, q_windows_count=q_windows, q_num=q_num,
                quant_bytes_len=head_dim if quant_bit_width == 8 else head_dim // 2)


def find_logical_window_span(lid, omega, h, wid, seq_len):
    """src/models/kv_cache/eviction.py:26-60."""
    pos = np.nonzero(lid[h] == int(wid))[0]
    if pos.size == 0:
        return None
    start, end = int(pos.min()), int(pos.max()) + 1
    if pos.size != end - start or not np.array_equal(pos, np.arange(start, end)):
        raise RuntimeError(f"Logical window {wid} has non-contiguous physical positions")
    if end - start != omega:
        return None
    if end > seq_len:
        return None
    return start, end


class OracleStickyLayer:
    """Reference-layout Sticky-KV state of one layer for one sequence: the state that
    STICKYKVCache_LayerWise (src/models/kv_cache/cache.py:41-427) keeps through its
    eviction and quantization managers (eviction_manager.py, quantize_manager.py)."""

    def __init__(self, num_heads, head_dim, omega, sink, local_num, k_windows, q_windows,
                 dtype, bit_width=8, max_windows=100, max_context=None, r_ratio=20,
                 window_sum="sequential"):
        self.H, self.D, self.omega, self.sink = num_heads, head_dim, omega, sink
        self.local_num, self.k_windows, self.q_windows = local_num, k_windows, q_windows
        self.dt, self.bits, self.maxW = dtype, bit_width, max_windows
        self.maxCtx = max_context if max_context is not None else sink + omega * max_windows + 1024
        self.r_ratio = r_ratio
        self.window_sum = window_sum
        self.qbl = head_dim if bit_width == 8 else head_dim // 2
        self.reset()

    # -- state -----------------------------------------------------------------
    def reset(self):
        """cache.py:581-597 / eviction_manager.py:423-433 / quantize_manager.py:335-341."""
        H = self.H
        self.window_scores = np.full((H, self.maxW, 3), np.nan, np.float32)
        self.votes = np.zeros((H, self.maxCtx), np.float32)
        self.local_history = np.zeros((H, self.maxW), np.float32)
        self.lid = None
        self.tokens_since = 0
        self.n_tokens = 0
        self.gen_step = 0
        self.dyn_local = 0
        self.global_counter = 0
        self.prefill_done = False
        self.q = None  # dict(kq, ks, kz, vq, vs, vz, ids, scores)
        self.meta = {}  # (wid, h) -> (ks, kz, vs, vz)
        self.oob_sticky_drops = 0
        self.oob_qcache_b_drops = 0
        self.oob_qcache_c_drops = 0
        # how many (head, window) entries each Q-cache rebuild path produced
        # (quantize_manager.py:168-182 A, :243-268 B, :273-318 C; "_zero": the
        # window was not found in the old cache and was filled with zeros)
        self.path_counts = dict(A=0, B=0, B_zero=0, C=0, C_zero=0)
        self.last_result = None
        self.last_survivors = None    # prefill survivor positions [H, N] (eviction.py:225-229)
        self.last_mapping = None      # last cycle's old -> new positions [H, S]
        self.last_cycle_votes = None  # the vote ledger the last cycle consumed [H, S]

    def window_to_token(self, ids):
        """Token indices of windows ids: sink + id*omega + [0, omega) (eviction.py:26-60)."""
        return self.sink + np.asarray(ids, np.int64)[..., None] * self.omega + np.arange(self.omega)

    # -- prefill -----------------------------------------------------------------
    def tally_prefill_scores(self, attn, seq_len, attn_dt):
        """eviction_manager.py:115-173; attn [H, Qrows, S] holds scores in attn_dt."""
        sink, om, H = self.sink, self.omega, self.H
        score_end = max(sink, seq_len - self.local_num)
        nw = max(0, (score_end - sink) // om)
        score_end = min(sink + nw * om, attn.shape[2])
        nw = (score_end - sink) // om
        score_end = sink + nw * om
        self.dyn_local = self.local_num
        wsum = self._prefill_window_sums
        if nw > 0:
            obs = sum_round(attn[:, :seq_len, sink:score_end], 1, attn_dt)
            win = wsum(obs.reshape(H, nw, om), attn_dt)
            idx = np.arange(nw, dtype=np.float32)
            self.window_scores[:, :nw, 0] = win
            self.window_scores[:, :nw, 1] = idx
            self.window_scores[:, :nw, 2] = idx
        tpw = max(0, (seq_len - sink) // om)
        if tpw > 0:
            afr = min(sink + tpw * om, attn.shape[2])
            tpw = (afr - sink) // om
            afr = sink + tpw * om
            if tpw > 0:
                full = sum_round(attn[:, :seq_len, sink:afr], 1, attn_dt)
                self.local_history[:, :tpw] = wsum(full.reshape(H, tpw, om), attn_dt)
        return score_end

    def _prefill_window_sums(self, x, attn_dt):
        """``.view(H, nw, omega).sum(dim=2)`` in the scores' dtype (eviction_manager.py:141-143)."""
        if self.window_sum == "tree":
            return rnd(tree_sum32(x), attn_dt)
        return f32(sum_round(x, 2, attn_dt))

    def evict_from_window_scores(self):
        """eviction.py:102-156 (mutates window_scores, returns top-q losers)."""
        ws = self.window_scores
        valid = ~np.isnan(ws[:, :, 1])
        scores = np.where(valid, ws[:, :, 0], NEG_INF).astype(np.float32)
        ids, orig = ws[:, :, 1].copy(), ws[:, :, 2].copy()
        nvalid = int(valid.sum(axis=1).min())
        curr_k = min(self.k_windows, nvalid)
        top_v, top_i = topk_desc(scores, curr_k)
        kept_ids = np.take_along_axis(ids, top_i, 1)
        kept_orig = np.take_along_axis(orig, top_i, 1)
        q_ids = q_scores = None
        if self.q_windows > 0:
            nl = nvalid - curr_k
            if nl > 0:
                ls = scores.copy()
                np.put_along_axis(ls, top_i, NEG_INF, 1)
                qc = min(self.q_windows, nl)
                qv, qi = topk_desc(ls, qc)
                q_ids = np.take_along_axis(ids, qi, 1)
                q_scores = qv
        srt = np.argsort(kept_ids, axis=1, kind="stable")
        ws[:] = np.nan
        ws[:, :curr_k, 0] = np.take_along_axis(top_v, srt, 1)
        ws[:, :curr_k, 1] = np.take_along_axis(kept_ids, srt, 1)
        ws[:, :curr_k, 2] = np.take_along_axis(kept_orig, srt, 1)
        return q_ids, q_scores

    def store_windows(self, kd, vd, ids, scores):
        """quantize_manager.py:91-98."""
        kq, ks, kz = quantize_k_per_window(kd, self.dt, self.bits)
        vq, vs, vz = quantize_v_per_window(vd, self.dt, self.bits)
        self.q = dict(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz,
                      ids=f32(ids), scores=f32(scores))

    def prefill(self, K, V, attn, attn_dt):
        """cache.py:269-355.  K, V [H, S, D]; attn [H, Qrows, S].  Returns (K', V')."""
        S = K.shape[1]
        self.global_counter = S
        if self.r_ratio >= 100 and self.q_windows == 0:
            self.prefill_done = True
            return K, V
        self.n_tokens += S
        score_end = self.tally_prefill_scores(attn, S, attn_dt)
        q_ids, q_scores = self.evict_from_window_scores()
        if q_ids is not None:
            qc = q_ids.shape[1]
            phys = np.clip(self.window_to_token(q_ids.astype(np.int64)).reshape(self.H, -1), 0, S - 1)
            hh = np.arange(self.H)[:, None]
            kd = K[hh, phys].reshape(self.H, qc, self.omega, self.D)
            vd = V[hh, phys].reshape(self.H, qc, self.omega, self.D)
            self.store_windows(kd, vd, q_ids, q_scores)
        # create_mask_and_evict_from_kv_cache_prompt_stage (eviction.py:163-240)
        H = self.H
        sinks = np.broadcast_to(np.arange(self.sink), (H, self.sink))
        raw_w = self.window_scores[:, :self.k_windows, 1]
        valid_k = int((~np.isnan(raw_w)).all(axis=0).sum())
        if valid_k > 0:
            sticky = self.window_scores[:, :valid_k, 1].astype(np.int64)
            wt = self.window_to_token(sticky).reshape(H, -1)
        else:
            wt = np.zeros((H, 0), np.int64)
        parts = [sinks, wt]
        if score_end < S:
            parts.append(np.broadcast_to(np.arange(score_end, S), (H, S - score_end)))
        allidx = np.clip(np.concatenate(parts, axis=1), 0, S - 1)
        surv = np.sort(allidx, axis=1)
        self.last_survivors = surv
        hh = np.arange(H)[:, None]
        Kn, Vn = K[hh, surv], V[hh, surv]
        # commit_prefill_result (eviction_manager.py:184-192)
        self.lid = np.where(surv >= self.sink, (surv - self.sink) // self.omega, -1).astype(np.int64)
        self.prefill_done = True
        return Kn, Vn

    # -- decode ------------------------------------------------------------------
    def _window_sums(self, votes_c, lid, n_new_votes, new_lids):
        """Scoreboard [H, maxW] (eviction_manager.py:229-255)."""
        H, maxW = self.H, self.maxW
        sb = np.zeros((H, maxW), np.float32)
        if self.window_sum == "sequential":
            for h in range(H):
                for p in range(lid.shape[1]):
                    w = lid[h, p]
                    if w >= 0:
                        sb[h, w] = np.float32(sb[h, w] + votes_c[h, p])
                    else:
                        sb[h, 0] = np.float32(sb[h, 0] + np.float32(0.0))
                for j, w in enumerate(new_lids):
                    if 0 <= w < maxW:
                        sb[h, w] = np.float32(sb[h, w] + n_new_votes[h, j])
            return sb
        # "tree": gather each window's tokens in position order and reduce like the kernel
        for h in range(H):
            buckets = {}
            for p in range(lid.shape[1]):
                w = lid[h, p]
                if w >= 0:
                    buckets.setdefault(int(w), []).append(votes_c[h, p])
            for j, w in enumerate(new_lids):
                if 0 <= w < maxW:
                    buckets.setdefault(int(w), []).append(n_new_votes[h, j])
            for w, vals in buckets.items():
                vals = f32(vals)
                if vals.size == self.omega:
                    sb[h, w] = tree_sum32(vals)
                else:
                    acc = np.float32(0)
                    for v in vals:
                        acc = np.float32(acc + v)
                    sb[h, w] = acc
        return sb

    def run_decode_cycle(self, seq_len):
        """eviction_manager.py:205-383.  Returns a dict mirroring DecodeEvictionResult."""
        H, om, sink = self.H, self.omega, self.sink
        lid = self.lid
        clen = lid.shape[1]
        votes_c = self.votes[:, :clen]
        new_lids, new_votes = [], None
        if seq_len > clen:
            n_new = seq_len - clen
            js = np.arange(n_new)
            new_lids = ((self.n_tokens - om + js - sink) // om).tolist()
            new_votes = self.votes[:, clen:seq_len]
        sb = self._window_sums(votes_c, lid, new_votes, new_lids)

        ws = self.window_scores
        valid_mask = ~np.isnan(ws[:, :, 1])
        vo = min(self.k_windows, int(valid_mask.sum(axis=1).min()))
        raw_ids = ws[:, :vo, 1]
        raw_scores = ws[:, :vo, 0]
        is_valid = ~np.isnan(raw_ids)
        old_ids = np.nan_to_num(raw_ids, nan=0.0).astype(np.float32)
        safe = old_ids.astype(np.int64)
        hist = np.nan_to_num(raw_scores, nan=0.0).astype(np.float32)
        if vo > 0:
            gen = np.take_along_axis(sb, safe, 1)
            gen = np.where(is_valid, gen, 0.0).astype(np.float32)
        else:
            gen = np.zeros_like(hist)
        old_scores = (hist + gen).astype(np.float32)

        raw_last = (self.n_tokens - sink - self.dyn_local) // om - 1
        raw_last = min(raw_last, self.maxW - 1)
        has = raw_last >= 0
        last = raw_last
        if has:
            already = (old_ids.astype(np.int64) == last).any(axis=1)
            gen_new = sb[:, last].copy()
            last_hist = self.local_history[:, last].copy()
            self.local_history[:, last] = np.where(already, self.local_history[:, last], 0.0)
            tot = (gen_new + last_hist).astype(np.float32)
            tot = np.where(already, NEG_INF, tot).astype(np.float32)
            cids = np.concatenate([old_ids, np.full((H, 1), float(last), np.float32)], axis=1)
            csc = np.concatenate([old_scores, tot[:, None]], axis=1)
        else:
            cids, csc = old_ids, old_scores
        if self.q_windows > 0 and self.q is not None:
            cids = np.concatenate([cids, self.q["ids"]], axis=1)
            csc = np.concatenate([csc, self.q["scores"]], axis=1)

        curr_k = min(self.k_windows, csc.shape[1])
        top_v, top_i = topk_desc(csc, curr_k)
        surv = np.take_along_axis(cids, top_i, 1)
        srt = np.argsort(surv, axis=1, kind="stable")
        final_v = np.take_along_axis(top_v, srt, 1)
        final_ids = np.take_along_axis(surv, srt, 1)

        l_ids = l_scores = None
        if self.q_windows > 0:
            ls = csc.copy()
            np.put_along_axis(ls, top_i, NEG_INF, 1)
            nrem = int((ls > NEG_INF).sum(axis=1).min())
            if nrem > 0:
                qc = min(self.q_windows, nrem)
                qv, qi = topk_desc(ls, qc)
                l_ids = np.take_along_axis(cids, qi, 1)
                l_scores = qv

        local_windows = (self.dyn_local + om - 1) // om
        if has:
            local_id_start = last + 1
        else:
            local_id_start = max(0, (self.n_tokens - sink - self.dyn_local) // om)
        nob = max(0, (clen - sink - self.dyn_local) // om)
        if nob > 0:
            pbw = lid[:, sink + np.arange(nob) * om]
        else:
            pbw = np.zeros((H, 0), np.int64)
        return dict(winner_ids=final_ids, winner_scores=final_v, curr_k=curr_k,
                    loser_ids=l_ids, loser_scores=l_scores, scoreboard=sb,
                    pre_num_old_blocks=nob, pre_block_wids=pbw,
                    local_id_start=local_id_start, local_windows=local_windows,
                    challenger=last if has else None)

    def update_local_history(self, res):
        """eviction_manager.py:398-412."""
        if res["local_windows"] <= 0:
            return
        ids = np.arange(res["local_id_start"], res["local_id_start"] + res["local_windows"])
        ids = ids[(ids >= 0) & (ids < self.maxW)]
        if ids.size:
            self.local_history[:, ids] = (self.local_history[:, ids] + res["scoreboard"][:, ids]).astype(np.float32)

    def get_promoted_windows(self, winner_ids):
        """quantize_manager.py:114-145.  Returns {(h, wid): (k [w,D], v [w,D])}."""
        out = {}
        if self.q is None:
            return out
        qids = self.q["ids"].astype(np.int64)
        win = winner_ids.astype(np.int64)
        mask = (qids[:, :, None] == win[:, None, :]).any(axis=2)
        if mask.any():
            kd = dequantize_from_quant(self.q["kq"], self.q["ks"], self.q["kz"], self.dt, self.bits)
            vd = dequantize_from_quant(self.q["vq"], self.q["vs"], self.q["vz"], self.dt, self.bits)
            for h, i in zip(*np.nonzero(mask)):
                wid = int(qids[h, i])
                out[(int(h), wid)] = (kd[h, i], vd[h, i])
                self.meta[(wid, int(h))] = (self.q["ks"][h, i].copy(), self.q["kz"][h, i].copy(),
                                            self.q["vs"][h, i].copy(), self.q["vz"][h, i].copy())
        return out

    def rebuild(self, l_ids, l_scores, K, V, pbw, seq_len):
        """quantize_manager.py:148-327 (paths A, B, C)."""
        if l_ids is None:
            self.q = None
            return
        H, om, D, dt = self.H, self.omega, self.D, self.dt
        qc = l_ids.shape[1]
        nkq = np.zeros((H, qc, om, self.qbl), np.uint8)
        nvq = np.zeros((H, qc, om, self.qbl), np.uint8)
        nks = np.zeros((H, qc, 1, D), np.float32)
        nkz = np.zeros((H, qc, 1, D), np.float32)
        nvs = np.zeros((H, qc, om, 1), np.float32)
        nvz = np.zeros((H, qc, om, 1), np.float32)
        if self.q is not None:
            match = l_ids[:, :, None] == self.q["ids"][:, None, :]
            ret = match.any(axis=2)
            old_idx = match.astype(np.uint8).argmax(axis=2)
            for h, j in zip(*np.nonzero(ret)):
                i = old_idx[h, j]
                self.path_counts["A"] += 1
                for dst, src in ((nkq, "kq"), (nvq, "vq"), (nks, "ks"), (nkz, "kz"), (nvs, "vs"), (nvz, "vz")):
                    dst[h, j] = self.q[src][h, i]
        else:
            ret = np.zeros((H, qc), bool)
        nr_h, nr_qi = np.nonzero(~ret)
        if nr_h.size:
            nr_w = l_ids[nr_h, nr_qi].astype(np.int64)
            nob = pbw.shape[1]
            if nob > 0:
                m = pbw[nr_h] == nr_w[:, None]
                found = m.any(axis=1)
                slot = m.astype(np.uint8).argmax(axis=1)
                phys = self.sink + slot * om
                oob = found & (phys + om > seq_len)
                if oob.any():
                    self.oob_qcache_b_drops += int(oob.sum())
                    found = found & ~oob
            else:
                found = np.zeros(nr_h.size, bool)
                phys = np.zeros(nr_h.size, np.int64)
            for n in range(nr_h.size):
                h, j, wid = int(nr_h[n]), int(nr_qi[n]), int(nr_w[n])
                if (wid, h) in self.meta:  # path C
                    if found[n]:
                        ps = int(phys[n])
                        if ps + om > seq_len:
                            self.oob_qcache_c_drops += 1
                            continue
                        kf, vf = K[h, ps:ps + om], V[h, ps:ps + om]
                    else:
                        kf = np.zeros((om, D), np.float32)
                        vf = np.zeros((om, D), np.float32)
                        self.path_counts["C_zero"] += 1
                    self.path_counts["C"] += 1
                    ks, kz, vs, vz = self.meta[(wid, h)]
                    nkq[h, j] = requantize_with_meta(kf[None], ks, kz, dt, self.bits)[0]
                    nvq[h, j] = requantize_with_meta(vf, vs, vz, dt, self.bits)
                    nks[h, j, 0], nkz[h, j, 0] = ks[0], kz[0]
                    nvs[h, j], nvz[h, j] = vs, vz
                else:  # path B
                    pos = np.clip(phys[n] + np.arange(om), 0, seq_len - 1)
                    kd = K[h, pos].copy()
                    vd = V[h, pos].copy()
                    self.path_counts["B"] += 1
                    if not found[n]:
                        kd[:] = 0
                        vd[:] = 0
                        self.path_counts["B_zero"] += 1
                    kq, ks, kz = quantize_k_per_window(kd[None], dt, self.bits)
                    vq, vs, vz = quantize_v_per_window(vd[None], dt, self.bits)
                    nkq[h, j], nks[h, j], nkz[h, j] = kq[0], ks[0], kz[0]
                    nvq[h, j], nvs[h, j], nvz[h, j] = vq[0], vs[0], vz[0]
        self.q = dict(kq=nkq, ks=nks, kz=nkz, vq=nvq, vs=nvs, vz=nvz,
                      ids=f32(l_ids), scores=f32(l_scores))

    def build_physical_cache(self, K, V, res, promoted):
        """cache.py:433-575."""
        H, om, sink, D = self.H, self.omega, self.sink, self.D
        ck = res["curr_k"]
        fid = res["winner_ids"]
        S = K.shape[1]
        new_len = sink + ck * om + self.dyn_local
        nk = np.zeros((H, new_len, D), np.float32)
        nv = np.zeros((H, new_len, D), np.float32)
        nl = np.full((H, new_len), -1, np.int64)
        nob = res["pre_num_old_blocks"]
        if nob > 0:
            m = res["pre_block_wids"][:, None, :] == fid[:, :, None]
            found = m.any(axis=2)
            slot = m.astype(np.uint8).argmax(axis=2)
            first = sink + slot * om
            oob = found & (first + om > S)
            if oob.any():
                self.oob_sticky_drops += int(oob.sum())
                found = found & ~oob
        else:
            found = np.zeros((H, ck), bool)
            first = np.zeros((H, ck), np.int64)
        # mapping: old physical position -> new one, -1 when the token left the
        # main zone (the token-ledger input, cache.py:456,509-510,527-528,542-557,570-573)
        mp = np.full((H, S), -1.0, np.float32)
        nk[:, :sink] = K[:, :sink]
        nv[:, :sink] = V[:, :sink]
        nl[:, :sink] = self.lid[:, :sink]
        mp[:, :sink] = np.arange(sink, dtype=np.float32)[None, :]
        ar = np.arange(om, dtype=np.float32)
        for h in range(H):
            for i in range(ck):
                npos = sink + i * om
                wid = int(fid[h, i])
                if found[h, i]:
                    fp = int(first[h, i])
                    nk[h, npos:npos + om] = K[h, fp:fp + om]
                    nv[h, npos:npos + om] = V[h, fp:fp + om]
                    nl[h, npos:npos + om] = wid
                    mp[h, fp:fp + om] = npos + ar
                    continue
                if (h, wid) in promoted:
                    pk, pv = promoted[(h, wid)]
                    nk[h, npos:npos + om] = pk
                    nv[h, npos:npos + om] = pv
                    nl[h, npos:npos + om] = wid
                    span = find_logical_window_span(self.lid, om, h, wid, S)
                    if span is not None:
                        mp[h, span[0]:span[1]] = npos + ar
                else:
                    span = find_logical_window_span(self.lid, om, h, wid, S)
                    if span is not None:
                        s0, e0 = span
                        nk[h, npos:npos + om] = K[h, s0:e0]
                        nv[h, npos:npos + om] = V[h, s0:e0]
                        mp[h, s0:e0] = npos + ar
                    nl[h, npos:npos + om] = wid
        if self.dyn_local > 0:
            ols = S - self.dyn_local
            nls = sink + ck * om
            act = min(self.dyn_local, S - ols)
            nk[:, nls:nls + act] = K[:, ols:ols + act]
            nv[:, nls:nls + act] = V[:, ols:ols + act]
            lsw = max(0, (self.n_tokens - sink - self.dyn_local) // om)
            nl[:, nls:nls + act] = (lsw + np.arange(self.dyn_local) // om)[:act][None, :]
            mp[:, ols:ols + act] = (nls + np.arange(act, dtype=np.float32))[None, :]
        self.last_mapping = mp
        return nk, nv, nl

    def decode(self, K, V, scores, q_scores, score_dt):
        """cache.py:357-427 for one decode token.

        K, V   [H, S, D] physical cache including the new token (reference order)
        scores [H, S] group-mean main-zone probabilities (values in score_dt)
        q_scores [H, W*omega] or None
        Returns (K', V') -- the same arrays, or the rebuilt cache on cycle steps.
        """
        if not self.tally(K, scores, q_scores, score_dt):
            return K, V
        return self.cycle(K, V)

    def tally(self, K, scores, q_scores, score_dt):
        """Counters + ledger accumulation of one decode token (cache.py:357-376,
        eviction_manager.py:198-203, quantize_manager.py:101-111).
        Returns True when an eviction cycle is due."""
        self.global_counter += 1
        S = K.shape[1]
        if self.lid is None:
            return False
        self.n_tokens += 1
        self.gen_step += 1
        self.votes[:, :S] = (self.votes[:, :S] + f32(scores)[:, :S]).astype(np.float32)
        self.tokens_since += 1
        if q_scores is not None and self.q is not None:
            qc = self.q["ids"].shape[1]
            tot = qc * self.omega
            if q_scores.shape[1] >= tot:
                per_w = sum_round(f32(q_scores)[:, :tot].reshape(self.H, qc, self.omega), 2, score_dt)
                self.q["scores"] = (self.q["scores"] + f32(per_w)).astype(np.float32)
        return self.tokens_since == self.omega

    def cycle(self, K, V):
        """The eviction cycle of cache.py:378-427 on the current ledger."""
        S = K.shape[1]
        res = self.run_decode_cycle(S)
        self.last_result = res
        self.update_local_history(res)
        ck = res["curr_k"]
        if self.r_ratio == 100:
            self.window_scores[:] = np.nan
            self.window_scores[:, :ck, 0] = res["winner_scores"]
            self.window_scores[:, :ck, 1] = res["winner_ids"]
            self.window_scores[:, :ck, 2] = res["winner_ids"]
            self.votes[:, :S] = 0
            self.tokens_since = 0
            return K, V
        promoted = self.get_promoted_windows(res["winner_ids"])
        self.rebuild(res["loser_ids"], res["loser_scores"], K, V, res["pre_block_wids"], S)
        nk, nv, nl = self.build_physical_cache(K, V, res, promoted)
        self.last_cycle_votes = self.votes[:, :S].copy()   # what the token ledger sees (cache.py:422-424)
        self.window_scores[:] = np.nan
        self.window_scores[:, :ck, 0] = res["winner_scores"]
        self.window_scores[:, :ck, 1] = res["winner_ids"]
        self.window_scores[:, :ck, 2] = res["winner_ids"]
        self.lid = nl
        self.votes[:, :S] = 0
        self.tokens_since = 0
        return nk, nv

    # -- views -------------------------------------------------------------------
    def q_tensors(self):
        """Q-cache tensors in reference shapes, or None."""
        return self.q

    def sticky_ids(self):
        """(ids, scores) of the tracked sticky windows, ascending id: the non-NaN rows of
        window_scores (eviction_manager.py:385-396 writes them id-sorted)."""
        ws = self.window_scores
        n = int((~np.isnan(ws[0, :, 1])).sum())
        return ws[:, :n, 1].astype(np.int64), ws[:, :n, 0].copy()


def rope_cos_sin(positions, head_dim, theta, dt, inv_freq_dt="fp32"):
    """HF default RoPE tables (transformers LlamaRotaryEmbedding, used by the
    reference through HFRopeWrapper, src/models/attention/rope.py:154-183).

    ``inv_freq_dt``: the dtype the module's ``inv_freq`` buffer was cast to
    (``module.to(bfloat16)`` casts it, and the cos/sin tables inherit that).
    """
    inv = (np.float32(1.0) / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)))).astype(np.float32)
    inv = rnd(inv, inv_freq_dt)
    fr = (np.asarray(positions, np.float32)[:, None] * inv[None, :]).astype(np.float32)
    emb = np.concatenate([fr, fr], axis=-1)
    return rnd(np.cos(emb), dt), rnd(np.sin(emb), dt)


def apply_rope(x, cos, sin, dt):
    """(x * cos) + (rotate_half(x) * sin) in the KV dtype (src/models/kv_cache/helpers.py:56-62).

    x [..., S, D] with cos/sin [S, D].
    """
    half = x.shape[-1] // 2
    rh = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = rnd(f32(x) * cos, dt)
    b = rnd(f32(rh) * sin, dt)
    return rnd(a + b, dt)


def sdpa_scale(head_dim):
    """sqrt(head_dim) as the float32 the logits are divided by (ops.py:40,45,123,126)."""
    return np.float32(math.sqrt(head_dim))
