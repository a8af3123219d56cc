"""Research token ledger restated in numpy (test infrastructure only).

Mirrors ``TrackingManager`` (src/models/kv_cache/tracking_manager.py:27-223)
and ``get_ledger_data`` (src/models/kv_cache/ledger.py:16-44) for one
sequence: a [max_context, 2 + 2H] float32 table of (global id, layer id,
physical position per head, cumulative importance per head) and a
[max_context, H] float32 score history, both initialised to -1.

Every update is the reference's float32 arithmetic in the reference's order;
the inputs are numpy arrays in the shapes the reference's torch calls get.
"""

import numpy as np

from .numerics import f32, sum_round


class OracleTracker:
    """The research token ledger of TrackingManager (src/models/kv_cache/tracking_manager.py:27-204)."""

    def __init__(self, max_context, num_heads):
        """tracking_manager.py:30-41."""
        self.H = num_heads
        self.C = max_context
        self.reset()

    def reset(self):
        """tracking_manager.py:196-200."""
        self.counter = 0
        self.ledger = np.full((self.C, 2 + 2 * self.H), -1.0, np.float32)
        self.history = np.full((self.C, self.H), -1.0, np.float32)
        self.prefill_attention_matrix = None

    def increment(self, n=1):
        """tracking_manager.py:58-59."""
        self.counter += n

    def record_prefill(self, seq_len, q_len, layer_idx, attn_score_cache, survivor_ids, full_attn_scores,
                       global_start, num_new_tokens, attn_dt="fp32"):
        """tracking_manager.py:61-124.  attn_score_cache [1, H, q, kv] (values of
        dtype attn_dt, whose sum over q is rounded to it); survivor_ids [H, N]."""
        H, L, C = self.H, self.ledger, self.C
        for i in range(num_new_tokens):                                     # :77-83
            g = global_start + i
            if g < C:
                L[g, 0] = np.float32(g)
                L[g, 1] = np.float32(layer_idx)
                L[g, 2:2 + H] = np.float32(seq_len - q_len + i)
        imp = sum_round(f32(attn_score_cache[0, :, :seq_len, :]), 1, attn_dt)   # :85-86
        n_pre = min(seq_len, C)                                             # :87-101
        active = (L[:n_pre, 2:2 + H] >= 0).any(axis=1) & (L[:n_pre, 0] >= 0)
        g_act = np.nonzero(active)[0]
        if g_act.size:
            phys = L[g_act, 2].astype(np.int64)
            ok = (phys >= 0) & (phys < imp.shape[1])
            vg, vp = g_act[ok], phys[ok]
            if vg.size:
                s = imp[:, vp].T.astype(np.float32)
                L[vg, 2 + H:2 + 2 * H] = s
                self.history[vg, :] = s
        full = full_attn_scores if full_attn_scores is not None else attn_score_cache   # :103-105
        self.prefill_attention_matrix = np.array(full[0], copy=True)
        L[:, 2:2 + H] = -1.0                                                # :107-124
        for h in range(H):
            surv = np.asarray(survivor_ids[h], np.int64)
            g_ids = global_start + surv - (seq_len - num_new_tokens)
            ok = (g_ids >= 0) & (g_ids < C)
            if ok.any():
                vg = g_ids[ok]
                pos = np.arange(surv.shape[0], dtype=np.float32)
                L[vg, 2 + h] = pos[ok]
                vp = surv[ok]
                inr = vp < imp.shape[1]
                if inr.any():
                    L[vg[inr], 2 + H + h] = imp[h, vp[inr]]

    def record_decode(self, attn_score_cache, seq_len, layer_idx, global_start):
        """tracking_manager.py:126-160.  attn_score_cache [1, H, 1, kv]."""
        H, L, C = self.H, self.ledger, self.C
        g = global_start
        if g < C:
            L[g, 0] = np.float32(g)
            L[g, 1] = np.float32(layer_idx)
            L[g, 2:2 + H] = np.float32(seq_len - 1)
            L[g, 2 + H:2 + 2 * H] = 0.0
            self.history[g, :] = 0.0
        n_active = min(self.counter, C)
        if n_active <= 0:
            return
        live = np.nonzero((L[:n_active, 2:2 + H] >= 0).any(axis=1))[0]
        if live.size == 0:
            return
        phys = L[live, 2:2 + H].astype(np.int64)
        kv = attn_score_cache.shape[-1]
        inr = (phys >= 0) & (phys < kv)
        safe = np.clip(phys, 0, kv - 1)
        gen = attn_score_cache[0, :, 0, :]
        got = gen[np.arange(H)[None, :], safe].astype(np.float32) * inr.astype(np.float32)
        L[live, 2 + H:2 + 2 * H] = L[live, 2 + H:2 + 2 * H] + got
        self.history[live, :] = self.history[live, :] + got

    def update_physical_positions(self, mapping, seq_len, running_attention_votes):
        """tracking_manager.py:162-191.  mapping [H, seq_len] (old -> new, -1 evicted);
        running_attention_votes [H, >= seq_len]."""
        H, L = self.H, self.ledger
        n_active = min(self.counter, self.C)
        if n_active <= 0:
            return
        live = np.nonzero((L[:n_active, 2:2 + H] >= 0).any(axis=1))[0]
        if live.size == 0:
            return
        phys = L[live, 2:2 + H].astype(np.int64)
        valid = (phys >= 0) & (phys < seq_len)
        safe = np.clip(phys, 0, seq_len - 1)
        hh = np.arange(H)[None, :]
        new = mapping[hh, safe].astype(np.float32)
        new = np.where(valid, new, np.float32(-1.0)).astype(np.float32)
        evicted = (new < 0) & valid
        add = running_attention_votes[hh, safe].astype(np.float32) * evicted.astype(np.float32)
        L[live, 2 + H:2 + 2 * H] = L[live, 2 + H:2 + 2 * H] + add
        self.history[live, :] = self.history[live, :] + add
        L[live, 2:2 + H] = new

    def get_ledger_data(self):
        """ledger.py:16-44."""
        a = self.ledger[:self.counter]
        return {"global_id": a[:, 0].astype(np.int64), "layer_id": a[:, 1].astype(np.int64),
                "physical_id": a[:, 2:2 + self.H].astype(np.int64),
                "attention_score": a[:, 2 + self.H:2 + 2 * self.H]}


# -- the cache object's calls into the ledger -----------------------------------------
def tracked_prefill(st, tr, K, V, attn, attn_dt, layer_idx):
    """Prefill of an OracleStickyLayer with its ledger: counter reset and advance
    (cache.py:251-257), the prefill (cache.py:269-345), record_prefill
    (cache.py:346-351).  attn [H, q, S]."""
    S = K.shape[1]
    tr.counter = 0
    tr.increment(S)
    Kn, Vn = st.prefill(K, V, attn, attn_dt)
    if st.lid is None:          # full-cache bypass returns before the ledger (cache.py:302-304)
        return Kn, Vn
    tr.record_prefill(S, S, layer_idx, attn[None], st.last_survivors, None, 0, S, attn_dt)
    return Kn, Vn


def tracked_decode(st, tr, K, V, scores, q_scores, score_dt, layer_idx):
    """One decode token with the ledger: counter (cache.py:258-260), tally and
    record_decode (cache.py:366-373), the cycle and update_physical_positions
    (cache.py:378-424).  K, V [H, S, D] with the new token; scores [H, S]."""
    gs = tr.counter
    tr.increment(1)
    if st.lid is None:
        return K, V
    S = K.shape[1]
    due = st.tally(K, scores, q_scores, score_dt)
    tr.record_decode(f32(scores)[None, :, None, :], S, layer_idx, gs)
    if not due:
        return K, V
    K2, V2 = st.cycle(K, V)
    if st.r_ratio != 100:
        tr.update_physical_positions(st.last_mapping, S, st.last_cycle_votes)
    return K2, V2
