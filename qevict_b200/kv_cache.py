"""The reference's cache API, ``STICKYKVCache_LayerWise``, over the device state.

Same constructor, call signature, properties and static codec methods as
``STICKYKVCache_LayerWise`` (src/models/kv_cache/cache.py:41-427), so code
written against the reference's cache object keeps working:

  * ``cache(past_key_values, attn_score_cache, full_attn_scores=None, q_len=None,
    q_attn_scores=None) -> (K, V)``.  At prefill, ``past_key_values`` is the
    rotated prompt K/V and ``attn_score_cache`` its per-key column scores; the
    budget comes from ``compute_budget`` and the prompt is split into sinks,
    sticky windows, Q-cache windows and the local zone on the device
    (``qv_prefill_build``).  At decode, ``past_key_values`` is the returned
    physical cache with the new token appended and ``attn_score_cache`` /
    ``q_attn_scores`` are the step's group-mean probabilities over it and over
    the Q-cache; they are folded into the ledger and, every OMEGA tokens, the
    eviction cycle runs (``qv_evict_cycle``).  The returned (K, V) is the
    physical cache in the reference's order: sinks, sticky windows by
    ascending id, then the local zone and the tokens appended since.
  * the ``q_cache_*`` / ``window_scores`` / ``global_token_counter`` properties
    present the device state in the reference's shapes and order.
  * with ``sticky_config.tracking_flag == 1`` the research token ledger
    (``qevict_b200.tracking.TrackingManager``, one per sequence) is kept on the
    device exactly as the reference's cache drives it (cache.py:251-260,
    346-351, 371-373, 414-424); ``token_ledger``, ``global_score_history``,
    ``prefill_attention_matrix`` and ``get_ledger_data()`` expose it.  The
    old -> new position mapping of a cycle comes from the token each physical
    position holds before and after the cycle.

This caller-computes-attention path exists for compatibility; the fused path,
where the attention kernel computes and folds the probabilities itself, is
``qevict_b200.attention.STICKYLlamaAttention``, which drives the same state.

Batch: the reference keeps one sequence per cache object; this class takes the
batch from the prompt's first dimension and keeps all sequences in lockstep.
Properties then carry a leading batch dimension when B > 1.
"""

import math

import torch

from . import _native as N
from . import codec as _codec
from . import sticky_config
from .allocator import compute_budget
from .layer_state import StickyLayerState, kv_dtype_code
from .tracking import NoOpTrackingManager, TrackingManager


class STICKYKVCache_LayerWise:
    """Sticky-KV cache of one attention layer (window ledger, sticky windows, Q-cache)."""

    def __init__(self, p_ratio, r_ratio, start_idx, num_heads, layer_idx, config=None, k_seq_dim=2, v_seq_dim=2):
        if k_seq_dim != 2 or v_seq_dim != 2:
            raise N.QevictError("only [B, H, S, D] key/value layouts (seq dim 2) are supported")
        self.total_cache_ratio = r_ratio
        self.local_cache_ratio = getattr(sticky_config, "P_RATIO", p_ratio)
        self.start_idx = start_idx
        self.k_seq_dim, self.v_seq_dim = k_seq_dim, v_seq_dim
        self.layer_idx = layer_idx
        self.num_heads = num_heads
        self.omega = sticky_config.OMEGA
        self.sink_tokens = sticky_config.SINK_TOKENS
        self.q_ratio = sticky_config.Q_RATIO
        self.quant_bit_width = sticky_config.QUANTIZATION_BIT_WIDTH
        local_fixed = getattr(sticky_config, "LOCAL_NUM_TOKENS", None)
        if local_fixed is None and config is not None and hasattr(config, "local_num_tokens"):
            local_fixed = config.local_num_tokens
        self.use_fixed_local_tokens = local_fixed is not None
        self.local_num_tokens = local_fixed if local_fixed is not None else 0
        if config is not None and hasattr(config, "hidden_size") and hasattr(config, "num_attention_heads"):
            self.head_dim = config.hidden_size // config.num_attention_heads
            kvh = getattr(config, "num_key_value_heads", config.num_attention_heads)
            self.group = config.num_attention_heads // kvh
        else:
            self.head_dim = 64
            self.group = 1
        max_context = getattr(config, "max_position_embeddings", None) if config is not None else None
        if max_context is not None:
            mw = max((max_context - self.sink_tokens) // self.omega, 1) if max_context > self.sink_tokens else 1
            self.max_windows = max(mw, 100)
        else:
            self.max_windows = 30000
        # research token ledger (cache.py:112-119,148-153,183-186)
        self._tracking_flag = getattr(sticky_config, "tracking_flag", 0) == 1
        self.max_context = max_context if max_context is not None else 131072
        self.tracking_managers = []
        self.k_windows = 0
        self.local_num = 0
        self.q_windows_count = 0
        self.q_num = 0
        self.state = None
        self._prefill_done = False
        self._bypass = False
        self._new_tokens = 0
        self._counter = 0     # global token counter while no device state exists (bypass)
        self._workspace = None
        self.reference_rounding = False

    # -- state ----------------------------------------------------------------
    def _clean_scores(self):
        """Forget the sequence: the next call is a prefill (cache.py:_clean_scores)."""
        self.state = None
        self._prefill_done = False
        self._bypass = False
        self._new_tokens = 0
        self._counter = 0
        for tr in self.tracking_managers:
            tr.reset()

    def attach_workspace(self, workspace):
        """Share one decode/cycle workspace between the layers of a model (one stream)."""
        self._workspace = workspace

    def _build_state(self, B, H, D, dtype, device, prompt_len):
        budget = compute_budget(
            total_cache_ratio=self.total_cache_ratio, sink_tokens=self.sink_tokens,
            use_fixed_local_tokens=self.use_fixed_local_tokens, local_num_tokens=self.local_num_tokens,
            local_cache_ratio=self.local_cache_ratio, q_ratio=self.q_ratio, quant_bit_width=self.quant_bit_width,
            head_dim=D, omega=self.omega, new_tokens=prompt_len,
            max_tokens=sticky_config.GENERATION_CONFIG.get("max_new_tokens", 512), layer_idx=self.layer_idx)
        self.local_num = budget.local_num
        self.k_windows = budget.k_windows
        self.q_windows_count = budget.q_windows_count if self.q_ratio > 0 else 0
        self.q_num = budget.q_num
        ws = self._workspace
        if ws is not None:
            dims = N.QvDims(B, H, self.group, D, self.omega, self.sink_tokens, self.local_num, self.k_windows,
                            self.q_windows_count, self.max_windows, self.quant_bit_width,
                            kv_dtype_code(dtype), 0)
            if not ws.fits(dims):
                ws = None
        st = StickyLayerState(B, H, self.group, D, self.omega, self.sink_tokens, self.local_num, self.k_windows,
                              self.q_windows_count, self.max_windows, self.quant_bit_width, dtype, device,
                              workspace=ws, reference_rounding=self.reference_rounding)
        self.state = st
        return st

    def prefill_state(self, key_states, value_states, colsum):
        """Build the device state from a rotated prompt (k/v [B, H, S, D], colsum [B, H, S])."""
        B, H, S, D = key_states.shape
        if H != self.num_heads:
            raise N.QevictError(f"expected {self.num_heads} KV heads, got {H}")
        st = self._build_state(B, H, D, key_states.dtype, key_states.device, S)
        st.prefill(key_states, value_states, colsum)
        self._prefill_done = True
        return st

    # -- reference call ---------------------------------------------------------------
    def __call__(self, past_key_values, attn_score_cache, full_attn_scores=None, q_len=None, q_attn_scores=None):
        if past_key_values is None:
            if not self._prefill_done:
                self._new_tokens = q_len if q_len is not None else attn_score_cache.shape[2]
            return past_key_values
        K, V = past_key_values
        if not self._prefill_done:
            ql = q_len if q_len is not None else attn_score_cache.shape[2]
            self._trackers(K.shape[0], K.device)
            for tr in self.tracking_managers:      # counter restarts at a prompt (cache.py:253-257)
                tr.set_counter(ql)
            if self.total_cache_ratio >= 100 and self.q_ratio == 0:
                # full cache requested: the prompt KV is kept untouched (cache.py:302-304)
                self._prefill_done = True
                self._bypass = True
                self._counter = ql
                return past_key_values
            if self.total_cache_ratio == 100:
                # the reference evicts at the prefill and then never compacts again
                # (cache.py:391-397): its physical cache grows without bound, which
                # a fixed slot layout cannot hold
                raise N.QevictError("R_RATIO == 100 with a Q-cache (Q_RATIO > 0) is not supported: the "
                                    "reference stops compacting after the prefill in that mode; use "
                                    "Q_RATIO = 0 for the full cache, or R_RATIO != 100")
            sc = attn_score_cache
            colsum = sc[:, :, 0, :] if sc.dim() == 4 else sc
            st = self.prefill_state(K.contiguous(), V.contiguous(), colsum.contiguous())
            S = K.shape[2]
            for b, tr in enumerate(self.tracking_managers):   # cache.py:346-351
                tr.record_prefill(seq_len=S, q_len=ql, layer_idx=self.layer_idx,
                                  attn_score_cache=attn_score_cache[b:b + 1],
                                  survivor_ids=st.reference_token_ids(b), full_attn_scores=(
                                      None if full_attn_scores is None else full_attn_scores[b:b + 1]),
                                  global_start=0, num_new_tokens=ql)
            return self._physical()
        gstart = [int(tr.global_token_counter) for tr in self.tracking_managers]
        for tr in self.tracking_managers:
            tr.increment(1)
        if self._bypass:
            self._counter += 1
            return past_key_values
        return self._decode_with_scores(K, V, attn_score_cache, q_attn_scores, gstart)

    def _trackers(self, B, device):
        if len(self.tracking_managers) != B:
            mk = (lambda: TrackingManager(self.max_context, self.num_heads, device)) if self._tracking_flag \
                else (lambda: NoOpTrackingManager(device))
            self.tracking_managers = [mk() for _ in range(B)]

    def _decode_with_scores(self, K, V, scores, q_scores, gstart=None):
        """One decode token whose attention the caller computed (cache.py:357-427)."""
        st = self.state
        B, H = st.B, st.H
        n_ref = K.shape[2] - 1
        pos = [st.reference_positions(b) for b in range(B)]
        if pos[0].shape[1] != n_ref:
            raise N.QevictError(f"physical cache length {n_ref} does not match the cache's {pos[0].shape[1]}")
        # append the (already rotated) new token at its ring slot, then advance
        # the token counter as the fused attention kernel would
        q_dummy = torch.zeros(B, H * st.G, st.D, dtype=st.dtype, device=st.device)
        st.append(q_dummy, K[:, :, -1].contiguous(), V[:, :, -1].contiguous())
        st.step_ctr[0] += 1
        st.n_tokens += 1
        # fold this step's probabilities into the ledger (eviction_manager.py:198-203)
        sc = scores[:, :, 0, :].float()
        for b in range(B):
            posb = st.reference_positions(b)
            st.votes[b].scatter_add_(1, posb, sc[b])
        # Q-window scores (quantize_manager.py:101-111)
        if q_scores is not None:
            ck, qc = st.counts()
            for b in range(B):
                if qc[b] == 0:
                    continue
                # per-window sums, rounded once to the scores' dtype
                win = q_scores[b, :, 0, :qc[b] * st.omega].reshape(H, qc[b], st.omega)
                per_win = win.double().sum(dim=2).to(q_scores.dtype).float()
                o = st.q_order[b, :, :qc[b]].long()
                st.q_score[b].scatter_add_(1, o, per_win)
        track = self._tracking_flag and gstart is not None
        if track:
            for b, tr in enumerate(self.tracking_managers):   # cache.py:371-373
                tr.record_decode(scores[b:b + 1], n_ref + 1, self.layer_idx, gstart[b])
        if st.cycle_due():
            if track:
                old = [(st.reference_token_ids(b), torch.gather(st.votes[b], 1, st.reference_positions(b)))
                       for b in range(B)]
            st.evict_cycle()
            if track:                                          # cache.py:414-424
                for b, tr in enumerate(self.tracking_managers):
                    tr.update_physical_positions(self._cycle_mapping(b, old[b][0]), n_ref + 1, old[b][1])
        return self._physical()

    def _cycle_mapping(self, b, old_ids):
        """[H, S_old] float32: the new physical position of the token each old
        position held, -1 where that token left the cache (cache.py:456-573)."""
        st = self.state
        new_ids = st.reference_token_ids(b)
        n = int(max(int(old_ids.max()), int(new_ids.max()))) + 1
        inv = torch.full((st.H, n), -1.0, dtype=torch.float32, device=st.device)
        pos = torch.arange(new_ids.shape[1], dtype=torch.float32, device=st.device)
        inv.scatter_(1, new_ids, pos[None].expand(st.H, -1).contiguous())
        return torch.gather(inv, 1, old_ids).contiguous()

    def _physical(self):
        st = self.state
        ks, vs = [], []
        for b in range(st.B):
            pos = st.reference_positions(b)
            idx = pos[:, :, None].expand(-1, -1, st.D)
            ks.append(torch.gather(st.k[b], 1, idx))
            vs.append(torch.gather(st.v[b], 1, idx))
        return torch.stack(ks), torch.stack(vs)

    # -- reference properties -----------------------------------------------------------
    def _per_seq(self, fn):
        st = self.state
        if st is None:
            return None
        vals = [fn(b) for b in range(st.B)]
        if any(v is None for v in vals):
            return None
        return vals[0] if st.B == 1 else torch.stack(vals)

    def _q_field(self, name):
        return self._per_seq(lambda b: (lambda q: None if q is None else q[name])(self.state.view_q(b)))

    @property
    def q_cache_k_quant(self):
        return self._q_field("kq")

    @property
    def q_cache_k_scale(self):
        return self._q_field("ks")

    @property
    def q_cache_k_zp(self):
        return self._q_field("kz")

    @property
    def q_cache_v_quant(self):
        return self._q_field("vq")

    @property
    def q_cache_v_scale(self):
        return self._q_field("vs")

    @property
    def q_cache_v_zp(self):
        return self._q_field("vz")

    @property
    def q_cache_ids(self):
        return self._q_field("ids")

    @property
    def q_cache_scores(self):
        return self._q_field("scores")

    @property
    def window_scores(self):
        """[H, max_windows, 3]: (score, id, id) of the sticky windows by ascending id, NaN elsewhere."""
        def one(b):
            ids, sc = self.state.view_sticky(b)
            ws = torch.full((self.state.H, self.max_windows, 3), math.nan)
            k = ids.shape[1]
            ws[:, :k, 0] = sc
            ws[:, :k, 1] = ids.float()
            ws[:, :k, 2] = ids.float()
            return ws
        return self._per_seq(one)

    @property
    def global_token_counter(self):
        if self.state is not None:
            n = self.state.n_tokens
        else:
            n = self._counter if self._bypass else self._new_tokens
        return torch.tensor(n, dtype=torch.long)

    def _tracked(self, fn):
        if not self.tracking_managers:
            return None
        vals = [fn(tr) for tr in self.tracking_managers]
        return vals[0] if len(vals) == 1 else vals

    @property
    def tracking_manager(self):
        return self._tracked(lambda tr: tr)

    @property
    def token_ledger(self):
        """[max_context, 2 + 2H] float32 token ledger (a list of them when B > 1)."""
        return self._tracked(lambda tr: tr.token_ledger)

    @property
    def global_score_history(self):
        return self._tracked(lambda tr: tr._global_score_history)

    @property
    def prefill_attention_matrix(self):
        return self._tracked(lambda tr: tr.prefill_attention_matrix)

    def get_ledger_data(self):
        return self._tracked(lambda tr: tr.get_ledger_data())

    # -- codec (reference static methods, cache.py:626-637; same parameter names) ----------
    @staticmethod
    def _quantize_k_per_window(tensor, bit_width=8):
        return _codec.quantize_k_per_window(tensor, bit_width)

    @staticmethod
    def _quantize_v_per_window(tensor, bit_width=8):
        return _codec.quantize_v_per_window(tensor, bit_width)

    @staticmethod
    def _dequantize_from_quant(quant_tensor, scale, zero_point, bit_width=8):
        return _codec.dequantize_from_quant(quant_tensor, scale, zero_point, bit_width)
