"""The reference's research token ledger, ``TrackingManager``, on the device.

Same class names, constructor, properties and methods as
src/models/kv_cache/tracking_manager.py:27-255 (``TrackingManager`` for
``tracking_flag == 1``, ``NoOpTrackingManager`` otherwise), one sequence per
object as in the reference.  The tables stay on the device and every update is
one native call (``qv_track_prefill`` / ``qv_track_decode`` /
``qv_track_positions``) that performs the reference's float32 arithmetic, so
the ledger and the score history match the reference's bit for bit.

The global token counter is kept on the host (the reference reads its device
copy back with ``.item()`` on every decode token); ``global_token_counter``
returns it as a long tensor.
"""

import torch

from . import _native as N
from .ledger import get_ledger_data as _get_ledger_data


def _f32(t, device):
    return t.to(device=device, dtype=torch.float32).contiguous()


class TrackingManager:
    """Token provenance and cumulative importance ledger of one layer and sequence."""

    def __init__(self, max_context, num_heads, device):
        self.num_heads = num_heads
        self.max_context = max_context
        self.device = torch.device(device)
        self._count = 0
        self._token_ledger = torch.full((max_context, 2 + 2 * num_heads), -1.0, dtype=torch.float32,
                                        device=self.device)
        self._global_score_history = torch.full((max_context, num_heads), -1.0, dtype=torch.float32,
                                                device=self.device)
        self.prefill_attention_matrix = None

    def to(self, device):
        self.device = torch.device(device)
        self._token_ledger = self._token_ledger.to(self.device)
        self._global_score_history = self._global_score_history.to(self.device)
        return self

    @property
    def token_ledger(self):
        return self._token_ledger

    @property
    def global_token_counter(self):
        return torch.tensor(self._count, dtype=torch.long)

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def increment(self, n=1):
        self._count += n

    def set_counter(self, n):
        """Counter reset at a new prompt (the reference zeroes it, cache.py:254-256)."""
        self._count = n

    def record_prefill(self, seq_len, q_len, layer_idx, attn_score_cache, survivor_ids, full_attn_scores,
                       global_start, num_new_tokens):
        """tracking_manager.py:61-124.  attn_score_cache [1, H, q, kv]; survivor_ids [H, N]."""
        dev = self.device
        imp = _f32(attn_score_cache[0, :, :seq_len, :].sum(dim=1), dev)
        surv = survivor_ids.to(device=dev, dtype=torch.int64).contiguous()
        rc = N.lib().qv_track_prefill(self.max_context, self.num_heads, seq_len, q_len, layer_idx, global_start,
                                      num_new_tokens, N.ptr(imp), imp.shape[1], N.ptr(surv), surv.shape[1],
                                      N.ptr(self._token_ledger), N.ptr(self._global_score_history), self._stream())
        N.check(rc, "qv_track_prefill")
        full = full_attn_scores if full_attn_scores is not None else attn_score_cache
        self.prefill_attention_matrix = full[0].detach().cpu()

    def record_decode(self, attn_score_cache, seq_len, layer_idx, global_start):
        """tracking_manager.py:126-160.  attn_score_cache [1, H, 1, kv]."""
        sc = _f32(attn_score_cache[0, :, 0, :], self.device)
        rc = N.lib().qv_track_decode(self.max_context, self.num_heads, self._count, global_start, seq_len, layer_idx,
                                     N.ptr(sc), sc.shape[1], N.ptr(self._token_ledger),
                                     N.ptr(self._global_score_history), self._stream())
        N.check(rc, "qv_track_decode")

    def update_physical_positions(self, mapping, seq_len, running_attention_votes):
        """tracking_manager.py:162-191.  mapping [H, seq_len]; votes [H, >= seq_len]."""
        mp = _f32(mapping[:, :seq_len], self.device)
        vt = _f32(running_attention_votes, self.device)
        rc = N.lib().qv_track_positions(self.max_context, self.num_heads, self._count, seq_len, N.ptr(mp), N.ptr(vt),
                                        vt.shape[1], N.ptr(self._token_ledger),
                                        N.ptr(self._global_score_history), self._stream())
        N.check(rc, "qv_track_positions")

    def get_ledger_data(self):
        return _get_ledger_data(self.global_token_counter, self._token_ledger, self.num_heads)

    def reset(self):
        self._count = 0
        self._token_ledger.fill_(-1.0)
        self._global_score_history.fill_(-1.0)
        self.prefill_attention_matrix = None


class NoOpTrackingManager:
    """tracking_manager.py:207-255: the ledger when tracking_flag == 0."""

    def __init__(self, device):
        self._count = 0
        self._token_ledger = torch.zeros(1, 2, dtype=torch.float32, device=device)
        self._global_score_history = torch.zeros(1, 1, dtype=torch.float32, device=device)
        self.prefill_attention_matrix = None

    def to(self, device):
        self._token_ledger = self._token_ledger.to(device)
        self._global_score_history = self._global_score_history.to(device)
        return self

    @property
    def token_ledger(self):
        return self._token_ledger

    @property
    def global_token_counter(self):
        return torch.tensor(self._count, dtype=torch.long)

    def increment(self, n=1):
        self._count += n

    def set_counter(self, n):
        self._count = n

    def record_prefill(self, seq_len, q_len, layer_idx, attn_score_cache, survivor_ids, full_attn_scores,
                       global_start, num_new_tokens):
        pass

    def record_decode(self, attn_score_cache, seq_len, layer_idx, global_start):
        pass

    def update_physical_positions(self, mapping, seq_len, running_attention_votes):
        pass

    def get_ledger_data(self):
        return {"global_id": torch.zeros(0), "layer_id": torch.zeros(0),
                "physical_id": torch.zeros(0), "attention_score": torch.zeros(0)}

    def reset(self):
        self._count = 0
