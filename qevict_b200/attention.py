"""The reference's attention-module API, ``STICKYLlamaAttention``, on the fused kernels.

Same constructor (``config, layer_idx``), projections (``q_proj``, ``k_proj``,
``v_proj``, ``o_proj``), cache attribute (``kv_cache``), ``_clean_cache()`` and
``forward`` signature as ``STICKYLlamaAttention`` (src/models/attention/module.py:73-369
and module_flash.py), returning ``(attn_output [B, q_len, hidden], None)``.

  * prefill (q_len > 1): projections, RoPE at positions 0..q_len-1 (``qv_rope``),
    causal attention with per-key column sums (``qv_prefill_attention``; the
    scores of module_flash.py / ops_flash.py:56-141), then the device state is
    built from the rotated prompt (``qv_prefill_build``);
  * decode (q_len == 1): RoPE at the true position and in-place append
    (``qv_rope_append``), the fused attention over [sinks | sticky | local] and
    the Q-cache with the ledger fold (``qv_decode_attention``), and every OMEGA
    tokens the eviction cycle (``qv_evict_cycle``).

Differences from the reference, by design: attention weights are never
materialised (``output_attentions`` returns None); the prompt must fill whole
windows after the sinks (``(q_len - SINK_TOKENS) % OMEGA == 0``) and cover
the local zone; one prefill per sequence (call ``_clean_cache()`` before the
next); the full-cache mode (R_RATIO >= 100 with Q_RATIO == 0) is not offered
by the fused path (the cache object alone supports it).
"""

import math

import torch
from torch import nn

from . import _native as N
from .kv_cache import STICKYKVCache_LayerWise
from .model import prefill_attention, rope_


def rope_inv_freq(config, head_dim):
    """Inverse frequencies of the rotary embedding the reference builds (rope.py:185-240):
    Llama-3 scaled when ``config.rope_scaling`` says ``llama3``, else the plain
    ``theta^(-2i/D)`` of HF's default Llama rotary embedding."""
    theta = float(getattr(config, "rope_theta", None) or (getattr(config, "rope_parameters", None) or {}).get(
        "rope_theta", 10000.0))
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    rs = getattr(config, "rope_scaling", None)
    if isinstance(rs, dict) and (rs.get("rope_type") or rs.get("type")) == "llama3":
        # Llama 3.1 frequency scaling: long wavelengths divided by `factor`, short
        # ones kept, a linear blend in between
        factor = float(rs.get("factor", 8.0))
        lo = float(rs.get("low_freq_factor", 1.0))
        hi = float(rs.get("high_freq_factor", 4.0))
        orig = float(rs.get("original_max_position_embeddings", 8192))
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen) - lo) / (hi - lo)
        blended = (1 - smooth) * inv / factor + smooth * inv
        inv = torch.where(wavelen > orig / lo, inv / factor, torch.where(wavelen < orig / hi, inv, blended))
    return inv


class StickyDynamicLayer:
    """Per-layer entry of a HF-style cache object (src/models/sticky_cache.py:25-152):
    the physical K/V the layer holds and the true number of tokens seen."""

    is_sliding = False
    is_compileable = False

    def __init__(self):
        self.keys = None
        self.values = None
        self.is_initialized = False
        self.cumulative_length = 0

    def set_evicted_kv(self, keys, values):
        self.keys, self.values = keys, values
        self.is_initialized = True

    def get_seq_length(self, *args, **kwargs):
        return self.cumulative_length

    def get_mask_sizes(self, cache_position, *args, **kwargs):
        q = cache_position.shape[0] if hasattr(cache_position, "shape") else int(cache_position)
        phys = self.keys.shape[-2] if self.keys is not None else 0
        return phys + q, 0

    def __repr__(self):
        phys = self.keys.shape[-2] if self.keys is not None else 0
        return f"StickyDynamicLayer(cumulative={self.cumulative_length}, physical={phys})"


class STICKYLlamaAttention(nn.Module):
    def __init__(self, config, layer_idx):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = self.hidden_size // self.num_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.max_position_embeddings = config.max_position_embeddings
        self.rope_theta = getattr(config, "rope_theta", None)
        if self.head_dim * self.num_heads != self.hidden_size:
            raise ValueError(f"hidden_size ({self.hidden_size}) not divisible by num_heads ({self.num_heads})")
        self.q_proj = nn.Linear(self.hidden_size, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.hidden_size, bias=False)
        self.kv_cache = STICKYKVCache_LayerWise(
            p_ratio=getattr(config, "p_ratio", 50), r_ratio=getattr(config, "r_ratio", 20),
            start_idx=getattr(config, "start_idx", 0), num_heads=self.num_key_value_heads,
            layer_idx=layer_idx, config=config)
        self.register_buffer("inv_freq", rope_inv_freq(config, self.head_dim), persistent=False)
        self._rope = None   # (dtype, device, length, cos, sin)

    def _clean_cache(self):
        self.kv_cache._clean_scores()

    def _tables(self, dtype, device, length):
        r = self._rope
        if r is None or r[0] != dtype or r[1] != device or r[2] < length:
            n = max(length, self.max_position_embeddings)
            t = torch.arange(n, device=device, dtype=torch.float32)
            fr = torch.outer(t, self.inv_freq.to(device=device, dtype=torch.float32))
            emb = torch.cat([fr, fr], dim=-1)
            r = (dtype, device, n, emb.cos().to(dtype).contiguous(), emb.sin().to(dtype).contiguous())
            self._rope = r
        return r[3], r[4]

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                output_attentions=False, use_cache=False, **kwargs):
        B, T, _ = hidden_states.shape
        Hq, H, D = self.num_heads, self.num_key_value_heads, self.head_dim
        cache = self.kv_cache
        if cache.state is None:
            if cache.total_cache_ratio >= 100 and cache.q_ratio == 0:
                raise N.QevictError("the fused path always evicts: R_RATIO >= 100 with Q_RATIO == 0 is not offered")
            cos, sin = self._tables(hidden_states.dtype, hidden_states.device, T + 1)
            q = self.q_proj(hidden_states).view(B, T, Hq, D).contiguous()
            k = self.k_proj(hidden_states).view(B, T, H, D).contiguous()
            v = self.v_proj(hidden_states).view(B, T, H, D).contiguous()
            rope_(q, cos, sin)
            rope_(k, cos, sin)
            out, colsum = prefill_attention(q, k, v)
            cache.prefill_state(k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous(), colsum)
            attn = out.reshape(B, T, Hq * D)
        else:
            if T != 1:
                raise N.QevictError("one prefill per sequence: call _clean_cache() before a new prompt")
            st = cache.state
            if B != st.B:
                raise N.QevictError(f"batch {B} does not match the prefilled batch {st.B}")
            cos, sin = self._tables(hidden_states.dtype, hidden_states.device, st.n_tokens + 2)
            x = hidden_states[:, 0]
            qr = st.append(self.q_proj(x).view(B, Hq, D), self.k_proj(x).view(B, H, D),
                           self.v_proj(x).view(B, H, D), cos, sin)
            out = torch.empty(B, Hq, D, dtype=hidden_states.dtype, device=hidden_states.device)
            st.attend(qr, out)
            if st.cycle_due():
                st.evict_cycle()
            attn = out.reshape(B, 1, Hq * D)
        if use_cache and past_key_values is not None and hasattr(past_key_values, "layers"):
            layers = past_key_values.layers
            while len(layers) <= self.layer_idx:
                layers.append(StickyDynamicLayer())
            if not isinstance(layers[self.layer_idx], StickyDynamicLayer):
                layers[self.layer_idx] = StickyDynamicLayer()
            entry = layers[self.layer_idx]
            entry.set_evicted_kv(cache.state.k, cache.state.v)
            entry.cumulative_length = cache.state.n_tokens
        return self.o_proj(attn), None
