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

Positions: at the prefill, ``position_ids`` (a contiguous range p0 .. p0+q_len-1)
set the prompt's RoPE positions (module.py:145-150 uses them when no cache is
present); at decode, as in the reference, the position is the true global
token count and the ``position_ids`` / ``attention_mask`` a caller passes are
not used (module.py:141-150 and 163-170 replace them).  With a Hugging Face
cache (``past_key_values``), each layer's entry becomes a
``qevict_b200.hf.StickyDynamicLayer`` bound to the device state: its
``get_seq_length()`` is the true token count and its ``keys`` / ``values``
are the physical cache in the reference's order.  A prompt arriving with a
cache that holds nothing for this layer starts a new sequence.

Differences from the reference, by design: attention weights are never
materialised (``output_attentions`` returns None); the prompt must fill whole
windows after the sinks (``(q_len - SINK_TOKENS) % OMEGA == 0``) and cover
the local zone; the full-cache mode (R_RATIO >= 100 with Q_RATIO == 0) is not
offered by the fused path (the cache object alone supports it).
"""

import math

import torch
from torch import nn

from . import _native as N
from .hf import StickyDynamicLayer, layer_entry  # noqa: F401  (re-exported: the reference's import path)
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
        entry = layer_entry(past_key_values, self.layer_idx)
        if T > 1 and cache.state is not None and entry is not None and not entry.is_initialized:
            # a prompt with a cache that holds nothing for this layer: a new sequence
            self._clean_cache()
        if cache.state is None:
            if cache.total_cache_ratio >= 100 and cache.q_ratio == 0:
                raise N.QevictError("the fused path always evicts: R_RATIO >= 100 with Q_RATIO == 0 is not offered")
            pos0 = 0
            if position_ids is not None:
                p = position_ids.reshape(-1, position_ids.shape[-1])[0].to("cpu", torch.long)
                pos0 = int(p[0])
                if not torch.equal(p, torch.arange(pos0, pos0 + T)):
                    raise N.QevictError("prefill position_ids must be a contiguous range")
            cos, sin = self._tables(hidden_states.dtype, hidden_states.device, pos0 + T + 1)
            q = self.q_proj(hidden_states).view(B, T, Hq, D).contiguous()
            k = self.k_proj(hidden_states).view(B, T, H, D).contiguous()
            v = self.v_proj(hidden_states).view(B, T, H, D).contiguous()
            rope_(q, cos, sin, pos0)
            rope_(k, cos, sin, pos0)
            out, colsum = prefill_attention(q, k, v)
            cache.prefill_state(k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous(), colsum)
            attn = out.reshape(B, T, Hq * D)
        else:
            if T != 1:
                raise N.QevictError("one prefill per sequence: call _clean_cache() (or pass a fresh cache) "
                                    "before a new prompt")
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
        if use_cache and entry is not None:
            # the layer's entry presents the device state (module.py:357-365)
            entry.attach_state(cache.state)
            entry.cumulative_length = cache.state.n_tokens
        return self.o_proj(attn), None
