"""Hugging Face integration: the cache layer and the causal-LM wrapper of the reference.

* ``StickyDynamicLayer`` -- a ``transformers`` ``DynamicLayer`` that keeps
  the true number of tokens seen (``cumulative_length``) apart from the
  physical K/V length, as the reference's (src/models/sticky_cache.py:25-152):
  ``get_seq_length()`` returns the cumulative length, so Hugging Face's own
  position bookkeeping (``LlamaModel.forward``: position ids = arange +
  ``past_key_values.get_seq_length()``) yields the true global positions;
  ``get_mask_sizes`` uses the physical length.  ``set_evicted_kv`` takes
  tensors, as in the reference; ``attach_state`` binds the layer to a device
  state instead, and ``keys`` / ``values`` then present that state's
  physical cache in the reference's order -- [sinks | sticky windows by
  ascending id | local zone and the tokens appended since] -- gathered on
  access (cached until the state advances).
* ``STICKYLlamaForCausalLM`` -- a ``LlamaForCausalLM`` whose layers use
  ``qevict_b200.attention.STICKYLlamaAttention``, built like the reference's
  (src/models/sticky_llama_model.py:28-56: the parent stack is constructed
  with RoPE scaling stripped, the attention keeps the original config), with
  its ``prepare_inputs_for_generation`` override (sticky_llama_model.py:72-126):
  once a cache exists, one new token per step at the true global position.
"""

from __future__ import annotations

import copy

import torch
from transformers.cache_utils import DynamicLayer


class StickyDynamicLayer(DynamicLayer):
    """Per-layer entry of a Hugging Face cache whose physical K/V is shorter than
    the sequence (src/models/sticky_cache.py:25-152)."""

    is_sliding = False
    is_compileable = False

    def __init__(self):
        self._state = None           # StickyLayerState the physical K/V are read from
        self._kv = (None, None)      # tensors given through set_evicted_kv / update
        self._view = None            # ((n_tokens, last_compaction), (K, V)) of the bound state
        super().__init__()
        self.cumulative_length = 0

    def __repr__(self):
        return f"StickyDynamicLayer(cumulative={self.cumulative_length}, physical={self.physical_length()})"

    # -- physical K/V -----------------------------------------------------------------------
    def _gather(self):
        st = self._state
        key = (st.n_tokens, st.last_compaction)
        if self._view is None or self._view[0] != key:
            ks, vs = [], []
            for b in range(st.B):
                pos = st.reference_positions(b)
                idx = pos[:, :, None].expand(-1, -1, st.D)
                ks.append(torch.gather(st.k[b], 1, idx))
                vs.append(torch.gather(st.v[b], 1, idx))
            self._view = (key, (torch.stack(ks), torch.stack(vs)))
        return self._view[1]

    @property
    def keys(self):
        return self._gather()[0] if self._state is not None else self._kv[0]

    @keys.setter
    def keys(self, t):
        self._state = None
        self._kv = (t, self._kv[1])

    @property
    def values(self):
        return self._gather()[1] if self._state is not None else self._kv[1]

    @values.setter
    def values(self, t):
        self._state = None
        self._kv = (self._kv[0], t)

    def physical_length(self):
        """Tokens of the physical cache (the reference's keys.shape[-2])."""
        st = self._state
        if st is not None:
            ck = st.counts()[0][0]
            return st.sink + ck * st.omega + st.local + (st.n_tokens - st.last_compaction)
        k = self._kv[0]
        return 0 if k is None or k.numel() == 0 else k.shape[-2]

    # -- the reference's cache-layer API --------------------------------------------------------
    def set_evicted_kv(self, keys, values):
        """Replace the physical K/V without touching cumulative_length (sticky_cache.py:104-108)."""
        self._state = None
        self._kv = (keys, values)
        self.is_initialized = True

    def attach_state(self, state):
        """Present a device state's physical cache (reference order) as keys / values."""
        self._state = state
        self._view = None
        self.is_initialized = True

    def increment_cumulative(self, n):
        self.cumulative_length += n

    def lazy_initialization(self, key_states, value_states=None):
        self.dtype, self.device = key_states.dtype, key_states.device
        self._state = None
        self._kv = (torch.tensor([], dtype=self.dtype, device=self.device),
                    torch.tensor([], dtype=self.dtype, device=self.device))
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        """DynamicLayer's append (for callers other than the Sticky-KV attention,
        which never calls it): concatenates and counts the tokens."""
        if not self.is_initialized or self._state is not None:
            self.lazy_initialization(key_states, value_states)
        self.cumulative_length += key_states.shape[-2]
        self._kv = (torch.cat([self._kv[0], key_states], dim=-2), torch.cat([self._kv[1], value_states], dim=-2))
        return self._kv

    def get_seq_length(self, *args, **kwargs):
        """The true number of tokens seen, not the physical length (sticky_cache.py:73-75)."""
        return self.cumulative_length

    def get_mask_sizes(self, query_length, *args, **kwargs):
        """(physical length + query length, 0): the K the attention consumes.
        query_length may be an int or a cache_position tensor (transformers 4.57)."""
        q = query_length.shape[0] if hasattr(query_length, "shape") else int(query_length)
        return self.physical_length() + q, 0

    def get_max_cache_shape(self):
        return -1

    def reset(self):
        if self._state is None and self._kv[0] is not None:
            self._kv[0].zero_()
            self._kv[1].zero_()
        self.cumulative_length = 0

    def offload(self):
        if self._state is None and self._kv[0] is not None:
            self._kv = (self._kv[0].to("cpu", non_blocking=True), self._kv[1].to("cpu", non_blocking=True))

    def prefetch(self):
        pass

    def crop(self, max_length):
        if self._state is not None:
            raise NotImplementedError("a Sticky-KV cache cannot be cropped: tokens are evicted by window")
        super().crop(max_length)

    def reorder_cache(self, beam_idx):
        if self._state is not None:
            raise NotImplementedError("beam search is not supported on a Sticky-KV device state")
        k, v = self._kv
        if k is not None and k.numel() > 0:
            self._kv = (k.index_select(0, beam_idx.to(k.device)), v.index_select(0, beam_idx.to(v.device)))

    def batch_repeat_interleave(self, repeats):
        if self._state is not None:
            raise NotImplementedError("the batch of a Sticky-KV device state is fixed at its prefill")
        k, v = self._kv
        if k is not None and k.numel() > 0:
            self._kv = (k.repeat_interleave(repeats, dim=0), v.repeat_interleave(repeats, dim=0))

    def batch_select_indices(self, indices):
        if self._state is not None:
            raise NotImplementedError("the batch of a Sticky-KV device state is fixed at its prefill")
        k, v = self._kv
        if k is not None and k.numel() > 0:
            self._kv = (k[indices, ...], v[indices, ...])


def layer_entry(past_key_values, layer_idx):
    """The StickyDynamicLayer of layer_idx in a Hugging Face cache (created, or
    swapped in for a plain DynamicLayer, as the reference's _write_kv_to_cache
    does at src/models/attention/module.py:47-70); None without a cache."""
    if past_key_values is None or not hasattr(past_key_values, "layers"):
        return None
    layers = past_key_values.layers
    while len(layers) <= layer_idx:
        layers.append(StickyDynamicLayer())
    if not isinstance(layers[layer_idx], StickyDynamicLayer):
        layers[layer_idx] = StickyDynamicLayer()
    return layers[layer_idx]


def _llama_for_causal_lm():
    from transformers.models.llama.modeling_llama import LlamaForCausalLM
    return LlamaForCausalLM


class STICKYLlamaForCausalLM(_llama_for_causal_lm()):
    """LlamaForCausalLM with the fused Sticky-KV attention in every layer
    (src/models/sticky_llama_model.py:28-126)."""

    def __init__(self, config, **kwargs):
        from .attention import STICKYLlamaAttention
        safe = copy.deepcopy(config)
        if hasattr(safe, "rope_scaling"):
            safe.rope_scaling = None
        safe.rope_parameters = {"rope_type": "default", "rope_theta": getattr(safe, "rope_theta", None) or
                                (getattr(config, "rope_parameters", None) or {}).get("rope_theta", 10000.0)}
        super().__init__(safe)
        self.config = config
        for i in range(len(self.model.layers)):
            self.model.layers[i].self_attn = STICKYLlamaAttention(config, i)

    def _get_true_global_position(self):
        """Tokens seen so far by layer 0's cache (sticky_llama_model.py:58-70)."""
        try:
            attn = self.model.layers[0].self_attn
            return int(attn.kv_cache.global_token_counter.item())
        except (IndexError, AttributeError):
            return None

    def prepare_inputs_for_generation(self, input_ids, past_key_values=None, attention_mask=None,
                                      inputs_embeds=None, **kwargs):
        """After the prompt, feed one token per step at the true global position
        (sticky_llama_model.py:72-126): the physical cache is shorter than the
        sequence, so lengths derived from it would be wrong."""
        inputs = super().prepare_inputs_for_generation(input_ids, past_key_values=past_key_values,
                                                       attention_mask=attention_mask, inputs_embeds=inputs_embeds,
                                                       **kwargs)
        tc = self._get_true_global_position()
        if past_key_values is not None and tc:
            dev = input_ids.device
            inputs["input_ids"] = input_ids[:, -1:]
            inputs.pop("inputs_embeds", None)
            inputs["past_key_values"] = past_key_values
            inputs["use_cache"] = True
            inputs["position_ids"] = torch.tensor([[tc]], dtype=torch.long, device=dev).expand(input_ids.shape[0], 1)
            inputs["cache_position"] = torch.tensor([tc], dtype=torch.long, device=dev)
        return inputs
