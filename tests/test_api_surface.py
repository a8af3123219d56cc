"""The reference-facing API surface, checked without a GPU.

The reference's only tests (scripts/verify_refactor.py:16-143) are smoke checks
of this kind: imports, properties present, the NoOp manager, compute_budget.
Here the names and signatures its callers use -- the HF decoder layer calling
the attention module, the module calling the cache object, code reading the
cache's properties -- are pinned to the reference's definitions (cited per
item), so that a caller written against the reference finds the same surface."""

import inspect

from qevict_b200 import sticky_config
from qevict_b200.allocator import compute_budget
from qevict_b200.attention import STICKYLlamaAttention, StickyDynamicLayer
from qevict_b200.kv_cache import STICKYKVCache_LayerWise


def _params(fn):
    return list(inspect.signature(fn).parameters)


def test_cache_object_constructor_and_call():
    # src/models/kv_cache/cache.py:44-53, :234-241
    assert _params(STICKYKVCache_LayerWise.__init__) == [
        "self", "p_ratio", "r_ratio", "start_idx", "num_heads", "layer_idx", "config", "k_seq_dim", "v_seq_dim"]
    assert _params(STICKYKVCache_LayerWise.__call__) == [
        "self", "past_key_values", "attn_score_cache", "full_attn_scores", "q_len", "q_attn_scores"]
    for name, default in (("config", None), ("k_seq_dim", 2), ("v_seq_dim", 2)):
        assert inspect.signature(STICKYKVCache_LayerWise.__init__).parameters[name].default == default
    assert callable(STICKYKVCache_LayerWise._clean_scores)        # cache.py:581
    assert callable(STICKYKVCache_LayerWise.get_ledger_data)      # cache.py:603


def test_cache_object_properties():
    # src/models/kv_cache/cache.py:201-228
    for name in ("q_cache_k_quant", "q_cache_k_scale", "q_cache_k_zp", "q_cache_v_quant", "q_cache_v_scale",
                 "q_cache_v_zp", "q_cache_ids", "q_cache_scores", "token_ledger", "global_token_counter",
                 "window_scores", "prefill_attention_matrix", "global_score_history"):
        assert isinstance(inspect.getattr_static(STICKYKVCache_LayerWise, name), property), name


def test_cache_object_static_codec():
    # src/models/kv_cache/cache.py:626-637 (static methods over quantize.py:19-71)
    for name, params in (("_quantize_k_per_window", ["tensor", "bit_width"]),
                         ("_quantize_v_per_window", ["tensor", "bit_width"]),
                         ("_dequantize_from_quant", ["quant_tensor", "scale", "zero_point", "bit_width"])):
        assert isinstance(inspect.getattr_static(STICKYKVCache_LayerWise, name), staticmethod), name
        assert _params(getattr(STICKYKVCache_LayerWise, name)) == params, name
        assert inspect.signature(getattr(STICKYKVCache_LayerWise, name)).parameters["bit_width"].default == 8


def test_attention_module_surface():
    # src/models/attention/module.py:75, :114, :118-127
    assert _params(STICKYLlamaAttention.__init__) == ["self", "config", "layer_idx"]
    assert callable(STICKYLlamaAttention._clean_cache)
    fwd = _params(STICKYLlamaAttention.forward)
    assert fwd[:7] == ["self", "hidden_states", "attention_mask", "position_ids", "past_key_values",
                       "output_attentions", "use_cache"]
    assert fwd[-1] == "kwargs"


def test_dynamic_layer_surface():
    # src/models/sticky_cache.py:25-152: the HF cache layer holding the evicted K/V
    for name in ("set_evicted_kv", "get_seq_length", "get_mask_sizes"):
        assert callable(getattr(StickyDynamicLayer, name)), name
    layer = StickyDynamicLayer()
    assert layer.get_seq_length() == 0 and layer.keys is None


def test_budget_and_config_knobs():
    # src/models/kv_cache/allocator.py:24-107 and src/sticky_config.py
    assert _params(compute_budget) == [
        "total_cache_ratio", "sink_tokens", "use_fixed_local_tokens", "local_num_tokens", "local_cache_ratio",
        "q_ratio", "quant_bit_width", "head_dim", "omega", "new_tokens", "max_tokens", "layer_idx"]
    # the hot-path knobs of src/sticky_config.py (its eval-driver knobs -- model
    # path, datasets, seeds -- are outside the path)
    for knob in ("OMEGA", "SINK_TOKENS", "LOCAL_NUM_TOKENS", "P_RATIO", "R_RATIO", "Q_RATIO",
                 "QUANTIZATION_BIT_WIDTH", "S_IDX", "tracking_flag", "GENERATION_CONFIG"):
        assert hasattr(sticky_config, knob), knob


def test_dynamic_layer_is_a_transformers_cache_layer():
    """The layer is a transformers DynamicLayer whose sequence length is the true
    token count, not the physical length (src/models/sticky_cache.py:25-152),
    so a DynamicCache holding it reports the global position to LlamaModel."""
    import torch
    from transformers import DynamicCache
    from transformers.cache_utils import DynamicLayer
    from qevict_b200.hf import layer_entry
    assert issubclass(StickyDynamicLayer, DynamicLayer)
    cache = DynamicCache()
    e = layer_entry(cache, 1)
    assert isinstance(cache.layers[1], StickyDynamicLayer) and e is cache.layers[1]
    assert not e.is_initialized
    k = torch.randn(1, 2, 7, 4)
    e.set_evicted_kv(k, k + 1)
    e.cumulative_length = 40
    assert e.is_initialized and e.keys is k and cache.get_seq_length(1) == 40
    # mask sizes follow the physical K the attention consumes; the query
    # length may be an int (transformers 5) or a cache_position tensor (4.57)
    assert e.get_mask_sizes(1) == (8, 0) and e.get_mask_sizes(torch.arange(3)) == (10, 0)
    assert cache.get_mask_sizes(1, 1) == (8, 0)
    # DynamicLayer's own append still works for other attention modules
    e2 = StickyDynamicLayer()
    kk, vv = e2.update(torch.ones(1, 2, 3, 4), torch.zeros(1, 2, 3, 4))
    assert kk.shape == (1, 2, 3, 4) and e2.get_seq_length() == 3
    e2.update(torch.ones(1, 2, 1, 4), torch.zeros(1, 2, 1, 4))
    assert e2.keys.shape[-2] == 4 and e2.get_seq_length() == 4
    # a plain layer already in the cache is swapped for a Sticky one
    cache.layers[0] = DynamicLayer()
    assert isinstance(layer_entry(cache, 0), StickyDynamicLayer)


def test_causal_lm_wrapper_surface():
    """STICKYLlamaForCausalLM (src/models/sticky_llama_model.py:28-126): a
    LlamaForCausalLM with the Sticky-KV attention in every layer and the
    generation-position override."""
    from types import SimpleNamespace  # noqa: F401
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaForCausalLM
    from qevict_b200.hf import STICKYLlamaForCausalLM
    assert issubclass(STICKYLlamaForCausalLM, LlamaForCausalLM)
    cfg = LlamaConfig(vocab_size=128, hidden_size=256, num_attention_heads=4, num_key_value_heads=2,
                      intermediate_size=512, num_hidden_layers=2, max_position_embeddings=1024)
    cfg.rope_theta = 500000.0
    m = STICKYLlamaForCausalLM(cfg)
    assert all(type(layer.self_attn).__name__ == "STICKYLlamaAttention" for layer in m.model.layers)
    assert [layer.self_attn.layer_idx for layer in m.model.layers] == [0, 1]
    assert m._get_true_global_position() == 0
