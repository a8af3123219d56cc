"""Sticky-KV knobs, under the names the reference's ``src/sticky_config.py`` uses.

The reference's cache reads these module attributes when a cache object is
constructed (``STICKYKVCache_LayerWise.__init__``, src/models/kv_cache/cache.py:66-119)
and when its prefill computes the budget (cache.py:263-287); the classes in
``qevict_b200.kv_cache`` read this module the same way, so a caller switches
configurations by assigning to it before constructing a layer.

Defaults are the decode workload this library is tuned for (Llama-3-8B shape,
32k context): windows of 64 tokens, 64 sinks, a fixed 512-token local zone and
an INT8 Q-cache.  The reference ships OMEGA = 8 and SINK_TOKENS = 4; the
kernels here take OMEGA in 16..128 (a multiple of 16), so OMEGA = 8 raises.
"""

OMEGA = 64                  # tokens per window
SINK_TOKENS = 64            # always-kept leading tokens
LOCAL_NUM_TOKENS = 512      # fixed local zone (set to None to use P_RATIO instead)
P_RATIO = 50                # local zone as % of the budget, when LOCAL_NUM_TOKENS is None
R_RATIO = 20                # total cache budget as % of (prompt + max_new_tokens)
Q_RATIO = 10                # % of the window budget given to the quantised Q-cache
QUANTIZATION_BIT_WIDTH = 8  # 8 (INT8) or 4 (packed INT4)
S_IDX = 0                   # start index for window tracking (start_idx)
tracking_flag = 0           # 1: keep the research token ledger (TrackingManager)
GENERATION_CONFIG = {"max_new_tokens": 512, "do_sample": False, "temperature": 1.0}
