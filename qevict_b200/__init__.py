"""qevict_b200 -- the Sticky-KV decode hot path of Qevict on B200 (sm_100a).

The hot path runs in hand-written CUDA kernels behind the C ABI declared in
include/qevict_b200.h (loaded with ctypes from qevict_b200/_lib).  The Python
classes keep the reference's public API so they drop into a Llama attention
forward:

  STICKYKVCache_LayerWise   (reference: src/models/kv_cache/cache.py)
  STICKYLlamaAttention      (reference: src/models/attention/module.py)
  StickyDynamicLayer        (reference: src/models/sticky_cache.py)
  compute_budget            (reference: src/models/kv_cache/allocator.py)
"""

from ._native import QevictError  # noqa: F401
from .layer_state import StickyLayerState, Workspace  # noqa: F401

__all__ = ["QevictError", "StickyLayerState", "Workspace"]
