"""Q-cache codec restated in numpy (test infrastructure only).

Follows ``src/models/kv_cache/quantize.py`` of the reference:
  * K: per window, per channel (min/max over the omega tokens), with the
    RoPE-paired channels i and i+D/2 tied to one range   (quantize.py:19-44)
  * V: per window, per token (min/max over the D channels) (quantize.py:47-59)
  * dequantisation ``code*scale + zp`` in the KV dtype      (quantize.py:62-71)
  * path-C re-quantisation with an archived scale/zp        (quantize_manager.py:305-314)

All arithmetic is evaluated the way torch evaluates it on the KV dtype: one
fp32 operation per torch op, rounded back to the dtype (see ``numerics``).
"""

import numpy as np

from .numerics import f32, op, rnd, to_uint8_like_torch


def _levels(bit_width):
    """Quantisation levels: 255 for INT8, 15 for INT4 (quantize.py:37-53)."""
    return 15.0 if bit_width == 4 else 255.0


def _pack4(q):
    """(q[..., 0::2] << 4) | q[..., 1::2]  (quantize.py:39)."""
    q = q.astype(np.uint8)
    return ((q[..., 0::2] << 4) | q[..., 1::2]).astype(np.uint8)


def _codes(x, t_min, scale, dt, bit_width):
    """round((x - t_min) / scale).clamp(0, L) -> uint8   (quantize.py:38,43,58)."""
    lv = _levels(bit_width)
    diff = op(np.subtract, dt, x, t_min)
    ratio = op(np.divide, dt, diff, scale)
    r = np.round(ratio)  # torch.round: half to even, exact on representable values
    with np.errstate(invalid="ignore"):
        r = np.clip(r, 0.0, lv)
    return to_uint8_like_torch(r)


def _scale(t_min, t_max, dt, bit_width):
    """torch.clamp((t_max - t_min) / L, min=1e-8) in the KV dtype (quantize.py:37,42)."""
    rng = op(np.subtract, dt, t_max, t_min)
    s = op(np.divide, dt, rng, np.float32(_levels(bit_width)))
    return op(np.maximum, dt, s, np.float32(1e-8))


def quantize_k_per_window(x, dt, bit_width=8):
    """x: [..., W, omega, D] (values in dt).  Returns (codes, scale[...,W,1,D], zp[...,W,1,D]).

    reference: src/models/kv_cache/quantize.py:19-44
    """
    x = f32(x)
    t_min = x.min(axis=-2, keepdims=True)
    t_max = x.max(axis=-2, keepdims=True)
    half = x.shape[-1] // 2
    mn = np.minimum(t_min[..., :half], t_min[..., half:])
    mx = np.maximum(t_max[..., :half], t_max[..., half:])
    t_min = np.concatenate([mn, mn], axis=-1)
    t_max = np.concatenate([mx, mx], axis=-1)
    scale = _scale(t_min, t_max, dt, bit_width)
    q = _codes(x, t_min, scale, dt, bit_width)
    if bit_width == 4:
        q = _pack4(q)
    return q, scale, rnd(t_min, dt)


def quantize_v_per_window(x, dt, bit_width=8):
    """x: [..., W, omega, D].  Returns (codes, scale[...,W,omega,1], zp[...,W,omega,1]).

    reference: src/models/kv_cache/quantize.py:47-59
    """
    x = f32(x)
    t_min = x.min(axis=-1, keepdims=True)
    t_max = x.max(axis=-1, keepdims=True)
    scale = _scale(t_min, t_max, dt, bit_width)
    q = _codes(x, t_min, scale, dt, bit_width)
    if bit_width == 4:
        q = _pack4(q)
    return q, scale, rnd(t_min, dt)


def dequantize_from_quant(codes, scale, zp, dt, bit_width=8):
    """code.to(dtype) * scale + zero_point in the KV dtype (quantize.py:62-71)."""
    codes = np.asarray(codes)
    if bit_width == 4:
        hi = (codes >> 4) & 0x0F
        lo = codes & 0x0F
        codes = np.stack([hi, lo], axis=-1).reshape(*codes.shape[:-1], -1)
    c = f32(codes)
    return op(np.add, dt, op(np.multiply, dt, c, scale), zp)


def requantize_with_meta(x, scale, zp, dt, bit_width=8):
    """Path C: round((x - zp) / scale).clamp(0, L) with archived scale/zp.

    reference: src/models/kv_cache/quantize_manager.py:305-314
    """
    q = _codes(x, zp, scale, dt, bit_width)
    if bit_width == 4:
        q = _pack4(q)
    return q
