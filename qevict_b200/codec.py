"""Q-cache codec on the GPU, with the reference's function signatures.

``quantize_k_per_window`` / ``quantize_v_per_window`` / ``dequantize_from_quant``
mirror src/models/kv_cache/quantize.py:19-71 (same argument meaning, same
shapes, bit-identical codes and scales); they run the sm_100a kernels behind
qv_quantize_k / qv_quantize_v / qv_dequantize.
"""

import ctypes

import torch

from . import _native as N
from .layer_state import kv_dtype_code


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check_input(tensor):
    if not tensor.is_cuda:
        raise N.QevictError("qevict_b200 codec runs on CUDA tensors only")
    return tensor.contiguous()


def quantize_k_per_window(tensor, bit_width=8):
    """[..., W, omega, D] -> (codes [..., W, omega, D or D/2] u8, scale [..., W, 1, D], zp [..., W, 1, D])."""
    x = _check_input(tensor)
    *lead, om, D = x.shape
    n = x.numel() // (om * D)
    qb = D if bit_width == 8 else D // 2
    codes = torch.empty(*lead, om, qb, dtype=torch.uint8, device=x.device)
    scale = torch.empty(*lead, 1, D, dtype=x.dtype, device=x.device)
    zp = torch.empty_like(scale)
    N.check(N.lib().qv_quantize_k(n, om, D, bit_width, kv_dtype_code(x.dtype), N.ptr(x), N.ptr(codes),
                                  N.ptr(scale), N.ptr(zp), _stream(x)), "qv_quantize_k")
    return codes, scale, zp


def quantize_v_per_window(tensor, bit_width=8):
    """[..., W, omega, D] -> (codes, scale [..., W, omega, 1], zp [..., W, omega, 1])."""
    x = _check_input(tensor)
    *lead, om, D = x.shape
    n = x.numel() // (om * D)
    qb = D if bit_width == 8 else D // 2
    codes = torch.empty(*lead, om, qb, dtype=torch.uint8, device=x.device)
    scale = torch.empty(*lead, om, 1, dtype=x.dtype, device=x.device)
    zp = torch.empty_like(scale)
    N.check(N.lib().qv_quantize_v(n, om, D, bit_width, kv_dtype_code(x.dtype), N.ptr(x), N.ptr(codes),
                                  N.ptr(scale), N.ptr(zp), _stream(x)), "qv_quantize_v")
    return codes, scale, zp


def dequantize_from_quant(quant_tensor, scale, zero_point, bit_width=8):
    """code * scale + zero_point in the scale's dtype (K: scale [...,1,D]; V: scale [...,omega,1])."""
    q = _check_input(quant_tensor)
    scale = _check_input(scale)
    zero_point = _check_input(zero_point)
    *lead, om, qb = q.shape
    D = qb if bit_width == 8 else qb * 2
    n = q.numel() // (om * qb)
    per_token = 1 if scale.shape[-1] == 1 and D != 1 else 0
    out = torch.empty(*lead, om, D, dtype=scale.dtype, device=q.device)
    N.check(N.lib().qv_dequantize(n, om, D, bit_width, kv_dtype_code(scale.dtype), per_token, N.ptr(q),
                                  N.ptr(scale), N.ptr(zero_point), N.ptr(out), _stream(q)), "qv_dequantize")
    return out
