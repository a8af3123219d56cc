"""ctypes binding of the C ABI declared in include/qevict_b200.h.

The shared library is built in-tree (``qevict_b200/_lib/libqevict_b200.so``)
by ``qevict_b200.build.build()``.  There is no fallback: importing a compute
entry point without the library raises immediately.
"""

import ctypes
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libqevict_b200.so")

QV_OK, QV_EINVAL, QV_ENOTALIGNED, QV_ESPACE, QV_ECUDA = 0, -1, -2, -3, -4
QV_F32, QV_BF16, QV_F16 = 0, 1, 2
QV_DERR_TABLE, QV_DERR_LAYOUT, QV_DERR_CAPACITY, QV_DERR_TIMEOUT = 1, 2, 4, 8
QV_PEER_HANDLE_BYTES = 64
QV_NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024   # include/qevict_b200.h

_ERRNAMES = {QV_EINVAL: "invalid argument", QV_ENOTALIGNED: "prompt/local zone not window-aligned",
             QV_ESPACE: "workspace too small", QV_ECUDA: "CUDA error"}


class QvDims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch", "kv_heads", "group", "head_dim", "omega", "sink", "local", "k_windows",
        "q_windows", "max_windows", "bits", "dtype", "flags")]

QV_FLAG_REFERENCE_ROUNDING = 1


class QvLayer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "k", "v", "kq", "vq", "ks", "kz", "vs", "vz", "sticky_wid", "sticky_score",
        "sticky_order", "q_wid", "q_score", "q_order", "votes", "local_hist", "arch_valid",
        "arch_ks", "arch_kz", "arch_vs", "arch_vz", "seq", "step", "err")]


class QevictError(RuntimeError):
    pass


_lib = None


def lib():
    """Load the native library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise QevictError(
            f"qevict_b200 native library not found at {_LIB_PATH}; build it with "
            "`python -c 'import qevict_b200.build as b; b.build()'` (nvcc, sm_100a)")
    L = ctypes.CDLL(_LIB_PATH)
    P = ctypes.POINTER
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    D, Lp = P(QvDims), P(QvLayer)
    sig = {
        "qv_ring_windows": (i32, [D]),
        "qv_main_capacity": (i32, [D]),
        "qv_decode_workspace_bytes": (sz, [D]),
        "qv_decode_path": (i32, [D]),
        "qv_decode_logits_offset": (sz, [D]),
        "qv_cycle_workspace_bytes": (sz, [D]),
        "qv_rope_append": (ctypes.c_int, [D, Lp, vp, vp, vp, vp, vp, vp, vp]),
        "qv_decode_attention": (ctypes.c_int, [D, Lp, vp, vp, vp, sz, vp]),
        "qv_decode_attention_noalloc": (ctypes.c_int, [D, Lp, vp, vp, vp]),
        "qv_decode_attention_nofold": (ctypes.c_int, [D, Lp, vp, vp, vp, sz, vp]),
        "qv_decode_fold": (ctypes.c_int, [D, Lp, vp, sz, vp]),
        "qv_rope": (ctypes.c_int, [i32, i32, i32, i32, i32, vp, vp, vp, i32, vp]),
        "qv_evict_cycle": (ctypes.c_int, [D, Lp, vp, sz, vp]),
        "qv_evict_cycle_count": (ctypes.c_int, [D, Lp, vp, sz, vp, vp]),
        "qv_evict_cycle_ext": (ctypes.c_int, [D, Lp, vp, sz, vp, vp]),
        "qv_prefill_build": (ctypes.c_int, [D, Lp, vp, vp, i32, vp, i32, vp]),
        "qv_prefill_attention": (ctypes.c_int, [D, vp, vp, vp, i32, vp, vp, vp, sz, vp]),
        "qv_prefill_workspace_bytes": (sz, [D, i32]),
        "qv_prefill_read_error": (ctypes.c_int, [vp, sz, P(i32), vp]),
        "qv_quantize_k": (ctypes.c_int, [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
        "qv_quantize_v": (ctypes.c_int, [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
        "qv_dequantize": (ctypes.c_int, [i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
        "qv_add_rmsnorm": (ctypes.c_int, [i32, i32, vp, vp, vp, ctypes.c_float, vp, vp]),
        "qv_silu_mul": (ctypes.c_int, [i32, i32, vp, vp, vp]),
        "qv_gemv": (ctypes.c_int, [i32, i32, i32, vp, vp, vp, vp]),
        "qv_argmax_workspace_bytes": (sz, [i32]),
        "qv_argmax": (ctypes.c_int, [i32, i32, vp, vp, vp, sz, vp]),
        "qv_track_prefill": (ctypes.c_int, [i32, i32, i32, i32, i32, i64, i32, vp, i32, vp, i32, vp, vp, vp]),
        "qv_track_decode": (ctypes.c_int, [i32, i32, i64, i64, i32, i32, vp, i32, vp, vp, vp]),
        "qv_track_positions": (ctypes.c_int, [i32, i32, i64, i32, vp, vp, i32, vp, vp, vp]),
        "qv_read_error": (ctypes.c_int, [Lp, P(i32), vp]),
        "qv_peer_sum_create": (ctypes.c_int, [i32, i32, sz, P(vp), vp]),
        "qv_peer_sum_open": (ctypes.c_int, [vp, ctypes.c_char_p]),
        "qv_peer_sum_bf16": (ctypes.c_int, [vp, vp, vp, i64, vp]),
        "qv_peer_max_i64": (ctypes.c_int, [vp, vp, vp, i64, vp]),
        "qv_peer_sum_read_error": (ctypes.c_int, [vp, P(i32), vp]),
        "qv_peer_sum_destroy": (ctypes.c_int, [vp]),
        "qv_last_cuda_error": (ctypes.c_char_p, []),
        "qv_version": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def exported_symbols():
    """Names the header declares (used by the CPU test that checks the exports)."""
    return ["qv_ring_windows", "qv_main_capacity", "qv_decode_workspace_bytes", "qv_decode_path",
            "qv_decode_logits_offset",
            "qv_cycle_workspace_bytes", "qv_rope_append", "qv_rope", "qv_decode_attention",
            "qv_decode_attention_noalloc", "qv_decode_attention_nofold", "qv_decode_fold", "qv_evict_cycle",
            "qv_evict_cycle_count", "qv_evict_cycle_ext",
            "qv_prefill_build", "qv_prefill_attention", "qv_prefill_workspace_bytes", "qv_prefill_read_error",
            "qv_quantize_k", "qv_quantize_v", "qv_dequantize", "qv_add_rmsnorm", "qv_silu_mul", "qv_gemv",
            "qv_argmax_workspace_bytes", "qv_argmax", "qv_track_prefill", "qv_track_decode",
            "qv_track_positions", "qv_read_error",
            "qv_peer_sum_create", "qv_peer_sum_open", "qv_peer_sum_bf16", "qv_peer_max_i64", "qv_peer_sum_read_error",
            "qv_peer_sum_destroy",
            "qv_last_cuda_error", "qv_version"]


def check(rc, what):
    if rc != QV_OK:
        msg = _ERRNAMES.get(rc, f"error {rc}")
        if rc == QV_ECUDA:
            msg += ": " + lib().qv_last_cuda_error().decode()
        raise QevictError(f"{what} failed: {msg}")


def ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())
