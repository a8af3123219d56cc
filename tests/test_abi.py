"""The C-ABI library: it loads without a GPU and exports every function the header declares.

Only host-side size helpers are called here (they touch no device).
"""

import ctypes
import os
import re

import pytest

from qevict_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qevict_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(qv_[a-z0-9_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_lists_the_entry_points():
    names = header_functions()
    for must in ("qv_decode_attention", "qv_evict_cycle", "qv_rope_append", "qv_prefill_build",
                 "qv_prefill_attention", "qv_quantize_k", "qv_quantize_v", "qv_dequantize",
                 "qv_decode_attention_noalloc"):
        assert must in names
    assert sorted(N.exported_symbols()) == names


def test_library_exports_every_header_symbol():
    lib = N.lib()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.qv_version().decode()


@pytest.mark.parametrize("local,omega,kw,expect_R", [(512, 64, 32, 9), (128, 64, 3, 3), (256, 32, 0, 9)])
def test_slot_layout_sizes(local, omega, kw, expect_R):
    d = N.QvDims(1, 8, 4, 128, omega, 64, local, kw, 16, 512, 8, N.QV_BF16, 0)
    assert N.lib().qv_ring_windows(ctypes.byref(d)) == expect_R
    assert N.lib().qv_main_capacity(ctypes.byref(d)) == 64 + (kw + expect_R) * omega


def test_invalid_dims_rejected():
    bad = [N.QvDims(1, 8, 4, 96, 64, 64, 512, 32, 32, 512, 8, N.QV_BF16, 0),   # head_dim 96
           N.QvDims(1, 8, 4, 128, 64, 64, 500, 32, 32, 512, 8, N.QV_BF16, 0),  # local not whole windows
           N.QvDims(1, 8, 4, 128, 64, 64, 512, 32, 32, 512, 3, N.QV_BF16, 0),  # 3-bit codes
           N.QvDims(1, 8, 16, 128, 64, 64, 512, 32, 32, 512, 8, N.QV_BF16, 0)]  # group 16
    for d in bad:
        assert N.lib().qv_ring_windows(ctypes.byref(d)) == -1
        assert N.lib().qv_main_capacity(ctypes.byref(d)) == -1


@pytest.mark.parametrize("name,dims,path", [
    # the production layer: bf16 / fp16, head_dim 128, omega 64, INT8, sink a multiple of 64
    ("bf16 int8 omega64", (1, 8, 4, 128, 64, 64, 512, 32, 32, 512, 8, N.QV_BF16, 0), 1),
    ("fp16 int8 omega64 MHA", (16, 32, 1, 128, 64, 64, 512, 8, 64, 512, 8, N.QV_F16, 0), 1),
    # everything else takes the CUDA-core kernel
    ("bf16 INT4", (1, 8, 4, 128, 64, 64, 512, 32, 32, 512, 4, N.QV_BF16, 0), 0),
    ("bf16 omega 16", (1, 8, 4, 128, 16, 64, 512, 32, 32, 512, 8, N.QV_BF16, 0), 0),
    ("bf16 omega 32", (1, 8, 4, 128, 32, 64, 512, 32, 32, 512, 8, N.QV_BF16, 0), 0),
    ("bf16 sink 4", (1, 8, 4, 128, 64, 4, 512, 32, 32, 512, 8, N.QV_BF16, 0), 0),
    ("bf16 head_dim 64", (1, 8, 4, 64, 64, 64, 512, 32, 32, 512, 8, N.QV_BF16, 0), 0),
    ("fp32", (1, 8, 4, 128, 64, 64, 512, 32, 32, 512, 8, N.QV_F32, 0), 0),
    ("bf16 reference rounding", (1, 8, 4, 128, 64, 64, 512, 32, 32, 512, 8, N.QV_BF16,
                                 N.QV_FLAG_REFERENCE_ROUNDING), 0),
])
def test_decode_path_selection(name, dims, path):
    """Which decode-attention kernel each configuration gets (qv_decode_path is host
    arithmetic only): 1 = the tensor-core kernel, 0 = the CUDA-core kernel.  A
    configuration that silently falls back to the slower kernel shows up here."""
    d = N.QvDims(*dims)
    assert N.lib().qv_decode_path(ctypes.byref(d)) == path, name


def test_reference_default_omega_8_rejected():
    """The reference's shipped defaults (src/sticky_config.py: OMEGA 8, SINK_TOKENS 4,
    4-bit codes) are refused: windows must be a multiple of 16 tokens, 16..128
    (every workload of this library uses omega 64)."""
    d = N.QvDims(1, 8, 4, 128, 8, 4, 32, 4, 4, 512, 4, N.QV_BF16, 0)
    assert N.lib().qv_decode_path(ctypes.byref(d)) == -1
    assert N.lib().qv_main_capacity(ctypes.byref(d)) == -1


def _dims(B, H, G, D, dt):
    return N.QvDims(B, H, G, D, 64, 0, 64, 0, 0, 1, 8, dt, 0)


@pytest.mark.parametrize("B,H,G,D,S", [(1, 8, 4, 128, 32768), (2, 2, 1, 64, 1100), (1, 1, 8, 128, 517)])
def test_prefill_workspace_holds_stats_partials_and_error_word(B, H, G, D, S):
    """qv_prefill_workspace_bytes: the per-row statistics, for bf16/fp16 the
    column-sum partials (a triangle of n (n + 1) / 2 rows of QB = 128 / G keys
    per sequence and KV head, n = ceil(S / QB)), and 256 bytes for the error
    word; fp32 (the CUDA-core lane) needs no partials."""
    lib = N.lib()
    al = lambda x: (x + 255) // 256 * 256
    stats = al(B * H * G * S * 2 * 4)
    QB = 128 // G
    n = -(-S // QB)
    partial = al(B * H * (QB * n * (n + 1) // 2) * 4)
    got16 = lib.qv_prefill_workspace_bytes(ctypes.byref(_dims(B, H, G, D, N.QV_BF16)), S)
    got32 = lib.qv_prefill_workspace_bytes(ctypes.byref(_dims(B, H, G, D, N.QV_F32)), S)
    assert got16 == stats + partial + 256
    assert got32 == stats + 256


def test_peer_sum_rejects_bad_arguments_without_a_device():
    """The argument checks of the peer sum run before any CUDA call."""
    lib = N.lib()
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(N.QV_PEER_HANDLE_BYTES)
    for rank, world, mb in ((0, 0, 1024), (2, 2, 1024), (0, 9, 1024), (0, 2, 0), (0, 2, 1000)):
        assert lib.qv_peer_sum_create(rank, world, mb, ctypes.byref(h), buf) == N.QV_EINVAL
    assert lib.qv_peer_sum_bf16(None, None, None, 8, None) == N.QV_EINVAL
    assert lib.qv_peer_max_i64(None, None, None, 1, None) == N.QV_EINVAL
    assert lib.qv_peer_sum_open(None, b"") == N.QV_EINVAL
    assert lib.qv_peer_sum_destroy(None) == N.QV_EINVAL
