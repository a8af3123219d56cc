"""qv_decode_attention_noalloc (scratch in a fixed device array) against qv_decode_attention.

Two layer states built from the same prompt decode the same two tokens in a
row, one through each entry point; outputs and vote ledgers must agree bit for
bit, since both run the same kernels on the same scratch layout.  The file is
named to be collected last, so it also runs after every other GPU test has
used the library.
"""

import ctypes

import pytest
import torch

from qevict_b200 import _native as N
from qevict_b200.layer_state import StickyLayerState

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _pair(dtype, B=2, H=2, G=4, D=128, om=64, sink=64, local=128, kw=3, qw=4, n_windows=10, seed=3):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    S = sink + n_windows * om
    k = torch.randn(B, H, S, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(B, H, S, D, generator=g, device="cuda").to(dtype)
    cs = torch.rand(B, H, S, generator=g, device="cuda") * 4
    states = []
    for _ in range(2):
        st = StickyLayerState(B, H, G, D, om, sink, local, kw, qw, 128, 8, dtype)
        st.prefill(k, v, cs)
        states.append(st)
    return states, g


def _noalloc(st, q_rot, out):
    rc = N.lib().qv_decode_attention_noalloc(ctypes.byref(st.dims), ctypes.byref(st.layer), N.ptr(q_rot),
                                             N.ptr(out), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    N.check(rc, "qv_decode_attention_noalloc")
    st.n_tokens += 1


@pytest.mark.parametrize("dtype,shape", [
    (torch.bfloat16, {}),
    (torch.float32, {}),
    # the largest shape the header names for the 8 MiB scratch: batch 8 at the
    # Llama-3-8B layer shape, 32 sticky + 32 Q windows of 64, local 512
    (torch.bfloat16, dict(B=8, H=8, G=4, local=512, kw=32, qw=32, n_windows=72)),
])
def test_noalloc_matches_workspace_entry_point(dtype, shape):
    (a, b), g = _pair(dtype, **shape)
    assert int(N.lib().qv_decode_workspace_bytes(ctypes.byref(a.dims))) <= N.QV_NOALLOC_SCRATCH_BYTES
    B, HG, D = a.B, a.H * a.G, a.D
    for step in range(2):
        q = torch.randn(B, HG, D, generator=g, device="cuda").to(dtype) * 0.3
        kn = torch.randn(B, a.H, D, generator=g, device="cuda").to(dtype)
        vn = torch.randn(B, a.H, D, generator=g, device="cuda").to(dtype)
        out_a = torch.full((B, HG, D), float("nan"), dtype=dtype, device="cuda")
        out_b = torch.full((B, HG, D), float("nan"), dtype=dtype, device="cuda")
        a.attend(a.append(q, kn, vn), out_a)
        _noalloc(b, b.append(q, kn, vn), out_b)
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b), f"step {step}: outputs differ"
        assert torch.equal(a.votes, b.votes), f"step {step}: vote ledgers differ"
        assert a.read_error() == 0 and b.read_error() == 0


def test_noalloc_rejects_oversize_dims():
    (a, _), _ = _pair(torch.bfloat16)
    big = N.QvDims(*[getattr(a.dims, f) for f, _ in N.QvDims._fields_])
    big.batch = 4096
    need = int(N.lib().qv_decode_workspace_bytes(ctypes.byref(big)))
    assert need > 8 * 1024 * 1024
    out = torch.empty(1, dtype=torch.bfloat16, device="cuda")
    rc = N.lib().qv_decode_attention_noalloc(ctypes.byref(big), ctypes.byref(a.layer), N.ptr(out), N.ptr(out),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == N.QV_ESPACE
    assert b"static scratch" in N.lib().qv_last_cuda_error()
